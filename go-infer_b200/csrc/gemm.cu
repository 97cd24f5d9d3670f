// gemm.cu -- batched prefill over raw GGUF blocks.
//
// First correct path: one decode GEMV per token, the same per-token
// semantics go-infer's CPU engine uses when MatMulBatch declines
// (pkg/engine/forward.go:482-495).  The tensor-core dequant-GEMM replaces
// it for large batches.
#include "gemm.cuh"

namespace gi {

int gemm_prepare_device() { return 0; }

int gemm_check(int qtype, int64_t batch, int64_t rows, int64_t cols) {
  if (batch < 1) return -4;
  return gemv_check(qtype, rows, cols);
}

int gemm_launch(int qtype, float* y, const float* x, const void* w, size_t w_bytes, int64_t batch,
                int64_t rows, int64_t cols, const GemvScratch& s, const GemvLaunch& L,
                cudaStream_t stream) {
  int rc = gemm_check(qtype, batch, rows, cols);
  if (rc) return rc;
  for (int64_t b = 0; b < batch; ++b) {
    rc = gemv_launch(qtype, y + b * rows, x + b * cols, w, w_bytes, rows, cols, s, L, stream);
    if (rc) return rc;
  }
  return 0;
}

}  // namespace gi
