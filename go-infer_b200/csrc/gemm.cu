// gemm.cu -- batched prefill over raw GGUF blocks: dispatch between the
// tensor-core dequant-GEMM (gemm_tc.cu) and one decode GEMV per token, the
// per-token semantics go-infer's CPU engine uses when MatMulBatch declines
// (pkg/engine/forward.go:482-495).
#include "gemm.cuh"

namespace gi {

int gemm_prepare_device() { return gemm_tc_prepare_device(); }

int gemm_check(int qtype, int64_t batch, int64_t rows, int64_t cols) {
  if (batch < 1) return -4;
  return gemv_check(qtype, rows, cols);
}

size_t gemm_workspace_need(int qtype, int64_t batch, int64_t rows, int64_t cols) {
  return gemm_tc_supported(qtype, batch, rows, cols) ? gemm_tc_workspace(batch, cols) : 0;
}

int gemm_launch(int qtype, float* y, const float* x, const void* w, size_t w_bytes, int64_t batch,
                int64_t rows, int64_t cols, const GemvScratch& s, const GemmWorkspace& ws,
                const GemvLaunch& L, cudaStream_t stream) {
  int rc = gemm_check(qtype, batch, rows, cols);
  if (rc) return rc;
  if (gemm_tc_supported(qtype, batch, rows, cols)) {
    if ((size_t)rows * (size_t)row_bytes(qtype, cols) > w_bytes) return -4;
    return gemm_tc_launch(qtype, y, x, w, batch, rows, cols, ws, s.error, stream);
  }
  for (int64_t b = 0; b < batch; ++b) {
    rc = gemv_launch(qtype, y + b * rows, x + b * cols, w, w_bytes, rows, cols, s, L, stream);
    if (rc) return rc;
  }
  return 0;
}

}  // namespace gi
