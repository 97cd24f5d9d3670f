// gemm.cuh -- batched prefill Y[batch][rows] = X[batch][cols] W^T over raw
// GGUF blocks (the work of Weights.MatMulBatch, pkg/engine/weights.go:328).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "gemv.cuh"

namespace gi {

// Batches at least this large take the tensor-core path (Q4_K, Q6_K, Q8_0);
// smaller ones run one decode GEMV per token.
constexpr int64_t kGemmTcMinBatch = 16;

// Device workspace of the tensor-core path: the activations staged as fp16
// hi/lo pairs, the Q4_K sub-block sums and the per-token scales.  Owned by
// the caller; gemm_workspace_need() says how large it must be.
struct GemmWorkspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};

int gemm_prepare_device();

// Returns 0, -2 unsupported type, -4 bad shape.
int gemm_check(int qtype, int64_t batch, int64_t rows, int64_t cols);

// Workspace bytes gemm_launch needs for this call (0 on the per-token path).
size_t gemm_workspace_need(int qtype, int64_t batch, int64_t rows, int64_t cols);

int gemm_launch(int qtype, float* y, const float* x, const void* w, size_t w_bytes, int64_t batch,
                int64_t rows, int64_t cols, const GemvScratch& s, const GemmWorkspace& ws,
                const GemvLaunch& L, cudaStream_t stream);

// ---- the tensor-core path (gemm_tc.cu) ----
bool gemm_tc_supported(int qtype, int64_t batch, int64_t rows, int64_t cols);
size_t gemm_tc_workspace(int64_t batch, int64_t cols);
int gemm_tc_prepare_device();
void gemm_tc_set_pair(bool on);  // CTA pairs (default) or single CTAs
// x 16-byte aligned; Q4_K weights 16-byte aligned, Q6_K and Q8_0 2-byte aligned.
int gemm_tc_launch(int qtype, float* y, const float* x, const void* w, int64_t batch, int64_t rows,
                   int64_t cols, const GemmWorkspace& ws, int* error, cudaStream_t stream);

}  // namespace gi
