// gemm.cuh -- batched prefill Y[batch][rows] = X[batch][cols] W^T over raw
// GGUF blocks (the work of Weights.MatMulBatch, pkg/engine/weights.go:328).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "gemv.cuh"

namespace gi {

int gemm_prepare_device();

// Returns 0, -2 unsupported type, -4 bad shape.
int gemm_check(int qtype, int64_t batch, int64_t rows, int64_t cols);

int gemm_launch(int qtype, float* y, const float* x, const void* w, size_t w_bytes, int64_t batch,
                int64_t rows, int64_t cols, const GemvScratch& s, const GemvLaunch& L,
                cudaStream_t stream);

}  // namespace gi
