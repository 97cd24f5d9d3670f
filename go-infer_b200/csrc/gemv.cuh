// gemv.cuh -- decode-time quantised GEMV (y = W x, batch 1) for sm_100a.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tp.cuh"

namespace gi {

// GGML type ids (pkg/gguf/types.go:25-52 of go-infer).
enum : int { kTypeF32 = 0, kTypeQ8_0 = 8, kTypeQ4_K = 12, kTypeQ6_K = 14 };

// Per-device state the kernels share: `error` (host-mapped) is set to 1 when
// a bounded device wait gives up (never expected; the host reports
// GI_ERR_TIMEOUT).
struct GemvScratch {
  int* error = nullptr;
};

// Fusions of the Q4_K GEMV used by the decode step (internal).
enum : int { kXPlain = 0, kXNorm = 1 };              // staged x, or RMSNorm(x) * x2 (weight)
// y = Wx, y += Wx, silu(W0 x) * (W1 x), or (kYPush) Wx pushed as this
// rank's partial into every rank's tensor-parallel exchange region, then
// y += the rank-ordered sum of all ranks' partials (tensor-parallel
// all-reduce fused into the epilogue).
enum : int { kYStore = 0, kYAdd = 1, kYSwiGLU = 2, kYPush = 3 };
struct GemvFuse {
  int xmode = kXPlain;
  const float* x2 = nullptr;
  float eps = 0.f;
  int ymode = kYStore;
  const TpDev* tp = nullptr;  // kYPush
};

struct GemvLaunch {
  int sm_count = 148;
  bool pdl = false;  // programmatic dependent launch (weights must not be
                     // written by the preceding kernel)
  bool q6k_mma = true;  // Q6_K rows of whole 2048-column groups on the int8
                        // tensor cores (gemv.cu, namespace q6m); false: the
                        // CUDA-core kernel
};

// Per-device one-time set-up (kernel attributes); call with the device current.
int gemv_prepare_device();

// Bytes of one row of `cols` weights of `qtype` (gemv.go:99,135,171).
int64_t row_bytes(int qtype, int64_t cols);

// Shape rules: rows >= 1; cols a positive multiple of 256 (Q4_K, Q6_K), 32
// (Q8_0) or 4 (F32 rows); Q4_K cols <= 45056 (activation staging in shared
// memory).
// Returns 0, -2 unsupported type, -4 bad shape, -5 CUDA launch error.
int gemv_check(int qtype, int64_t rows, int64_t cols);

// y[rows] = W[rows x cols] * x[cols]; every pointer is device memory.
// `w_bytes` bounds the weight reads (no access beyond w + w_bytes).
int gemv_launch(int qtype, float* y, const float* x, const void* w, size_t w_bytes,
                int64_t rows, int64_t cols, const GemvScratch& s, const GemvLaunch& L,
                cudaStream_t stream);

// Several matrices of the same type and width against one activation
// vector in one launch (gate and up, or Q, K and V): y[m] = W[m] x for
// m < nmat <= 3.  Q4_K stages x once for all of them.
int gemv_multi_launch(int qtype, int nmat, float* const* y, const float* x, const void* const* w,
                      const size_t* w_bytes, const int64_t* rows, int64_t cols, const GemvScratch& s,
                      const GemvLaunch& L, cudaStream_t stream);

// Q4_K only: gemv_multi_launch with the prologue / epilogue fusions above.
// kYSwiGLU takes nmat == 2 matrices of equal rows (gate, up) and writes the
// SwiGLU product into y[0].
int gemv_q4k_fused(int nmat, float* const* y, const float* x, const void* const* w, const size_t* w_bytes,
                   const int64_t* rows, int64_t cols, const GemvFuse& f, const GemvLaunch& L, cudaStream_t stream);

}  // namespace gi
