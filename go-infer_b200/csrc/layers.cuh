// layers.cuh -- the persistent decode-layer kernel: every layer of one
// decode step (pkg/engine/forward.go:140-297) in one cooperative launch.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "gemv.cuh"
#include "model.cuh"

namespace gi {

struct LayersPlan;  // device-side phase table and smem layout (layers.cu)

// Everything the kernel reads besides the phase table: the attention
// operands and buffers of DecodeModel, the grid-barrier counter (zeroed
// before each launch) and the error word (mapped host memory).
struct LayersCfg {
  int n_layers = 0;
  const StepState* st = nullptr;
  float *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *part = nullptr;
  float *kcache = nullptr, *vcache = nullptr;
  const float2* rope = nullptr;
  size_t layer_kv = 0;  // floats of one layer's K (or V) cache
  int kv_mul = 1, hd = 0, kv_dim = 0, n_kv_heads = 0, n_heads = 0, splits = 1;
  int hq = 1;  // query heads per attention item (divides kv_mul)
  float scale = 1.f;
  uint32_t max_pos = 0;
  unsigned* bar = nullptr;
  int* error = nullptr;
};

// One Q4_K projection of a layer as the persistent kernel runs it.
struct LayersMat {
  const void* w[3] = {};
  float* y[3] = {};
  int64_t rows[3] = {};
  int nmat = 0;
  GemvFuse fuse;
};

// Builds the phase table of a model whose seven layer matrices are all
// Q4_K (per layer: QKV with the attention RMSNorm, O with the residual add
// or the tensor-parallel push, gate/up with the FFN RMSNorm and SwiGLU, down
// as O) and checks that one layout of shared memory serves every phase.
// Returns 0, -2 (a matrix is not Q4_K, or biases are present), -4 (shape),
// -5 (CUDA).  The plan is released with layers_plan_free.
int layers_plan_build(const LayerRef* layers, int n_layers, const ModelCfg& cfg, float* x, float* q, float* k,
                      float* v, float* att, float* gate, float* up, const TpDev* tp, int sm_count,
                      LayersPlan** out);
void layers_plan_free(LayersPlan* plan);
// Device bytes the plan holds (phase table and barrier counter).
size_t layers_plan_bytes(const LayersPlan* plan);

// Enqueues the layers of one step on `s`: zeroes the barrier counter, then
// one cooperative launch of sm_count CTAs.  The embedding (before) and the
// final norm, output head and argmax (after) stay separate launches.
int layers_enqueue(const LayersPlan* plan, LayersCfg cfg, cudaStream_t s);

// Per-device one-time set-up (kernel attributes).
int layers_prepare_device();

}  // namespace gi
