// model.cuh -- device-resident Llama decode step (the work of
// Engine.Forward / ForwardSample, pkg/engine/forward.go:14-405) built from
// the quantised GEMVs plus small fused kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "gemv.cuh"
#include "tp.cuh"

namespace gi {

struct LayersPlan;  // layers.cuh

// One weight matrix in device memory: raw GGUF rows (rows = outputs),
// `qtype` a GGML id (F32 rows are float32).
struct MatRef {
  const void* w = nullptr;
  size_t bytes = 0;
  int qtype = -1;
};

struct LayerRef {
  MatRef wq, wk, wv, wo, gate, up, down;
  const float* attn_norm = nullptr;  // dim
  const float* ffn_norm = nullptr;   // dim
  const float* bq = nullptr;         // optional biases (Qwen 2), dim / kv_dim
  const float* bk = nullptr;
  const float* bv = nullptr;
};

struct ModelCfg {
  int n_layers = 0, dim = 0, hidden = 0, n_heads = 0, n_kv_heads = 0, head_dim = 0, vocab = 0;
  int max_seq = 0;   // KV-cache slots (rolling, slot = pos % max_seq)
  int max_pos = 0;   // positions covered by the RoPE table
  float eps = 1e-5f, rope_theta = 10000.f, attn_scale = 0.f;
  // Tensor parallelism (Megatron): n_heads, n_kv_heads, hidden and vocab are
  // this rank's shares; wq/wk/wv/gate/up/output hold its rows, wo/down its
  // columns; the output and down projections are summed across ranks, the
  // argmax compared across the vocabulary slices (vocab_offset = first row).
  int tp_world = 1, tp_rank = 0, vocab_offset = 0;
};

// Position state the captured step reads and advances on the device.
struct StepState {
  uint32_t token;   // input token of the next step
  uint32_t pos;     // its position
  uint32_t slot;    // pos % max_seq
  uint32_t active;  // min(pos + 1, max_seq)
  uint32_t n_out;   // tokens written to the output list so far
  uint32_t pad[3];
};

class DecodeModel {
 public:
  ~DecodeModel();
  // Validates shapes, allocates activations, KV cache and the RoPE table.
  int init(const ModelCfg& cfg, const LayerRef* layers, const MatRef& tok_embd, const float* out_norm,
           const MatRef& out, int sm_count, int* error_word, const TpDev* tp = nullptr);
  // Enqueue one decode step on `s`: embedding of st.token (if `embed`),
  // all layers, final norm, logits and the greedy argmax, which writes the
  // next token into st and tokens_out[st.n_out] and advances the position.
  int enqueue_step(cudaStream_t s, bool embed, bool pdl);
  void reset_cache(cudaStream_t s);
  // Re-point the weights (same shapes) without touching the KV cache.
  void bind(const LayerRef* layers, const MatRef& tok_embd, const float* out_norm, const MatRef& out);
  int project_partial(const MatRef& W, const float* in, int cols, cudaStream_t s, bool pdl);
  // Run the layers of each step as one persistent cooperative kernel
  // (layers.cu) instead of six launches per layer: 0, or -2 when a layer
  // matrix is not Q4_K or biases are present, -4 when its shared-memory
  // layout does not fit, -5 on a CUDA error.  Off by default.
  int set_persistent(bool on);
  bool persistent() const { return plan_ != nullptr; }

  const ModelCfg& cfg() const { return cfg_; }
  float* x() const { return x_; }
  float* logits() const { return logits_; }
  StepState* state() const { return st_; }
  uint32_t* tokens_out() const { return tokens_out_; }
  int max_out() const { return max_out_; }
  size_t device_bytes() const { return dev_bytes_; }

  // The captured step (built on first use, replayed per token).
  cudaGraphExec_t graph = nullptr;
  bool graph_pdl = false;

 private:
  ModelCfg cfg_;
  LayerRef* layers_ = nullptr;
  int n_layers_ = 0;
  MatRef tok_embd_, out_;
  const float* out_norm_ = nullptr;
  GemvScratch scratch_;
  TpDev tp_;
  int sm_count_ = 148;
  float *x_ = nullptr, *xb_ = nullptr, *q_ = nullptr, *k_ = nullptr, *v_ = nullptr, *att_ = nullptr;
  float *proj_ = nullptr, *gate_ = nullptr, *up_ = nullptr, *logits_ = nullptr;
  float *kcache_ = nullptr, *vcache_ = nullptr;
  float* part_ = nullptr;  // attention split partials
  float2* rope_ = nullptr;
  StepState* st_ = nullptr;
  uint32_t* tokens_out_ = nullptr;
  int max_out_ = 0;
  int att_splits_ = 1;
  size_t dev_bytes_ = 0;
  LayersPlan* plan_ = nullptr;
};

// attn_scale of forward.go:33: float32(1 / math_sqrt(headDim)) with the
// 10-step Newton square root of forward.go:771-780.
float attn_scale_for(int head_dim);

// gate[i] = silu(gate[i]) * up[i] for i < n (kernels.go:39-46), on `s`.
cudaError_t swiglu_launch(float* gate, const float* up, int64_t n, cudaStream_t s);
// x[i] += p[i] for i < n (float32 adds, forward.go's residual), on `s`.
cudaError_t add_launch(float* x, const float* p, int64_t n, cudaStream_t s);

}  // namespace gi
