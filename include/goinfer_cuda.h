/*
 * goinfer_cuda.h -- C ABI of the B200 (sm_100a) engine for go-infer's
 * quantised matrix-vector hot path.
 *
 * This is the CUDA counterpart of go-infer's GPU plugin seam
 * pkg/metal/metal_bridge.h: the same entry points (gi_cuda_* for metal_*),
 * the same argument meaning (GGML quant type ids, row-major raw GGUF weight
 * blocks with rows = output features, fp32 activations, y[b*rows + r] /
 * x[b*cols + k] for batches) and the same int status convention (0 = ok,
 * negative = failure, which the Go wrapper turns into an error and the
 * engine answers by falling back, pkg/engine/weights.go:251-289).  Every
 * declaration names the reference declaration it replaces
 * (file:line within abmarcum/go-infer).
 *
 * Plain C types only: no CUDA or torch types cross this boundary; streams
 * are passed as void* (a cudaStream_t, NULL = the library's own stream).
 *
 * Threading: one process per GPU.  Calls on one device are serialised by
 * an internal mutex (the pattern of CModelContext, c_bridge_cgo.go:19-82).
 */
#ifndef GOINFER_CUDA_H
#define GOINFER_CUDA_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  -1..-3 keep metal_bridge_darwin.m's meaning (:3349,3361,
 * 3377): unavailable / no buffer, unsupported quant type, buffer failure. */
#define GI_OK 0
#define GI_ERR_UNAVAILABLE (-1)
#define GI_ERR_UNSUPPORTED_TYPE (-2)
#define GI_ERR_BUFFER (-3)
#define GI_ERR_SHAPE (-4)   /* cols not a multiple of the block, size too small, misaligned */
#define GI_ERR_CUDA (-5)    /* CUDA runtime error; text in gi_cuda_last_error() */
#define GI_ERR_TIMEOUT (-6) /* a bounded device-side wait gave up */

/* GGML quant type ids, pkg/gguf/types.go:25-52. */
#define GI_TYPE_F32 0
#define GI_TYPE_Q8_0 8
#define GI_TYPE_Q4_K 12
#define GI_TYPE_Q6_K 14

/* Replaces int metal_init(void), metal_bridge.h:13.  Selects the device in
 * $GOINFER_CUDA_DEVICE, else the calling thread's current CUDA device;
 * idempotent. */
int gi_cuda_init(void);

/* Like gi_cuda_init for an explicit device ordinal (no reference
 * counterpart: Metal has one device). */
int gi_cuda_init_device(int device);

/* Replaces bool metal_is_available(void), metal_bridge.h:16. */
bool gi_cuda_is_available(void);

/* Replace void metal_begin_batch(void) / metal_end_batch(void),
 * metal_bridge.h:19-20: between the two calls the host-pointer entry points
 * enqueue without waiting; their outputs reach the host buffers at
 * end_batch, in call order.  As with Metal's shared memory, a call inside
 * the batch that reads a host slice an earlier call of the batch wrote sees
 * that result (it is read from the device; a slice that straddles several
 * outputs is first written back). */
void gi_cuda_begin_batch(void);
void gi_cuda_end_batch(void);

/* Replaces metal_buffer_t / metal_create_buffer(const void*, size_t),
 * metal_bridge.h:44-45.  Copies `bytes` host bytes into device memory once
 * (Metal wraps unified memory without a copy); the handle stays valid
 * until gi_cuda_release_buffer.  NULL on failure. */
typedef void* gi_cuda_buffer_t;
gi_cuda_buffer_t gi_cuda_create_buffer(const void* ptr, size_t bytes);

/* Replaces void metal_release_buffer(metal_buffer_t), metal_bridge.h:46. */
void gi_cuda_release_buffer(gi_cuda_buffer_t buf);

/* Replaces int metal_gemv_buf(int quant_type, float* y, const float* x,
 * metal_buffer_t w_buf, uint32_t rows, uint32_t cols), metal_bridge.h:49:
 * y[rows] = W x with host y/x and a device-resident weight buffer.
 * quant_type: GI_TYPE_Q8_0, GI_TYPE_Q4_K or GI_TYPE_Q6_K. */
int gi_cuda_gemv_buf(int quant_type, float* y, const float* x, gi_cuda_buffer_t w_buf,
                     uint32_t rows, uint32_t cols);

/* Replaces int metal_gemm_buf(int quant_type, float* y, const float* x,
 * metal_buffer_t w_buf, uint32_t batch_size, uint32_t rows, uint32_t cols),
 * metal_bridge.h:50: Y[batch][rows] = X[batch][cols] W^T (prefill). */
int gi_cuda_gemm_buf(int quant_type, float* y, const float* x, gi_cuda_buffer_t w_buf,
                     uint32_t batch_size, uint32_t rows, uint32_t cols);

/* Replaces int metal_gemm_fused_gate_up_buf(int quant_type, float* y,
 * const float* x, metal_buffer_t gate_buf, metal_buffer_t up_buf,
 * uint32_t batch_size, uint32_t rows, uint32_t cols), metal_bridge.h:51:
 * Y[b][r] = silu(G x_b)[r] * (U x_b)[r] (SwiGLU of kernels.go:39-46) with
 * host y/x and device-resident gate/up buffers of rows x cols.  Q4_K only,
 * as the reference (-2 for other types, metal_bridge_darwin.m:3547); -1
 * for a null buffer. */
int gi_cuda_gemm_fused_gate_up_buf(int quant_type, float* y, const float* x, gi_cuda_buffer_t gate_buf,
                                   gi_cuda_buffer_t up_buf, uint32_t batch_size, uint32_t rows,
                                   uint32_t cols);

/* Replaces int metal_add_residual(float* x, const float* proj, uint32_t dim),
 * metal_bridge.h:199: x[i] += proj[i] for i < dim (float32 adds).  The
 * engine calls it on outputs of the same batch without checking the status
 * (pkg/engine/forward.go:590, 639), so it honours the batch order above. */
int gi_cuda_add_residual(float* x, const float* proj, uint32_t dim);

/* Replaces int metal_swiglu(float* gate, const float* up, uint32_t hidden_dim),
 * metal_bridge.h:198: gate[i] = silu(gate[i]) * up[i] with kernels.go:39-46's
 * roundings (float64 exp); batch order as above (forward.go:624). */
int gi_cuda_swiglu(float* gate, const float* up, uint32_t hidden_dim);

/* Replace metal_gemv_q8_0 / metal_gemv_q4_k / metal_gemv_q6_k,
 * metal_bridge.h:181-183: host y, x and host weight bytes (copied per call). */
int gi_cuda_gemv_q8_0(float* y, const float* x, const void* w, uint32_t rows, uint32_t cols);
int gi_cuda_gemv_q4_k(float* y, const float* x, const void* w, uint32_t rows, uint32_t cols);
int gi_cuda_gemv_q6_k(float* y, const float* x, const void* w, uint32_t rows, uint32_t cols);

/* Replace metal_gemm_q8_0 / metal_gemm_q4_k / metal_gemm_q6_k,
 * metal_bridge.h:187-189. */
int gi_cuda_gemm_q8_0(float* y, const float* x, const void* w, uint32_t batch_size, uint32_t rows,
                      uint32_t cols);
int gi_cuda_gemm_q4_k(float* y, const float* x, const void* w, uint32_t batch_size, uint32_t rows,
                      uint32_t cols);
int gi_cuda_gemm_q6_k(float* y, const float* x, const void* w, uint32_t batch_size, uint32_t rows,
                      uint32_t cols);

/* ---- Device-pointer entry points (the measured path; no reference
 * counterpart, Metal's buffers are host-visible).  y, x and w are device
 * pointers; x 16-byte aligned, Q4_K weights 16-byte aligned; w_bytes bounds
 * every weight read.  Asynchronous on `stream` (NULL = library stream). */
int gi_cuda_gemv_dev(int quant_type, float* y, const float* x, const void* w, size_t w_bytes,
                     uint32_t rows, uint32_t cols, void* stream);
int gi_cuda_gemm_dev(int quant_type, float* y, const float* x, const void* w, size_t w_bytes,
                     uint32_t batch_size, uint32_t rows, uint32_t cols, void* stream);

/* gi_cuda_gemm_dev without any allocation (no counterpart in the reference).
 * The prefill workspace is a fixed 16 MiB device array inside the library
 * instead of memory grown at call time, so a call never allocates or
 * synchronises the device.  Limit: the staged activations of the call must
 * fit: about 4.1 bytes per column per token, tokens rounded up to a
 * multiple of 128; 512 tokens x 4096 columns fit.  Larger calls return
 * GI_ERR_SHAPE (batches under 16 need no scratch).  The first call on a device looks up the array's
 * address (make it before any stream capture); the array is shared by all
 * calls on the device, so calls that overlap in time race on it. */
int gi_cuda_gemm_dev_noalloc(int quant_type, float* y, const float* x, const void* w, size_t w_bytes,
                             uint32_t batch_size, uint32_t rows, uint32_t cols, void* stream);

/* Up to 3 matrices of one type and width against one activation vector in
 * one launch: y[m] = W[m] x for m < nmat (Q, K and V of a layer, or gate
 * and up).  The decode counterpart of the fused gate/up entry point
 * metal_gemm_fused_gate_up_buf (metal_bridge.h:51); Q4_K stages x once for
 * all matrices.  Device pointers; arrays of nmat entries. */
int gi_cuda_gemv_multi_dev(int quant_type, int nmat, float* const* y, const float* x,
                           const void* const* w, const size_t* w_bytes, const uint32_t* rows,
                           uint32_t cols, void* stream);

/* The feed-forward half of one decode layer on this rank's shard of it, in
 * two launches: x += W_down SwiGLU(W_gate n, W_up n), n = RMSNorm(x) * norm
 * -- the steps of Engine.Forward at pkg/engine/forward.go:275-287 (rmsnorm,
 * the gate and up MatMuls, SwiGLU, the down MatMul, the residual add), which
 * the reference makes as separate calls (no single counterpart).  Q4_K
 * weights; dim and hidden multiples of 256.  After gi_cuda_tp_connect the
 * caller holds rows [h0, h0 + hidden) of gate and up and the same columns of
 * down (Megatron: column split, then row split), and the down launch sums
 * the ranks' partials in its epilogue, so every rank ends with the same x.
 * _dev: device pointers, h = `hidden` floats of scratch; _buf: x in host
 * memory (copied in and back), weights and the norm as buffers, blocking and
 * not allowed inside a batch (-4). */
int gi_cuda_ffn_dev(float* x, const float* norm, const void* gate, const void* up, const void* down,
                    size_t gate_bytes, size_t up_bytes, size_t down_bytes, float* h, uint32_t dim,
                    uint32_t hidden, float eps, void* stream);
int gi_cuda_ffn_buf(float* x, gi_cuda_buffer_t norm, gi_cuda_buffer_t gate, gi_cuda_buffer_t up,
                    gi_cuda_buffer_t down, uint32_t dim, uint32_t hidden, float eps);

/* ---- whole-model decode (Llama layers) ---------------------------------- */

/* Replaces int metal_alloc_buffers(uint32_t dim, uint32_t hidden_dim,
 * uint32_t kv_dim, uint32_t vocab_size, uint32_t num_layers, uint32_t
 * max_seq), metal_bridge.h:23: records the sizes of the persistent
 * activation and KV-cache buffers of gi_cuda_forward_transformer (allocated
 * at its first call, when the head layout is known).  Releases the previous
 * ones; the KV cache starts at zero. */
int gi_cuda_alloc_buffers(uint32_t dim, uint32_t hidden_dim, uint32_t kv_dim, uint32_t vocab_size,
                          uint32_t num_layers, uint32_t max_seq);

/* Replaces metal_layer_weights_t, metal_bridge.h:54-67.  Matrices are
 * buffers of raw GGUF rows with their GGML type; attn_norm / ffn_norm are
 * float32 buffers of dim values; bq / bk / bv are optional float32 biases
 * (NULL for Llama). */
typedef struct {
  gi_cuda_buffer_t wq;
  int wq_type;
  gi_cuda_buffer_t wk;
  int wk_type;
  gi_cuda_buffer_t wv;
  int wv_type;
  gi_cuda_buffer_t wo;
  int wo_type;
  gi_cuda_buffer_t ffn_gate;
  int ffn_gate_type;
  gi_cuda_buffer_t ffn_up;
  int ffn_up_type;
  gi_cuda_buffer_t ffn_down;
  int ffn_down_type;
  gi_cuda_buffer_t attn_norm;
  gi_cuda_buffer_t ffn_norm;
  gi_cuda_buffer_t bq;
  gi_cuda_buffer_t bk;
  gi_cuda_buffer_t bv;
} gi_cuda_layer_weights_t;

/* Replaces int metal_forward_transformer(...), metal_bridge.h:134-157: one
 * decode step over all layers with device-resident activations and KV cache
 * (the work of Engine.Forward, pkg/engine/forward.go:102-130).  initial_x:
 * host float32[dim], the embedding the caller extracted; out_logits (host
 * float32[vocab_size]) and out_token (first maximum) may each be NULL.
 * Blocks until the results are on the host. */
int gi_cuda_forward_transformer(const float* initial_x, float* out_logits, uint32_t* out_token,
                                const gi_cuda_layer_weights_t* layers, gi_cuda_buffer_t output_norm_buf,
                                gi_cuda_buffer_t output_weight_buf, int output_weight_type, uint32_t num_layers,
                                uint32_t dim, uint32_t hidden_dim, uint32_t kv_dim, uint32_t vocab_size,
                                uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim, uint32_t pos,
                                uint32_t slot, uint32_t max_seq, uint32_t active_context, float norm_eps,
                                float rope_theta, float attn_scale);

/* Device-resident greedy generation (no reference counterpart: the
 * engine's greedy loop, pkg/engine/engine.go:505-545, with the embedding
 * lookup, the argmax and the position advance on the device and each token
 * one CUDA-graph replay).  The model keeps its own KV cache. */
typedef struct {
  uint32_t num_layers, dim, hidden_dim, num_heads, num_kv_heads, head_dim, vocab_size;
  uint32_t max_seq; /* KV-cache slots (rolling) */
  uint32_t max_pos; /* positions the RoPE table covers; 0 = 32768 */
  float norm_eps, rope_theta;
  const gi_cuda_layer_weights_t* layers; /* num_layers entries */
  gi_cuda_buffer_t token_embd;           /* vocab_size rows of dim */
  int token_embd_type;
  gi_cuda_buffer_t output_norm;
  gi_cuda_buffer_t output_weight;
  int output_weight_type;
  /* Tensor parallelism (0 or 1 = off): this process is rank tp_rank of
   * tp_world (gi_cuda_tp_connect first).  num_heads, num_kv_heads,
   * hidden_dim and vocab_size are then this rank's shares and the weight
   * buffers its shards: rows of wq/wk/wv/ffn_gate/ffn_up/output, columns of
   * wo/ffn_down; vocab_offset is the first output row it holds. */
  uint32_t tp_world, tp_rank, vocab_offset;
} gi_cuda_model_desc_t;

typedef void* gi_cuda_model_t;

/* NULL on failure (text in gi_cuda_last_error). */
gi_cuda_model_t gi_cuda_model_create(const gi_cuda_model_desc_t* desc);
void gi_cuda_model_destroy(gi_cuda_model_t model);

/* Zeroes the KV cache. */
int gi_cuda_model_reset(gi_cuda_model_t model);

/* Runs the layers of each decode step as one persistent cooperative kernel
 * (one CTA per SM; the phases of every layer separated by grid-wide
 * barriers, each projection's first weights requested before the barrier
 * in front of it) instead of six launches per layer; enable = 0 returns to
 * the per-layer launches.  No reference counterpart: the reference runs a
 * step as separate Metal dispatches.  The arithmetic is the per-layer
 * kernels' own.  Needs every layer matrix in Q4_K and no biases, else
 * GI_ERR_UNSUPPORTED_TYPE (-2); off by default.  The step is captured again
 * at the next gi_cuda_model_generate. */
int gi_cuda_model_set_persistent(gi_cuda_model_t model, int enable);

/* Runs tokens[0..n_tokens) at positions start_pos.. (one step each), then
 * greedy steps: out_tokens[0..n_gen) are the argmax after the last prompt
 * token and after each generated token (n_gen >= 1).  out_logits (host
 * float32[vocab_size] or NULL) receives the logits of the last step;
 * decode_ms (or NULL) the device time of the n_gen - 1 generation steps. */
int gi_cuda_model_generate(gi_cuda_model_t model, const int32_t* tokens, uint32_t n_tokens, uint32_t start_pos,
                           uint32_t n_gen, uint32_t* out_tokens, float* out_logits, float* decode_ms);

/* ---- tensor parallelism across the GPUs of one node -------------------------
 * The device-side counterpart of TPCoordinator (pkg/distributed/
 * tensor_parallel.go:13-31, AllReduce :33-108): instead of HTTP peers, each
 * rank allocates an exchange region in its own HBM that every peer writes over
 * NVLink.  1) gi_cuda_tp_prepare allocates it and returns its CUDA IPC handle
 * (64 bytes) for the caller to share (e.g. an all-gather over
 * torch.distributed); 2) gi_cuda_tp_connect maps every peer's region
 * (handles[r * 64 ...] is rank r's); then models created with tp_world > 1
 * sum their row-split projections across the ranks. */
int gi_cuda_tp_prepare(int world, uint32_t max_dim, void* handle_out);
int gi_cuda_tp_connect(int rank, int world, const void* handles);
/* Unmaps the peers and frees the region (no model may use it any more). */
int gi_cuda_tp_close(void);

/* Device address / size of a buffer created by gi_cuda_create_buffer. */
const void* gi_cuda_buffer_device_ptr(gi_cuda_buffer_t buf);
size_t gi_cuda_buffer_bytes(gi_cuda_buffer_t buf);

/* Launch kernels with programmatic dependent launch (1) or plainly (0,
 * default).  With it on, a GEMV starts streaming its weights while the
 * previous kernel on the stream drains; weights must then not be written by
 * the kernel just before. */
int gi_cuda_set_pdl(int enable);

/* Q6_K GEMVs of rows of whole 2048-column groups on the int8 tensor cores
 * (1, default) or on the CUDA cores (0) -- no reference counterpart: a
 * choice between two kernels of this library.  Same results within the
 * GEMV tolerance; on B200 the tensor-core kernel streams the 32000 x 4096
 * and 128256 x 8192 heads about 30 % faster. */
int gi_cuda_set_q6k_mma(int enable);

/* Batched (prefill) GEMMs on single CTAs (0, default) or on CTA pairs (1:
 * clusters of two CTAs, 256-row cta_group::2 tcgen05 MMAs, each CTA loading
 * half of the activation tile) -- no reference counterpart: a choice between
 * two launch shapes of this library's tensor-core GEMM, with bit-identical
 * results.  On B200 the pairs are slower at the config-3 shapes (the
 * cross-CTA hand-off of the decoded weight tiles outlasts the 4-stage
 * pipeline), so single CTAs stay the default. */
int gi_cuda_set_prefill_pair(int enable);

/* Text of the last failure on the calling thread ("" if none). */
const char* gi_cuda_last_error(void);

/* Bytes of one weight row, pkg/math/gemv.go:99,135,171; -1 for an
 * unsupported type. */
int64_t gi_quant_row_bytes(int quant_type, int64_t cols);

/* Host quantiser (the counterpart of cmd/quantize/main.go:52-158): rows x
 * cols fp32 -> GGUF blocks in dst (rows * gi_quant_row_bytes bytes).
 * GI_TYPE_Q8_0 is go-infer's QuantizeQ8_0 (pkg/quant/quant.go:407-455);
 * GI_TYPE_Q4_K / GI_TYPE_Q6_K are this library's own fits (go-infer has no
 * K-quant quantiser).  threads <= 0 uses every host core. */
int gi_quantize(int quant_type, const float* src, int64_t rows, int64_t cols, void* dst,
                int threads);

/* Synthetic weights for the benchmark configurations (no reference
 * counterpart): rows [row0, row0 + rows) x columns [col0, col0 + cols) of a
 * matrix drawn from N(0, stddev) by a generator keyed by (seed, row,
 * 256-column block), quantised like gi_quantize (GI_TYPE_F32 stores the
 * float32 values).  col0 is a multiple of 256, so a tensor-parallel shard is
 * generated on its own; the bytes do not depend on `threads` (<= 0: every
 * core). */
int gi_quantize_seeded(int quant_type, uint64_t seed, float stddev, int64_t row0, int64_t rows, int64_t col0,
                       int64_t cols, void* dst, int threads);

/* Copies the first `bytes` of a buffer to host memory (no reference
 * counterpart). */
int gi_cuda_buffer_read(gi_cuda_buffer_t buf, void* dst, size_t bytes);

/* A device buffer of `bytes` without host contents (no reference
 * counterpart); release with gi_cuda_release_buffer.  NULL on failure. */
gi_cuda_buffer_t gi_cuda_alloc_buffer(size_t bytes);

/* Fills `buf` with the synthetic matrix slice of gi_quantize_seeded drawn on
 * the device (the same (seed, row, 256-column block) streams, a float32
 * Box-Muller transform, the same block quantisers; cols a multiple of 256).
 * Deterministic on a given GPU, not bit-identical to gi_quantize_seeded.
 * Returns when the buffer is written. */
int gi_synth_weights(gi_cuda_buffer_t buf, int quant_type, uint64_t seed, float stddev, int64_t row0, int64_t rows,
                     int64_t col0, int64_t cols);

#ifdef __cplusplus
}
#endif
#endif /* GOINFER_CUDA_H */
