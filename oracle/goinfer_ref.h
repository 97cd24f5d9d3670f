/*
 * goinfer_ref.h -- CPU restatement of go-infer's quantised GEMV path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA engine and the timed CPU baseline in bench.py's reference arm.  It
 * is never linked into, loaded by, or called from the product library
 * (go-infer_b200/), and the product never falls back to it.
 *
 * Every function restates one Go function of abmarcum/go-infer (module
 * "go-inference"); the citation in each comment is file:line within that
 * project.  The Go code cannot be compiled here (no Go toolchain), so the
 * restatement is compiled with gcc -O2 -ffp-contract=off: Go on amd64
 * (GOAMD64=v1) rounds every float32 operation individually and does not
 * contract a*b+c into an FMA, and this flag gives C the same semantics.
 *
 * Parity pins: the reference's own known-answer tests for this path
 * (pkg/quant/quant_test.go:10-19, :55-83, :129-143 and
 * pkg/metal/metal_test.go:91-125, :127-164) are re-run against this
 * library by tests/test_oracle.py.
 */
#ifndef GOINFER_REF_H
#define GOINFER_REF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids, pkg/gguf/types.go:25-52 */
#define REF_GGML_F32 0
#define REF_GGML_Q8_0 8
#define REF_GGML_Q4_K 12
#define REF_GGML_Q6_K 14

/* pkg/quant/fp16.go:8-35 */
float ref_fp16_to_fp32(uint16_t h);
/* pkg/quant/fp16.go:38-69 (truncating, not rounding) */
uint16_t ref_fp32_to_fp16(float v);

/* pkg/quant/quant.go:196-212 */
void ref_dequantize_q8_0(const uint8_t* data, size_t nbytes, float* out, int64_t n);
/* pkg/quant/quant.go:215-253 */
void ref_dequantize_q4_k(const uint8_t* data, size_t nbytes, float* out, int64_t n);
/* pkg/quant/quant.go:256-291 */
void ref_dequantize_q6_k(const uint8_t* data, size_t nbytes, float* out, int64_t n);

/* pkg/quant/quant.go:548-566 */
float ref_dot_vec_f32(const float* x, const float* w, int64_t n);
/* pkg/quant/quant.go:320-339 */
float ref_dot_vec_q8_0(const float* x, const uint8_t* raw, int64_t n);
/* pkg/quant/quant.go:536-539 (dequantise into a fresh zeroed buffer, then DotVecF32) */
float ref_dot_vec_q4_k(const float* x, const uint8_t* raw, int64_t n);
/* pkg/quant/quant.go:542-545 */
float ref_dot_vec_q6_k(const float* x, const uint8_t* raw, int64_t n);

/* pkg/quant/quant.go:407-455; out must hold ceil(n/32)*34 bytes */
void ref_quantize_q8_0(const float* src, int64_t n, uint8_t* out);

/* Bytes of one weight row, as pkg/math/gemv.go:99,135,171 compute them. */
int64_t ref_bytes_per_row(int type, int64_t cols);

/*
 * GEMVEngine.MatMul{Q8_0,Q4_K,Q6_K}, pkg/math/gemv.go:98-203: y[r] =
 * DotVec*(x, row r) with rows split into ceil(rows/numWorkers) contiguous
 * chunks, one thread per chunk (numWorkers = min(nthreads, rows); the
 * reference defaults nthreads to runtime.NumCPU(), gemv.go:17-24).
 * Returns 0, or -2 for an unsupported type.
 */
int ref_matmul(int type, float* y, const float* x, const uint8_t* raw,
               int64_t rows, int64_t cols, int nthreads);

/*
 * Conditioning aid (not a reference function): y[r] = sum_k deq[r,k]*x[k]
 * accumulated in double over the reference's own float32 dequantised
 * weights.  Used by tests to separate summation-order noise from real
 * errors near zero outputs.
 */
int ref_matmul_f64(int type, double* y, const float* x, const uint8_t* raw,
                   int64_t rows, int64_t cols, int nthreads);

/*
 * Batched prefill semantics, pkg/engine/forward.go:482-495 with
 * weights.go:328-350 returning false on CPU: the caller loops
 * Weights.MatMul per token, so Y[b, :] = MatMul(W, X[b, :]).
 * Layout as the Metal batched kernels use it (kernels.metal:678):
 * y[b*rows + r], x[b*cols + k].
 */
/* Per row, sum of |w*x| in double (the conditioning of each output). */
int ref_matmul_absdot(int type, double* y, const float* x, const uint8_t* raw, int64_t rows,
                      int64_t cols, int nthreads);
int ref_matmul_batch(int type, float* y, const float* x, const uint8_t* raw,
                     int64_t batch, int64_t rows, int64_t cols, int nthreads);

/* ---- whole-model decode: the CPU branch of Engine.Forward ------------------
 * (pkg/engine/forward.go:14-297 with the Metal paths off), Llama layers only.
 * Weight matrices are raw GGUF rows (rows = output features) of `type`
 * (REF_GGML_F32 rows are float32).  The KV cache is the reference's float32
 * rolling cache (pkg/engine/kvcache.go): key/value[layer][slot][kv_dim],
 * slot = pos % max_seq. */
typedef struct {
  int type;
  const uint8_t* raw;
} ref_mat;

typedef struct {
  ref_mat wq, wk, wv, wo, gate, up, down;
  const float* attn_norm; /* dim */
  const float* ffn_norm;  /* dim */
  /* optional Q, K, V biases (NULL when absent; Qwen 2): dim, kv_dim, kv_dim
   * floats added after the projections (forward.go:211-225) */
  const float* bq;
  const float* bk;
  const float* bv;
} ref_layer;

typedef struct {
  int n_layers, dim, hidden, n_heads, n_kv_heads, vocab, max_seq;
  float eps, rope_theta;
  ref_mat tok_embd;       /* vocab x dim */
  const float* out_norm;  /* dim */
  ref_mat out;            /* vocab x dim */
  const ref_layer* layers;
  int nthreads;           /* GEMV workers, gemv.go:17-24 */
} ref_model;

/* pkg/math/kernels.go:9-19 */
void ref_rmsnorm(float* out, const float* x, const float* w, int64_t n, float eps);
/* pkg/math/kernels.go:22-36 */
void ref_apply_rope(float* vec, int pos, int head_dim, float theta);
/* pkg/math/kernels.go:39-46 */
void ref_swiglu(float* gate, const float* up, int64_t n);
/* pkg/math/kernels.go:49-71 */
void ref_softmax(float* x, int64_t n);
/* forward.go:771-780 (10 Newton steps) */
double ref_math_sqrt(double x);
/* weights.go:132-234 for F32, Q8_0, Q4_K and Q6_K tables */
int ref_extract_embedding(const ref_mat* tbl, int token, float* out, int dim);
/* Engine.Forward: logits[vocab] for `token` at `pos`; key/value caches are
 * n_layers * max_seq * kv_dim floats.  Returns 0, or -2 for an unsupported
 * weight type. */
int ref_forward(const ref_model* m, float* key, float* value, int token, int pos, float* logits);
/* forward.go:397-404: first maximum wins. */
int ref_argmax(const float* logits, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
