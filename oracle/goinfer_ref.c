/*
 * goinfer_ref.c -- CPU restatement of go-infer's quantised GEMV path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); the
 * product library never links or calls this file.  See goinfer_ref.h for
 * the floating-point rules (gcc -O2 -ffp-contract=off, float32 rounding
 * after every operation, as Go/amd64 does).
 *
 * Citations are file:line within abmarcum/go-infer.
 */
#include "goinfer_ref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static inline float bits_to_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint32_t f32_to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline uint16_t le16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* pkg/quant/fp16.go:8-35.  uint32 arithmetic wraps exactly as Go's does in
 * the subnormal loop (exp can step below zero before the +112 bias). */
float ref_fp16_to_fp32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (uint32_t)(h & 0x7C00) >> 10;
  uint32_t mant = (uint32_t)(h & 0x03FF);
  uint32_t f;
  if (exp == 0) {
    if (mant == 0) {
      f = sign;
    } else {
      exp = 1;
      while ((mant & 0x0400) == 0) {
        mant <<= 1;
        exp--;
      }
      mant &= 0x03FF;
      f = sign | ((exp + (127 - 15)) << 23) | (mant << 13);
    }
  } else if (exp == 0x1F) {
    f = sign | 0x7F800000u | (mant << 13);
  } else {
    f = sign | ((exp + (127 - 15)) << 23) | (mant << 13);
  }
  return bits_to_f32(f);
}

/* pkg/quant/fp16.go:38-69: truncates the mantissa (mant >> 13). */
uint16_t ref_fp32_to_fp16(float val) {
  uint32_t bits = f32_to_bits(val);
  uint32_t sign = (bits >> 16) & 0x8000;
  int exp = (int)((bits >> 23) & 0xFF);
  uint32_t mant = bits & 0x007FFFFF;
  if (exp == 255) {
    if (mant != 0) return (uint16_t)(sign | 0x7E00);
    return (uint16_t)(sign | 0x7C00);
  }
  exp = exp - 127 + 15;
  if (exp >= 31) return (uint16_t)(sign | 0x7C00);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant = (mant | 0x00800000u) >> (1 - exp);
    return (uint16_t)(sign | (mant >> 13));
  }
  return (uint16_t)(sign | ((uint32_t)exp << 10) | (mant >> 13));
}

/* pkg/quant/quant.go:196-212 */
void ref_dequantize_q8_0(const uint8_t* data, size_t nbytes, float* out, int64_t n) {
  memset(out, 0, (size_t)n * sizeof(float));
  int64_t nblocks = n / 32;
  size_t off = 0;
  int64_t o = 0;
  for (int64_t i = 0; i < nblocks && off + 34 <= nbytes; i++) {
    float d = ref_fp16_to_fp32(le16(data + off));
    off += 2;
    for (int j = 0; j < 32; j++) out[o + j] = (float)(int8_t)data[off + j] * d;
    off += 32;
    o += 32;
  }
}

/* getScaleMin closure of DequantizeQ4_K, pkg/quant/quant.go:228-235 */
static inline void q4k_scale_min(const uint8_t* scales, int j, float d, float dmin,
                                 float* sc, float* m) {
  if (j < 4) {
    *sc = (float)(scales[j] & 63) * d;
    *m = (float)(scales[j + 4] & 63) * dmin;
    return;
  }
  *sc = (float)((scales[j + 4] & 0xF) | ((scales[j - 4] >> 6) << 4)) * d;
  *m = (float)((scales[j + 4] >> 4) | ((scales[j] >> 6) << 4)) * dmin;
}

/* pkg/quant/quant.go:215-253 */
void ref_dequantize_q4_k(const uint8_t* data, size_t nbytes, float* out, int64_t n) {
  memset(out, 0, (size_t)n * sizeof(float));
  int64_t nblocks = n / 256;
  size_t off = 0;
  int64_t o = 0;
  for (int64_t i = 0; i < nblocks && off + 144 <= nbytes; i++) {
    float d = ref_fp16_to_fp32(le16(data + off));
    float dmin = ref_fp16_to_fp32(le16(data + off + 2));
    const uint8_t* scales = data + off + 4;
    const uint8_t* qs = data + off + 16;
    off += 144;
    for (int c = 0; c < 4; c++) {
      float d1, m1, d2, m2;
      q4k_scale_min(scales, 2 * c, d, dmin, &d1, &m1);
      q4k_scale_min(scales, 2 * c + 1, d, dmin, &d2, &m2);
      const uint8_t* q = qs + 32 * c;
      int64_t base = o + 64 * c;
      for (int l = 0; l < 32; l++) {
        uint8_t b = q[l];
        float lo = (float)(b & 0x0F) * d1; /* product rounds, then subtract rounds */
        float hi = (float)(b >> 4) * d2;
        out[base + l] = lo - m1;
        out[base + l + 32] = hi - m2;
      }
    }
    o += 256;
  }
}

/* pkg/quant/quant.go:256-291; products associate as (d * sc) * q. */
void ref_dequantize_q6_k(const uint8_t* data, size_t nbytes, float* out, int64_t n) {
  memset(out, 0, (size_t)n * sizeof(float));
  int64_t nblocks = n / 256;
  size_t off = 0;
  int64_t o = 0;
  for (int64_t i = 0; i < nblocks && off + 210 <= nbytes; i++) {
    const uint8_t* ql = data + off;
    const uint8_t* qh = data + off + 128;
    const uint8_t* sc = data + off + 192;
    float d = ref_fp16_to_fp32(le16(data + off + 208));
    off += 210;
    for (int h = 0; h < 2; h++) {
      const uint8_t* qls = ql + 64 * h;
      const uint8_t* qhs = qh + 32 * h;
      const uint8_t* scs = sc + 8 * h;
      int64_t base = o + 128 * h;
      for (int l = 0; l < 32; l++) {
        int is = l / 16;
        int q1 = (int)((qls[l] & 0x0F) | (((qhs[l] >> 0) & 3) << 4)) - 32;
        int q2 = (int)((qls[l + 32] & 0x0F) | (((qhs[l] >> 2) & 3) << 4)) - 32;
        int q3 = (int)(((qls[l] >> 4) & 0x0F) | (((qhs[l] >> 4) & 3) << 4)) - 32;
        int q4 = (int)(((qls[l + 32] >> 4) & 0x0F) | (((qhs[l] >> 6) & 3) << 4)) - 32;
        float t;
        t = d * (float)(int8_t)scs[is + 0];
        out[base + l + 0] = t * (float)q1;
        t = d * (float)(int8_t)scs[is + 2];
        out[base + l + 32] = t * (float)q2;
        t = d * (float)(int8_t)scs[is + 4];
        out[base + l + 64] = t * (float)q3;
        t = d * (float)(int8_t)scs[is + 6];
        out[base + l + 96] = t * (float)q4;
      }
    }
    o += 256;
  }
}

/* pkg/quant/quant.go:548-566: eight products summed left to right, the
 * group then added to the running sum; scalar tail. */
float ref_dot_vec_f32(const float* x, const float* w, int64_t n) {
  float sum = 0.0f;
  int64_t i = 0;
  for (; i <= n - 8; i += 8) {
    float g = x[i] * w[i];
    g = g + x[i + 1] * w[i + 1];
    g = g + x[i + 2] * w[i + 2];
    g = g + x[i + 3] * w[i + 3];
    g = g + x[i + 4] * w[i + 4];
    g = g + x[i + 5] * w[i + 5];
    g = g + x[i + 6] * w[i + 6];
    g = g + x[i + 7] * w[i + 7];
    sum = sum + g;
  }
  for (; i < n; i++) sum = sum + x[i] * w[i];
  return sum;
}

/* pkg/quant/quant.go:320-339: sequential float32 block sum, then
 * total += blockSum * d. */
float ref_dot_vec_q8_0(const float* x, const uint8_t* raw, int64_t n) {
  int64_t nblocks = n / 32;
  float total = 0.0f;
  for (int64_t b = 0; b < nblocks; b++) {
    const uint8_t* blk = raw + 34 * b;
    float d = ref_fp16_to_fp32(le16(blk));
    const float* xb = x + 32 * b;
    float bs = 0.0f;
    for (int j = 0; j < 32; j++) bs = bs + (float)(int8_t)blk[2 + j] * xb[j];
    total = total + bs * d;
  }
  return total;
}

/* pkg/quant/quant.go:536-539.  The Go code allocates a fresh zeroed
 * []float32 per call (make inside DequantizeQ4_K); calloc mirrors that. */
float ref_dot_vec_q4_k(const float* x, const uint8_t* raw, int64_t n) {
  float* deq = (float*)calloc((size_t)n, sizeof(float));
  ref_dequantize_q4_k(raw, (size_t)(n / 256) * 144, deq, n);
  float s = ref_dot_vec_f32(x, deq, n);
  free(deq);
  return s;
}

/* pkg/quant/quant.go:542-545 */
float ref_dot_vec_q6_k(const float* x, const uint8_t* raw, int64_t n) {
  float* deq = (float*)calloc((size_t)n, sizeof(float));
  ref_dequantize_q6_k(raw, (size_t)(n / 256) * 210, deq, n);
  float s = ref_dot_vec_f32(x, deq, n);
  free(deq);
  return s;
}

/* pkg/quant/quant.go:407-455.  math.Round is round-half-away-from-zero,
 * as roundf is; the clamp comes before the rounding. */
void ref_quantize_q8_0(const float* src, int64_t n, uint8_t* out) {
  int64_t nblocks = (n + 31) / 32;
  memset(out, 0, (size_t)nblocks * 34);
  for (int64_t b = 0; b < nblocks; b++) {
    int64_t start = b * 32, end = start + 32;
    if (end > n) end = n;
    float maxv = 0.0f;
    for (int64_t i = start; i < end; i++) {
      float v = fabsf(src[i]);
      if (v > maxv) maxv = v;
    }
    float scale = maxv / 127.0f;
    uint16_t h = 0;
    if (scale > 0) {
      h = ref_fp32_to_fp16(scale);
      scale = ref_fp16_to_fp32(h);
    }
    float inv = 0.0f;
    if (scale > 0) inv = 1.0f / scale;
    uint8_t* o = out + b * 34;
    o[0] = (uint8_t)(h & 0xFF);
    o[1] = (uint8_t)(h >> 8);
    for (int i = 0; i < 32; i++) {
      int8_t q = 0;
      if (start + i < n && inv > 0) {
        float v = src[start + i] * inv;
        if (v > 127) v = 127;
        else if (v < -128) v = -128;
        q = (int8_t)round((double)v);
      }
      o[2 + i] = (uint8_t)q;
    }
  }
}

int64_t ref_bytes_per_row(int type, int64_t cols) {
  switch (type) {
    case REF_GGML_Q8_0: return (cols / 32) * 34;   /* gemv.go:99 */
    case REF_GGML_Q4_K: return (cols / 256) * 144; /* gemv.go:135 */
    case REF_GGML_Q6_K: return (cols / 256) * 210; /* gemv.go:171 */
    case REF_GGML_F32: return cols * 4;
    default: return -1;
  }
}

typedef struct {
  int type;
  float* y;
  double* y64;
  const float* x;
  const uint8_t* raw;
  int64_t start, end, cols, bpr;
} chunk_t;

static float row_dot(int type, const float* x, const uint8_t* row, int64_t cols) {
  switch (type) {
    case REF_GGML_Q8_0: return ref_dot_vec_q8_0(x, row, cols);
    case REF_GGML_Q4_K: return ref_dot_vec_q4_k(x, row, cols);
    case REF_GGML_Q6_K: return ref_dot_vec_q6_k(x, row, cols);
    default: return ref_dot_vec_f32(x, (const float*)row, cols);
  }
}

static void* chunk_run(void* arg) {
  chunk_t* c = (chunk_t*)arg;
  for (int64_t r = c->start; r < c->end; r++)
    c->y[r] = row_dot(c->type, c->x, c->raw + r * c->bpr, c->cols);
  return NULL;
}

static void deq_row(int type, const uint8_t* row, int64_t cols, int64_t bpr, float* out) {
  switch (type) {
    case REF_GGML_Q8_0: ref_dequantize_q8_0(row, (size_t)bpr, out, cols); break;
    case REF_GGML_Q4_K: ref_dequantize_q4_k(row, (size_t)bpr, out, cols); break;
    case REF_GGML_Q6_K: ref_dequantize_q6_k(row, (size_t)bpr, out, cols); break;
    default: memcpy(out, row, (size_t)cols * 4);
  }
}

static void* chunk_run_f64(void* arg) {
  chunk_t* c = (chunk_t*)arg;
  float* deq = (float*)malloc((size_t)c->cols * sizeof(float));
  for (int64_t r = c->start; r < c->end; r++) {
    deq_row(c->type, c->raw + r * c->bpr, c->cols, c->bpr, deq);
    double s = 0.0;
    for (int64_t k = 0; k < c->cols; k++) s += (double)deq[k] * (double)c->x[k];
    c->y64[r] = s;
  }
  free(deq);
  return NULL;
}

/* Sum over k of |w[r][k] * x[k]| in double, over the reference's float32
 * dequantised rows: the conditioning of each output (a test statistic, not
 * a reference function). */
static void* chunk_run_abs(void* arg) {
  chunk_t* c = (chunk_t*)arg;
  float* deq = (float*)malloc((size_t)c->cols * sizeof(float));
  for (int64_t r = c->start; r < c->end; r++) {
    deq_row(c->type, c->raw + r * c->bpr, c->cols, c->bpr, deq);
    double s = 0.0;
    for (int64_t k = 0; k < c->cols; k++) s += fabs((double)deq[k] * (double)c->x[k]);
    c->y64[r] = s;
  }
  free(deq);
  return NULL;
}

/* The row chunking of pkg/math/gemv.go:134-167 (identical for every type). */
static int run_chunks(int type, float* y, double* y64, const float* x, const uint8_t* raw,
                      int64_t rows, int64_t cols, int nthreads, void* (*fn)(void*)) {
  int64_t bpr = ref_bytes_per_row(type, cols);
  if (bpr < 0) return -2;
  int64_t workers = nthreads;
  if (rows < workers) workers = rows;
  if (workers <= 1) {
    chunk_t c = {type, y, y64, x, raw, 0, rows, cols, bpr};
    fn(&c);
    return 0;
  }
  int64_t chunk = (rows + workers - 1) / workers;
  chunk_t* cs = (chunk_t*)calloc((size_t)workers, sizeof(chunk_t));
  pthread_t* th = (pthread_t*)calloc((size_t)workers, sizeof(pthread_t));
  for (int64_t w = 0; w < workers; w++) {
    int64_t s = w * chunk, e = s + chunk;
    if (e > rows) e = rows;
    if (s > rows) s = rows;
    chunk_t c = {type, y, y64, x, raw, s, e, cols, bpr};
    cs[w] = c;
    pthread_create(&th[w], NULL, fn, &cs[w]);
  }
  for (int64_t w = 0; w < workers; w++) pthread_join(th[w], NULL);
  free(cs);
  free(th);
  return 0;
}

int ref_matmul(int type, float* y, const float* x, const uint8_t* raw, int64_t rows,
               int64_t cols, int nthreads) {
  return run_chunks(type, y, NULL, x, raw, rows, cols, nthreads, chunk_run);
}

int ref_matmul_f64(int type, double* y, const float* x, const uint8_t* raw, int64_t rows,
                   int64_t cols, int nthreads) {
  return run_chunks(type, NULL, y, x, raw, rows, cols, nthreads, chunk_run_f64);
}

int ref_matmul_absdot(int type, double* y, const float* x, const uint8_t* raw, int64_t rows,
                      int64_t cols, int nthreads) {
  return run_chunks(type, NULL, y, x, raw, rows, cols, nthreads, chunk_run_abs);
}

int ref_matmul_batch(int type, float* y, const float* x, const uint8_t* raw, int64_t batch,
                     int64_t rows, int64_t cols, int nthreads) {
  for (int64_t b = 0; b < batch; b++) {
    int rc = ref_matmul(type, y + b * rows, x + b * cols, raw, rows, cols, nthreads);
    if (rc) return rc;
  }
  return 0;
}

/* ---------------------------------------------------------------------------
 * Whole-model decode.  Float32 arithmetic is written one rounding per Go
 * operation (the file is built with -ffp-contract=off, like Go on amd64 which
 * never fuses); Go's float64 math.Sqrt/Pow/Cos/Sin/Exp become libm's double
 * functions (sqrt is correctly rounded in both; the others agree to within an
 * ulp of the double result, which the float32 conversion hides except in
 * rare ties).
 * ------------------------------------------------------------------------- */

void ref_rmsnorm(float* out, const float* x, const float* w, int64_t n, float eps) {
  float sum = 0.0f;
  for (int64_t i = 0; i < n; i++) sum = sum + x[i] * x[i];
  float mean = sum / (float)n;
  float scale = (float)(1.0 / sqrt((double)(mean + eps)));
  for (int64_t i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

void ref_apply_rope(float* vec, int pos, int head_dim, float theta) {
  int half = head_dim / 2;
  for (int i = 0; i < half; i++) {
    double freq = 1.0 / pow((double)theta, (double)(2 * i) / (double)head_dim);
    double val = (double)pos * freq;
    float c = (float)cos(val);
    float sn = (float)sin(val);
    float v0 = vec[i], v1 = vec[i + half];
    vec[i] = v0 * c - v1 * sn;
    vec[i + half] = v0 * sn + v1 * c;
  }
}

void ref_swiglu(float* gate, const float* up, int64_t n) {
  for (int64_t i = 0; i < n; i++) {
    float g = gate[i];
    float silu = g / (1.0f + (float)exp((double)(-g)));
    gate[i] = silu * up[i];
  }
}

void ref_softmax(float* x, int64_t n) {
  if (n == 0) return;
  float maxv = x[0];
  for (int64_t i = 1; i < n; i++)
    if (x[i] > maxv) maxv = x[i];
  float sum = 0.0f;
  for (int64_t i = 0; i < n; i++) {
    float v = (float)exp((double)(x[i] - maxv));
    x[i] = v;
    sum = sum + v;
  }
  if (sum > 0) {
    float inv = 1.0f / sum;
    for (int64_t i = 0; i < n; i++) x[i] = x[i] * inv;
  }
}

double ref_math_sqrt(double x) {
  if (x <= 0) return 0;
  double z = x / 2;
  for (int i = 0; i < 10; i++) z = (z + x / z) / 2;
  return z;
}

int ref_extract_embedding(const ref_mat* tbl, int token, float* out, int dim) {
  int64_t bpr = ref_bytes_per_row(tbl->type, dim);
  if (bpr < 0) return -2;
  deq_row(tbl->type, tbl->raw + (int64_t)token * bpr, dim, bpr, out);
  return 0;
}

int ref_argmax(const float* logits, int64_t n) {
  int64_t best = 0;
  float maxv = logits[0];
  for (int64_t i = 0; i < n; i++)
    if (logits[i] > maxv) {
      maxv = logits[i];
      best = i;
    }
  return (int)best;
}

static int mm(const ref_model* m, const ref_mat* w, float* y, const float* x, int64_t rows, int64_t cols) {
  return ref_matmul(w->type, y, x, w->raw, rows, cols, m->nthreads);
}

int ref_forward(const ref_model* m, float* key, float* value, int token, int pos, float* logits) {
  const int dim = m->dim, hd = dim / m->n_heads;           /* config.go:29-37 */
  const int kv_dim = hd * m->n_kv_heads;                   /* config.go:48-56 */
  const int kv_mul = m->n_heads / m->n_kv_heads;           /* config.go:59-64 */
  const int64_t layer_stride = (int64_t)m->max_seq * kv_dim;
  float* x = (float*)calloc((size_t)dim, 4);
  float* xb = (float*)calloc((size_t)dim, 4);
  float* q = (float*)calloc((size_t)dim, 4);
  float* k = (float*)calloc((size_t)kv_dim, 4);
  float* v = (float*)calloc((size_t)kv_dim, 4);
  float* att = (float*)calloc((size_t)dim, 4);
  float* proj = (float*)calloc((size_t)dim, 4);
  float* gate = (float*)calloc((size_t)m->hidden, 4);
  float* up = (float*)calloc((size_t)m->hidden, 4);
  float* down = (float*)calloc((size_t)dim, 4);
  float* scores = (float*)calloc((size_t)m->max_seq, 4);
  int rc = ref_extract_embedding(&m->tok_embd, token, x, dim);
  int active = pos + 1;
  if (active > m->max_seq) active = m->max_seq;
  const float attn_scale = (float)(1.0 / ref_math_sqrt((double)hd));
  for (int l = 0; l < m->n_layers && rc == 0; l++) {
    const ref_layer* L = &m->layers[l];
    float* kc = key + l * layer_stride;
    float* vc = value + l * layer_stride;
    ref_rmsnorm(xb, x, L->attn_norm, dim, m->eps);
    rc |= mm(m, &L->wq, q, xb, dim, dim);
    rc |= mm(m, &L->wk, k, xb, kv_dim, dim);
    rc |= mm(m, &L->wv, v, xb, kv_dim, dim);
    /* forward.go:211-225: a.Q[i] += b for each bias that is present */
    if (L->bq)
      for (int i = 0; i < dim; i++) q[i] = q[i] + L->bq[i];
    if (L->bk)
      for (int i = 0; i < kv_dim; i++) k[i] = k[i] + L->bk[i];
    if (L->bv)
      for (int i = 0; i < kv_dim; i++) v[i] = v[i] + L->bv[i];
    for (int h = 0; h < m->n_heads; h++) ref_apply_rope(q + h * hd, pos, hd, m->rope_theta);
    for (int h = 0; h < m->n_kv_heads; h++) ref_apply_rope(k + h * hd, pos, hd, m->rope_theta);
    const int slot = pos % m->max_seq;
    memcpy(kc + (int64_t)slot * kv_dim, k, (size_t)kv_dim * 4);
    memcpy(vc + (int64_t)slot * kv_dim, v, (size_t)kv_dim * 4);
    memset(att, 0, (size_t)dim * 4);
    for (int h = 0; h < m->n_heads; h++) {
      const float* qh = q + h * hd;
      const int kvh = h / kv_mul;
      for (int t = 0; t < active; t++)
        scores[t] = ref_dot_vec_f32(qh, kc + (int64_t)t * kv_dim + kvh * hd, hd) * attn_scale;
      ref_softmax(scores, active);
      float* oh = att + h * hd;
      for (int t = 0; t < active; t++) {
        const float* vh = vc + (int64_t)t * kv_dim + kvh * hd;
        const float wt = scores[t];
        for (int d = 0; d < hd; d++) oh[d] = oh[d] + wt * vh[d];
      }
    }
    rc |= mm(m, &L->wo, proj, att, dim, dim);
    for (int i = 0; i < dim; i++) x[i] = x[i] + proj[i];
    ref_rmsnorm(xb, x, L->ffn_norm, dim, m->eps);
    rc |= mm(m, &L->gate, gate, xb, m->hidden, dim);
    rc |= mm(m, &L->up, up, xb, m->hidden, dim);
    ref_swiglu(gate, up, m->hidden);
    rc |= mm(m, &L->down, down, gate, dim, m->hidden);
    for (int i = 0; i < dim; i++) x[i] = x[i] + down[i];
  }
  if (rc == 0) {
    ref_rmsnorm(xb, x, m->out_norm, dim, m->eps);
    rc = mm(m, &m->out, logits, xb, m->vocab, dim);
  }
  free(x); free(xb); free(q); free(k); free(v); free(att); free(proj);
  free(gate); free(up); free(down); free(scores);
  return rc ? -2 : 0;
}
