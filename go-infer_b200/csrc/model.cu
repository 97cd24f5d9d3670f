// model.cu -- device-resident Llama decode step: the CPU branch of
// Engine.Forward (pkg/engine/forward.go:140-297) and the greedy pick of
// ForwardSample (forward.go:394-405), on the device, one token per call of
// enqueue_step (captured once into a CUDA graph and replayed per token).
//
// The element-wise kernels repeat the reference's float32 operation order
// (one rounding per Go operation, __f*_rn so nothing is contracted into an
// FMA) and its float64 detours (sqrt in RMSNorm, exp in SwiGLU/softmax, the
// RoPE angles, precomputed on the host in double).  Reductions that the
// reference does sequentially (the RMSNorm sum of squares, softmax sums, the
// attention weighted sum) are parallel here: they differ from the
// reference by float32 rounding only, as the GEMVs do.
#include <cmath>
#include <cstring>
#include <vector>

#include "attn.cuh"
#include "common.cuh"
#include "layers.cuh"
#include "model.cuh"

namespace gi {
namespace {

// Launch with programmatic dependent launch when `pdl` (every kernel here
// waits for its predecessor before touching its outputs).
template <typename... KArgs, typename... Args>
cudaError_t launch(bool pdl, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void (*k)(KArgs...),
                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

GI_DEVINL float f16_bits_to_f32(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// ---- embedding: one row of the token table (weights.go:132-234) ----------
// Q4_K: float32(q)*d1 - m1 with d1 = sc*d, m1 = m*dmin (quant.go:228-248);
// Q6_K: d * float32(sc) * float32(q) (quant.go:277-282); Q8_0:
// float32(q) * d (quant.go:205-207); F32: a copy.
__global__ void embed_kernel(const StepState* __restrict__ st, const uint8_t* __restrict__ tbl, int qtype,
                             int dim, size_t rowb, float* __restrict__ x) {
  griddep_wait();
  griddep_launch_dependents();
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= dim) return;
  const uint8_t* row = tbl + (size_t)st->token * rowb;
  float out;
  if (qtype == kTypeQ4_K) {
    const uint8_t* b = row + (size_t)(e >> 8) * 144;
    const int r = e & 255, c = r >> 6, l = r & 63;
    const int j = 2 * c + (l >> 5);
    const uint8_t* sc = b + 4;
    const float d = f16_bits_to_f32(b[0] | (b[1] << 8)), dmin = f16_bits_to_f32(b[2] | (b[3] << 8));
    uint32_t s6, m6;
    if (j < 4) {
      s6 = sc[j] & 63;
      m6 = sc[j + 4] & 63;
    } else {
      s6 = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
      m6 = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    const uint8_t qb = b[16 + 32 * c + (l & 31)];
    const uint32_t q = l < 32 ? (qb & 0xF) : (qb >> 4);
    const float d1 = __fmul_rn((float)s6, d), m1 = __fmul_rn((float)m6, dmin);
    out = __fsub_rn(__fmul_rn((float)q, d1), m1);
  } else if (qtype == kTypeQ6_K) {
    const uint8_t* b = row + (size_t)(e >> 8) * 210;
    const int r = e & 255, n = r >> 7, g = (r >> 5) & 3, l = r & 31;
    const uint8_t qlb = b[n * 64 + (g & 1) * 32 + l];
    const uint32_t lo = (g >> 1) ? (qlb >> 4) : (qlb & 0xF);
    const uint32_t hi = (b[128 + n * 32 + l] >> (2 * g)) & 3;
    const int q = (int)(lo | (hi << 4)) - 32;
    const float sc = (float)(int8_t)b[192 + n * 8 + 2 * g + (l >> 4)];
    const float d = f16_bits_to_f32(b[208] | (b[209] << 8));
    out = __fmul_rn(__fmul_rn(d, sc), (float)q);
  } else if (qtype == kTypeQ8_0) {
    const uint8_t* b = row + (size_t)(e >> 5) * 34;
    out = __fmul_rn((float)(int8_t)b[2 + (e & 31)], f16_bits_to_f32(b[0] | (b[1] << 8)));
  } else {
    out = reinterpret_cast<const float*>(row)[e];
  }
  x[e] = out;
}

// ---- RMSNorm (pkg/math/kernels.go:9-19) ------------------------------------
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                       float* __restrict__ out, int n, float eps) {
  __shared__ float red[32];
  griddep_wait();
  griddep_launch_dependents();
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float mean = __fdiv_rn(red[0], (float)n);
  const float scale = (float)(1.0 / sqrt((double)__fadd_rn(mean, eps)));
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], scale), w[i]);
}

// ---- biases (forward.go:207-223) --------------------------------------------
__global__ void add_kernel(float* __restrict__ y, const float* __restrict__ b, int n) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __fadd_rn(y[i], b[i]);
}

// ---- attention (attn.cuh): one CTA per work item ----------------------------
__global__ void __launch_bounds__(256) attn_partial_kernel(const StepState* __restrict__ st,
                                                           const float* __restrict__ q, const float* __restrict__ k,
                                                           const float* __restrict__ v,
                                                           const float2* __restrict__ rope, float* __restrict__ kc,
                                                           float* __restrict__ vc, float* __restrict__ part,
                                                           int kv_mul, int hd, int kv_dim, int splits, float scale,
                                                           uint32_t max_pos, int* error, int hq) {
  extern __shared__ __align__(16) float sm[];
  griddep_wait();
  griddep_launch_dependents();
  const int ng = kv_mul / hq;  // head groups per kv head: blockIdx.x = g * ng + hg
  attn_partial_item(st, q, k, v, rope, kc, vc, part, kv_mul, hd, kv_dim, splits, scale, max_pos, error,
                    blockIdx.x / ng, blockIdx.y, blockIdx.x % ng, hq, sm);
}

__global__ void attn_combine_kernel(const float* __restrict__ part, float* __restrict__ att, int hd, int splits) {
  griddep_wait();
  griddep_launch_dependents();
  attn_combine_one(part, att, hd, splits, blockIdx.x, threadIdx.x);
}

// ---- residual add (forward.go:271-273, 285-287) ------------------------------
__global__ void residual_kernel(float* __restrict__ x, const float* __restrict__ p, int n) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __fadd_rn(x[i], p[i]);
}

// ---- SwiGLU (kernels.go:39-46) ---------------------------------------------
__global__ void swiglu_kernel(float* __restrict__ gate, const float* __restrict__ up, int n) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float g = gate[i];
  const float silu = __fdiv_rn(g, __fadd_rn(1.0f, (float)exp(-(double)g)));
  gate[i] = __fmul_rn(silu, up[i]);
}

}  // namespace

cudaError_t swiglu_launch(float* gate, const float* up, int64_t n, cudaStream_t s) {
  if (n <= 0 || n > INT32_MAX) return cudaErrorInvalidValue;
  return launch(false, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, swiglu_kernel, gate, up, (int)n);
}

cudaError_t add_launch(float* x, const float* p, int64_t n, cudaStream_t s) {
  if (n <= 0 || n > INT32_MAX) return cudaErrorInvalidValue;
  return launch(false, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, add_kernel, x, p, (int)n);
}

namespace {

// ---- tensor-parallel exchange (TPCoordinator.AllReduce,
// pkg/distributed/tensor_parallel.go:33-108) --------------------------------
GI_DEVINL bool wait_flag(const uint32_t* f, uint32_t want, const int* error) {
  return tp_wait_flag(f, want, error);
}

// Push this rank's partial p[n] into slot `rank` of every rank's region and
// publish it (used when the projection is not the Q4_K GEMV, which pushes
// from its own epilogue).
__global__ void __launch_bounds__(1024) tp_push_kernel(const float* __restrict__ p, int n, TpDev tp) {
  griddep_wait();
  griddep_launch_dependents();
  const uint32_t seq = *tp.seq;
  const size_t base = ((size_t)(seq & 1u) * tp.world + tp.rank) * tp.max_dim;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = p[i];
    for (int r = 0; r < tp.world; ++r) tp.recv[r][base + i] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const size_t f = (size_t)(seq & 1u) * tp.world + tp.rank;
    for (int r = 0; r < tp.world; ++r)
      asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(tp.flags[r] + f), "r"(seq) : "memory");
  }
}

// x += sum of the ranks' partials, in rank order (the same x on every rank),
// once every rank's push of this exchange has landed; then seq += 1.  Each
// CTA waits for the flags and sums its slice of x; the last CTA to finish
// advances seq (no CTA reads seq after that: each read it at its start).
constexpr int kReduceCtas = 32, kReduceThreads = 256;
__global__ void __launch_bounds__(kReduceThreads) tp_reduce_kernel(float* __restrict__ x, int n, TpDev tp,
                                                                   int* error) {
  __shared__ int ok;
  griddep_wait();
  griddep_launch_dependents();
  const uint32_t seq = *tp.seq;
  const uint32_t set = seq & 1u;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < tp.world && !wait_flag(tp.flags[tp.rank] + (size_t)set * tp.world + threadIdx.x, seq, error)) {
    ok = 0;
    atomicExch(error, 1);
  }
  __syncthreads();
  const float* rv = tp.recv[tp.rank] + (size_t)set * tp.world * tp.max_dim;
  const int i0 = (int)((long long)n * blockIdx.x / gridDim.x), i1 = (int)((long long)n * (blockIdx.x + 1) / gridDim.x);
  if (ok)
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
      float v[kTpMaxWorld];
#pragma unroll
      for (int r = 0; r < kTpMaxWorld; ++r) v[r] = r < tp.world ? __ldcg(rv + (size_t)r * tp.max_dim + i) : 0.f;
      float s = v[0];
#pragma unroll
      for (int r = 1; r < kTpMaxWorld; ++r)
        if (r < tp.world) s = __fadd_rn(s, v[r]);
      x[i] = __fadd_rn(x[i], s);
    }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(tp.rdone, 1u) == gridDim.x - 1) {
    *tp.rdone = 0u;
    *tp.seq = seq + 1;
  }
}

// ---- greedy pick (forward.go:397-404: the first maximum wins) and the
// position advance of the generation loop ------------------------------------
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int n, StepState* st,
                                                      uint32_t* __restrict__ out, int max_out, int max_seq,
                                                      int vocab_offset, TpDev tp, int* error) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  griddep_wait();
  griddep_launch_dependents();
  float v = -INFINITY;
  int idx = 0x7fffffff;
  auto consider = [&](float l, int i) {  // i increases along each thread's walk
    if (idx == 0x7fffffff || l > v) {    // strictly greater: the first maximum stays
      v = l;
      idx = i;
    }
  };
  // 16-byte loads, 8 in flight per thread (the logits sit in L2, written by
  // the head GEMV just before), then the scalar tail.
  constexpr int U = 8;
  const int n4 = n >> 2;
  const float4* l4 = reinterpret_cast<const float4*>(logits);
  for (int base = threadIdx.x; base < n4; base += U * blockDim.x) {
    float4 q[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = base + u * blockDim.x;
      q[u] = j < n4 ? l4[j] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = base + u * blockDim.x;
      if (j < n4) {
        consider(q[u].x, 4 * j);
        consider(q[u].y, 4 * j + 1);
        consider(q[u].z, 4 * j + 2);
        consider(q[u].w, 4 * j + 3);
      }
    }
  }
  for (int i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) consider(logits[i], i);
  // combine (value, index): larger value wins, equal values keep the lower index
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = v;
    bi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    v = threadIdx.x < nw ? bv[threadIdx.x] : -INFINITY;
    idx = threadIdx.x < nw ? bi[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (threadIdx.x == 0) {
      if (idx == 0x7fffffff) idx = 0;
      idx += vocab_offset;
      if (tp.world > 1) {  // compare the vocabulary slices' maxima across ranks
        const uint32_t seq = *tp.seq;
        const size_t f = (size_t)(seq & 1u) * tp.world;
        for (int r = 0; r < tp.world; ++r) tp.argv[r][f + tp.rank] = make_float2(v, __int_as_float(idx));
        __threadfence_system();  // orders the argv stores before the flags: one fence, `world` plain stores
        for (int r = 0; r < tp.world; ++r)
          asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(tp.aflag[r] + f + tp.rank), "r"(seq) : "memory");
        float bv2 = -INFINITY;
        int bi2 = 0x7fffffff;
        for (int r = 0; r < tp.world; ++r) {
          if (!wait_flag(tp.aflag[tp.rank] + f + r, seq, error)) {
            atomicExch(error, 1);
            continue;
          }
          const float2 e = __ldcg(tp.argv[tp.rank] + f + r);
          const int ei = __float_as_int(e.y);
          if (bi2 == 0x7fffffff || e.x > bv2 || (e.x == bv2 && ei < bi2)) {
            bv2 = e.x;
            bi2 = ei;
          }
        }
        idx = bi2 == 0x7fffffff ? 0 : bi2;
        *tp.seq = seq + 1;
      }
      if ((int)st->n_out < max_out) out[st->n_out] = (uint32_t)idx;
      st->n_out += 1;
      st->token = (uint32_t)idx;
      const uint32_t pos = st->pos + 1;
      st->pos = pos;
      st->slot = pos % (uint32_t)max_seq;
      st->active = pos + 1 < (uint32_t)max_seq ? pos + 1 : (uint32_t)max_seq;
    }
  }
}

template <typename T>
int dev_alloc(T** p, size_t n, size_t* total) {
  if (cudaMalloc(reinterpret_cast<void**>(p), sizeof(T) * (n ? n : 1)) != cudaSuccess) return -5;
  *total += sizeof(T) * (n ? n : 1);
  return 0;
}

}  // namespace

float attn_scale_for(int head_dim) {
  const double x = (double)head_dim;
  double z = 0.0;
  if (x > 0) {
    z = x / 2;
    for (int i = 0; i < 10; i++) z = (z + x / z) / 2;
  }
  return (float)(1.0 / z);
}

DecodeModel::~DecodeModel() {
  if (graph) cudaGraphExecDestroy(graph);
  layers_plan_free(plan_);
  for (void* p : {(void*)x_, (void*)xb_, (void*)q_, (void*)k_, (void*)v_, (void*)att_, (void*)proj_, (void*)gate_,
                  (void*)up_, (void*)logits_, (void*)kcache_, (void*)vcache_, (void*)part_, (void*)rope_, (void*)st_,
                  (void*)tokens_out_})
    if (p) cudaFree(p);
  delete[] layers_;
}

int DecodeModel::init(const ModelCfg& cfg, const LayerRef* layers, const MatRef& tok_embd, const float* out_norm,
                      const MatRef& out, int sm_count, int* error_word, const TpDev* tp) {
  cfg_ = cfg;
  if (cfg.tp_world > 1) {
    if (!tp || tp->world != cfg.tp_world || tp->rank != cfg.tp_rank || tp->max_dim < cfg.dim) return -4;
    tp_ = *tp;
    tp_.error = error_word;
  } else {
    tp_ = TpDev();
  }
  if (cfg.n_layers < 1 || cfg.dim < 1 || cfg.n_heads < 1 || cfg.n_kv_heads < 1 || cfg.head_dim < 2 ||
      cfg.head_dim % 2 || cfg.head_dim > 1024 || cfg.n_heads % cfg.n_kv_heads || cfg.max_seq < 1 ||
      cfg.max_pos < 1 || cfg.vocab < 1 || cfg.hidden < 1)
    return -4;
  const int kv_mul = cfg.n_heads / cfg.n_kv_heads;
  if (cfg.head_dim % 4) return -4;  // float4 staging of K / V rows
  const size_t att_smem = attn_smem_bytes(kv_mul, cfg.head_dim);
  if (att_smem > 200 * 1024) return -4;
  if (att_smem > 48 * 1024 &&
      cudaFuncSetAttribute(attn_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)att_smem) !=
          cudaSuccess)
    return -5;
  n_layers_ = cfg.n_layers;
  layers_ = new LayerRef[n_layers_];
  for (int l = 0; l < n_layers_; ++l) layers_[l] = layers[l];
  tok_embd_ = tok_embd;
  out_ = out;
  out_norm_ = out_norm;
  sm_count_ = sm_count;
  scratch_.error = error_word;
  const int q_dim = cfg.n_heads * cfg.head_dim, kv_dim = cfg.n_kv_heads * cfg.head_dim;
  att_splits_ = (cfg.max_seq + kAttChunk - 1) / kAttChunk;
  max_out_ = 1 << 16;
  size_t t = 0;
  int rc = 0;
  rc |= dev_alloc(&x_, cfg.dim, &t);
  rc |= dev_alloc(&xb_, cfg.dim, &t);
  rc |= dev_alloc(&q_, q_dim, &t);
  rc |= dev_alloc(&k_, kv_dim, &t);
  rc |= dev_alloc(&v_, kv_dim, &t);
  rc |= dev_alloc(&att_, q_dim, &t);
  rc |= dev_alloc(&proj_, cfg.dim, &t);
  rc |= dev_alloc(&gate_, cfg.hidden, &t);
  rc |= dev_alloc(&up_, cfg.hidden, &t);
  rc |= dev_alloc(&logits_, cfg.vocab, &t);
  rc |= dev_alloc(&kcache_, (size_t)cfg.n_layers * cfg.max_seq * kv_dim, &t);
  rc |= dev_alloc(&vcache_, (size_t)cfg.n_layers * cfg.max_seq * kv_dim, &t);
  rc |= dev_alloc(&part_, (size_t)cfg.n_heads * att_splits_ * (cfg.head_dim + 2), &t);
  rc |= dev_alloc(&rope_, (size_t)cfg.max_pos * (cfg.head_dim / 2), &t);
  rc |= dev_alloc(&st_, 1, &t);
  rc |= dev_alloc(&tokens_out_, max_out_, &t);
  if (rc) return -5;
  dev_bytes_ = t;
  // RoPE angles in double, rounded to float32 (kernels.go:25-29).
  const int half = cfg.head_dim / 2;
  std::vector<float2> tab((size_t)cfg.max_pos * half);
  for (int i = 0; i < half; ++i) {
    const double freq = 1.0 / std::pow((double)cfg.rope_theta, (double)(2 * i) / (double)cfg.head_dim);
    for (int p = 0; p < cfg.max_pos; ++p) {
      const double val = (double)p * freq;
      tab[(size_t)p * half + i] = make_float2((float)std::cos(val), (float)std::sin(val));
    }
  }
  if (cudaMemcpy(rope_, tab.data(), sizeof(float2) * tab.size(), cudaMemcpyHostToDevice) != cudaSuccess) return -5;
  if (cudaMemset(kcache_, 0, sizeof(float) * (size_t)cfg.n_layers * cfg.max_seq * kv_dim) != cudaSuccess ||
      cudaMemset(vcache_, 0, sizeof(float) * (size_t)cfg.n_layers * cfg.max_seq * kv_dim) != cudaSuccess ||
      cudaMemset(st_, 0, sizeof(StepState)) != cudaSuccess)
    return -5;
  return 0;
}

void DecodeModel::bind(const LayerRef* layers, const MatRef& tok_embd, const float* out_norm, const MatRef& out) {
  for (int l = 0; l < n_layers_; ++l) layers_[l] = layers[l];
  tok_embd_ = tok_embd;
  out_norm_ = out_norm;
  out_ = out;
  if (plan_ && set_persistent(true)) set_persistent(false);  // the plan holds the weight pointers
}

int DecodeModel::set_persistent(bool on) {
  layers_plan_free(plan_);
  plan_ = nullptr;
  if (!on) return 0;
  if (int rc = layers_prepare_device()) return rc;
  return layers_plan_build(layers_, n_layers_, cfg_, x_, q_, k_, v_, att_, gate_, up_,
                           cfg_.tp_world > 1 ? &tp_ : nullptr, sm_count_, &plan_);
}

void DecodeModel::reset_cache(cudaStream_t s) {
  const size_t kv = (size_t)cfg_.n_layers * cfg_.max_seq * cfg_.n_kv_heads * cfg_.head_dim;
  cudaMemsetAsync(kcache_, 0, sizeof(float) * kv, s);
  cudaMemsetAsync(vcache_, 0, sizeof(float) * kv, s);
}

// x += (sum over ranks of) W_shard * in: this rank's partial goes to every
// rank's exchange region (from the Q4_K GEMV's epilogue, or through
// tp_push_kernel), then the rank-ordered sum is added to x.
int DecodeModel::project_partial(const MatRef& W, const float* in, int cols, cudaStream_t s, bool pdl) {
  GemvLaunch L;
  L.sm_count = sm_count_;
  L.pdl = pdl;
  if (W.qtype == kTypeQ4_K) {  // push, wait and sum in the GEMV's epilogue: x += sum of the ranks' W x
    float* ys[1] = {x_};
    const void* ws[1] = {W.w};
    const size_t wb[1] = {W.bytes};
    const int64_t rows[1] = {cfg_.dim};
    GemvFuse f;
    f.ymode = kYPush;
    f.tp = &tp_;
    return gemv_q4k_fused(1, ys, in, ws, wb, rows, cols, f, L, s);
  }
  int rc = gemv_launch(W.qtype, proj_, in, W.w, W.bytes, cfg_.dim, cols, scratch_, L, s);
  if (!rc && launch(pdl, dim3(1), dim3(1024), 0, s, tp_push_kernel, (const float*)proj_, cfg_.dim, tp_) !=
                 cudaSuccess)
    rc = -5;
  if (rc) return rc;
  return launch(pdl, dim3(kReduceCtas), dim3(kReduceThreads), 0, s, tp_reduce_kernel, x_, cfg_.dim, tp_,
                scratch_.error) == cudaSuccess
             ? 0
             : -5;
}

int DecodeModel::enqueue_step(cudaStream_t s, bool embed, bool pdl) {
  const ModelCfg& c = cfg_;
  const int hd = c.head_dim, q_dim = c.n_heads * hd, kv_dim = c.n_kv_heads * hd;
  const int kv_mul = c.n_heads / c.n_kv_heads;
  GemvLaunch L;
  L.sm_count = sm_count_;
  L.pdl = pdl;
  auto blocks = [](int n, int b) { return dim3((unsigned)((n + b - 1) / b)); };
  cudaError_t e = cudaSuccess;
  int rc = 0;
  if (embed) {
    const int64_t rb = tok_embd_.qtype == kTypeF32 ? (int64_t)c.dim * 4 : row_bytes(tok_embd_.qtype, c.dim);
    if (rb <= 0) return -2;
    e = launch(pdl, blocks(c.dim, 256), dim3(256), 0, s, embed_kernel, (const StepState*)st_,
               (const uint8_t*)tok_embd_.w, tok_embd_.qtype, c.dim, (size_t)rb, x_);
    if (e != cudaSuccess) return -5;
  }
  const size_t layer_kv = (size_t)c.max_seq * kv_dim;
  if (plan_) {  // every layer in one persistent launch
    LayersCfg a;
    a.n_layers = n_layers_;
    a.st = st_;
    a.q = q_, a.k = k_, a.v = v_, a.att = att_, a.part = part_;
    a.kcache = kcache_, a.vcache = vcache_;
    a.rope = rope_;
    a.layer_kv = layer_kv;
    a.kv_mul = kv_mul, a.hd = hd, a.kv_dim = kv_dim, a.n_kv_heads = c.n_kv_heads, a.n_heads = c.n_heads;
    a.splits = att_splits_;
    // items split only while twice as many still run in one round of CTAs
    // (one CTA per SM): one round of whole items beats two of halves
    a.hq = attn_heads_per_item(kv_mul, c.n_kv_heads, att_splits_, sm_count_ / 2 + 1);
    a.scale = c.attn_scale;
    a.max_pos = (uint32_t)c.max_pos;
    a.error = scratch_.error;
    rc = layers_enqueue(plan_, a, s);
    if (rc) return rc;
  }
  const int n_launched = plan_ ? 0 : n_layers_;  // layers run by per-layer launches
  for (int l = 0; l < n_launched; ++l) {
    const LayerRef& Ly = layers_[l];
    float* kc = kcache_ + l * layer_kv;
    float* vc = vcache_ + l * layer_kv;
    // RMSNorm + Q, K, V.  Q4_K: one launch, the norm folded into the GEMV's
    // activation staging.
    if (Ly.wq.qtype == kTypeQ4_K && Ly.wk.qtype == kTypeQ4_K && Ly.wv.qtype == kTypeQ4_K) {
      float* ys[3] = {q_, k_, v_};
      const void* ws[3] = {Ly.wq.w, Ly.wk.w, Ly.wv.w};
      const size_t wb[3] = {Ly.wq.bytes, Ly.wk.bytes, Ly.wv.bytes};
      const int64_t rows[3] = {q_dim, kv_dim, kv_dim};
      GemvFuse f;
      f.xmode = kXNorm;
      f.x2 = Ly.attn_norm;
      f.eps = c.eps;
      rc = gemv_q4k_fused(3, ys, x_, ws, wb, rows, c.dim, f, L, s);
    } else {
      e = launch(pdl, dim3(1), dim3(1024), 0, s, rmsnorm_kernel, (const float*)x_, Ly.attn_norm, xb_, c.dim, c.eps);
      if (e != cudaSuccess) return -5;
      rc = gemv_launch(Ly.wq.qtype, q_, xb_, Ly.wq.w, Ly.wq.bytes, q_dim, c.dim, scratch_, L, s);
      if (!rc) rc = gemv_launch(Ly.wk.qtype, k_, xb_, Ly.wk.w, Ly.wk.bytes, kv_dim, c.dim, scratch_, L, s);
      if (!rc) rc = gemv_launch(Ly.wv.qtype, v_, xb_, Ly.wv.w, Ly.wv.bytes, kv_dim, c.dim, scratch_, L, s);
    }
    if (rc) return rc;
    if (Ly.bq) e = launch(pdl, blocks(q_dim, 256), dim3(256), 0, s, add_kernel, q_, Ly.bq, q_dim);
    if (Ly.bk && e == cudaSuccess) e = launch(pdl, blocks(kv_dim, 256), dim3(256), 0, s, add_kernel, k_, Ly.bk, kv_dim);
    if (Ly.bv && e == cudaSuccess) e = launch(pdl, blocks(kv_dim, 256), dim3(256), 0, s, add_kernel, v_, Ly.bv, kv_dim);
    if (e != cudaSuccess) return -5;
    // at least two items per SM: under tensor parallelism a rank's few kv
    // heads are split by query-head groups
    const int hq = attn_heads_per_item(kv_mul, c.n_kv_heads, att_splits_, 2 * sm_count_);
    e = launch(pdl, dim3(c.n_kv_heads * (kv_mul / hq), att_splits_), dim3(256), attn_smem_bytes(hq, hd), s,
               attn_partial_kernel,
               (const StepState*)st_, (const float*)q_, (const float*)k_, (const float*)v_, (const float2*)rope_, kc,
               vc, part_, kv_mul, hd, kv_dim, att_splits_, c.attn_scale, (uint32_t)c.max_pos, scratch_.error, hq);
    if (e != cudaSuccess) return -5;
    e = launch(pdl, dim3(c.n_heads), dim3(hd), 0, s, attn_combine_kernel, (const float*)part_, att_, hd, att_splits_);
    if (e != cudaSuccess) return -5;
    // Output projection + residual (x += Wo att); across ranks the partial
    // products are summed first.
    if (c.tp_world > 1) {
      rc = project_partial(Ly.wo, att_, q_dim, s, pdl);
      if (rc) return rc;
    } else if (Ly.wo.qtype == kTypeQ4_K) {
      float* ys[1] = {x_};
      const void* ws[1] = {Ly.wo.w};
      const size_t wb[1] = {Ly.wo.bytes};
      const int64_t rows[1] = {c.dim};
      GemvFuse f;
      f.ymode = kYAdd;
      rc = gemv_q4k_fused(1, ys, att_, ws, wb, rows, q_dim, f, L, s);
    } else {
      rc = gemv_launch(Ly.wo.qtype, proj_, att_, Ly.wo.w, Ly.wo.bytes, c.dim, q_dim, scratch_, L, s);
      if (!rc && launch(pdl, blocks(c.dim, 256), dim3(256), 0, s, residual_kernel, x_, (const float*)proj_, c.dim) !=
                     cudaSuccess)
        rc = -5;
    }
    if (rc) return rc;
    // RMSNorm + gate and up + SwiGLU: one launch for Q4_K.
    if (Ly.gate.qtype == kTypeQ4_K && Ly.up.qtype == kTypeQ4_K) {
      float* ys[2] = {gate_, up_};
      const void* ws[2] = {Ly.gate.w, Ly.up.w};
      const size_t wb[2] = {Ly.gate.bytes, Ly.up.bytes};
      const int64_t rows[2] = {c.hidden, c.hidden};
      GemvFuse f;
      f.xmode = kXNorm;
      f.x2 = Ly.ffn_norm;
      f.eps = c.eps;
      f.ymode = kYSwiGLU;
      rc = gemv_q4k_fused(2, ys, x_, ws, wb, rows, c.dim, f, L, s);
    } else {
      e = launch(pdl, dim3(1), dim3(1024), 0, s, rmsnorm_kernel, (const float*)x_, Ly.ffn_norm, xb_, c.dim, c.eps);
      if (e != cudaSuccess) return -5;
      rc = gemv_launch(Ly.gate.qtype, gate_, xb_, Ly.gate.w, Ly.gate.bytes, c.hidden, c.dim, scratch_, L, s);
      if (!rc) rc = gemv_launch(Ly.up.qtype, up_, xb_, Ly.up.w, Ly.up.bytes, c.hidden, c.dim, scratch_, L, s);
      if (!rc && launch(pdl, blocks(c.hidden, 256), dim3(256), 0, s, swiglu_kernel, gate_, (const float*)up_,
                        c.hidden) != cudaSuccess)
        rc = -5;
    }
    if (rc) return rc;
    // Down projection + residual (x += Wdown h).
    if (c.tp_world > 1) {
      rc = project_partial(Ly.down, gate_, c.hidden, s, pdl);
      if (rc) return rc;
    } else if (Ly.down.qtype == kTypeQ4_K) {
      float* ys[1] = {x_};
      const void* ws[1] = {Ly.down.w};
      const size_t wb[1] = {Ly.down.bytes};
      const int64_t rows[1] = {c.dim};
      GemvFuse f;
      f.ymode = kYAdd;
      rc = gemv_q4k_fused(1, ys, gate_, ws, wb, rows, c.hidden, f, L, s);
    } else {
      rc = gemv_launch(Ly.down.qtype, proj_, gate_, Ly.down.w, Ly.down.bytes, c.dim, c.hidden, scratch_, L, s);
      if (!rc && launch(pdl, blocks(c.dim, 256), dim3(256), 0, s, residual_kernel, x_, (const float*)proj_, c.dim) !=
                     cudaSuccess)
        rc = -5;
    }
    if (rc) return rc;
  }
  // after the cooperative layers kernel: plain stream order
  e = launch(pdl && !plan_, dim3(1), dim3(1024), 0, s, rmsnorm_kernel, (const float*)x_, out_norm_, xb_, c.dim,
             c.eps);
  if (e != cudaSuccess) return -5;
  rc = gemv_launch(out_.qtype, logits_, xb_, out_.w, out_.bytes, c.vocab, c.dim, scratch_, L, s);
  if (rc) return rc;
  e = launch(pdl, dim3(1), dim3(1024), 0, s, argmax_kernel, (const float*)logits_, c.vocab, st_, tokens_out_,
             max_out_, c.max_seq, c.vocab_offset, tp_, scratch_.error);
  return e == cudaSuccess ? 0 : -5;
}

}  // namespace gi
