// layers.cu -- the persistent decode-layer kernel.
//
// The multi-launch decode step (model.cu) runs six kernels per layer (QKV,
// attention partials, combine, O, gate/up, down); every launch carries a
// few microseconds of fixed cost -- the next grid's CTAs start only as the
// previous grid's exit, then wait for their first weights -- which at the
// Llama shapes is more than the layer's weight streaming.  Here the layers
// of one step run in one cooperative launch of one 16-warp CTA per SM:
// the same phases, separated by grid-wide barriers, with each projection's
// first weight units requested into the CTA's rings as soon as the previous
// projection is done in that CTA -- before the barrier and the attention
// phases that precede it -- so DRAM latency overlaps the synchronisation.
//
// The arithmetic is that of the stand-alone kernels, from the same device
// code (q4k.cuh, attn.cuh): a step computes the same bits as the
// multi-launch step.  Activations written earlier in the launch are read
// with plain (coherent) loads, never through the read-only path.
//
// Every wait is bounded: a grid barrier gives up after 2 s (or as soon as
// the error word is set), marks the error word and the CTA returns after
// draining its own copies in flight; the tensor-parallel exchange waits are
// the bounded ones of the stand-alone kernel.
#include <algorithm>
#include <cstring>
#include <vector>

#include "attn.cuh"
#include "common.cuh"
#include "layers.cuh"
#include "q4k.cuh"

namespace gi {

namespace {

constexpr int kLW = q4k::kWarpsLarge;  // warps per CTA
constexpr int kLThreads = kLW * 32;

// One phase's GEMV parameters, padded so the table's entries are 16-byte
// aligned (copied into shared memory with 16-byte loads).
struct alignas(16) PhaseSlot {
  q4k::Params p;
};

struct PlanDev {
  const PhaseSlot* ph;  // [n_layers][4]: QKV, O, gate/up, down
  int x_off;            // staged activations, and the attention work area
  int prm_off;          // the current phase's Params
  int flag_off;         // barrier result (one int)
};

GI_DEVINL uint32_t ld_acquire_gpu(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier in two halves: the counter at `bar` (zero at launch)
// reaches `target` = (barrier number) x (CTAs).  All writes of the CTA
// before grid_arrive are visible to every CTA after its grid_wait (fence,
// add; acquire poll, fence).  The halves are split so that a CTA can
// request its next projection's weights in between: a fence issued after
// those cp.async requests waits for them (measured: the barrier released
// 4-5 us after the last CTA arrived, against ~1 us when nothing was in
// flight).  grid_wait is false when it gave up: after 2 s, or soon after
// another wait set the error word (read every 256 polls: mapped host
// memory, a PCIe round trip).
GI_DEVINL void grid_arrive(unsigned* bar) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
  }
}

GI_DEVINL bool grid_wait(unsigned* bar, unsigned target, int* error, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    if (ld_acquire_gpu(bar) < target) {
      const uint64_t t0 = now_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_gpu(bar) >= target) break;
        if ((i & 255u) == 0) {
          if (*(volatile const int*)error) {
            ok = 0;
            break;
          }
          if (now_ns() - t0 > 2000000000ull) {
            *(volatile int*)error = 1;
            ok = 0;
            break;
          }
        }
      }
    }
    // No trailing fence: the acquire load above orders this thread after
    // every arriving CTA's release (fence + add), and the CTA barrier below
    // orders the other threads after it; a fence here would also wait for
    // the weight requests issued since grid_arrive.
    *flag = ok;
  }
  __syncthreads();
  return *flag != 0;
}

// The current phase's Params into shared memory (after every thread is done
// with the previous phase's).
GI_DEVINL void load_params(q4k::Params* dst, const PhaseSlot* src) {
  __syncthreads();
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int i = threadIdx.x; i < (int)(sizeof(PhaseSlot) / 16); i += blockDim.x) d[i] = __ldg(s + i);
  __syncthreads();
}

// One CTA's share of a Q4_K GEMV phase: the stand-alone kernel's body
// (gemv.cu, gemv_q4k_kernel with the fusions compiled in) split in two.
// begin() sets up the cursors and requests the first S units; run() stages
// the activations and streams the rest.  Between the two the CTA may wait
// at grid barriers and run attention work, which touches neither the rings
// nor the partial-sum slots.  Differences from the kernel: the Params live
// in shared memory; the activations are read coherently; the exchange
// counters are read with volatile loads; the CTA that finishes a push phase
// last is counted against the phase's CTAs, not the grid.
template <int W, int S>
struct GemvPhase {
  int lane, warp, g, t;
  uint64_t pol;
  bool active;
  int T0, ntl, n, nku;
  long long rowb, step15;
  uint32_t ring, dst0, dst1, dsth;
  int ltile, lku, next, fast_end;
  const uint8_t* pa;
  const uint8_t* pb;

  GI_DEVINL void init() {
    lane = threadIdx.x & 31;
    warp = threadIdx.x >> 5;
    g = lane >> 2;
    t = lane & 3;
    pol = l2_evict_first_policy();
    active = false;
  }

  GI_DEVINL void seek(const q4k::Params& p) {
    int m, lt;
    q4k::tile_of<true>(p, T0 + ltile, m, lt);
    const int r0 = lt * 16, rl = p.rows[m] - 1;
    pa = p.w[m] + (long long)min(r0 + g, rl) * rowb + lku * 144;
    pb = p.w[m] + (long long)min(r0 + g + 8, rl) * rowb + lku * 144;
    fast_end = p.ymode == kYSwiGLU ? 0 : p.tstart[m] + (p.rows[m] >> 4);
  }

  GI_DEVINL void request(const q4k::Params& p, int stage) {  // always commits one group (possibly empty)
    if (next < n) {
      const uint32_t o = (uint32_t)stage * q4k::kStageBytes;
      cp_async16_hint(dst0 + o, pa + 16 + 32 * t, pol);
      cp_async16_hint(dst1 + o, pa + 32 + 32 * t, pol);
      cp_async16_hint(dst0 + o + 1024, pb + 16 + 32 * t, pol);
      cp_async16_hint(dst1 + o + 1024, pb + 32 + 32 * t, pol);
      if (t < 2) cp_async16_hint(dsth + o, t ? pb : pa, pol);
      next += W;
      lku += W;
      pa += W * 144;
      pb += W * 144;
      if (lku >= nku) {
        int dt = 0;
        do {
          lku -= nku;
          ++dt;
        } while (lku >= nku);
        ltile += dt;
        if (next < n) {
          if (T0 + ltile < fast_end) {
            pa += dt * step15;
            pb += dt * step15;
          } else {
            seek(p);
          }
        }
      }
    }
    cp_async_commit();
  }

  GI_DEVINL void begin(const q4k::Params& p, uint8_t* smem, int c) {
    active = c < p.ctas;
    if (!active) return;
    const int gran = p.ymode == kYSwiGLU ? 2 : 1, nun = p.ntiles / gran;
    T0 = gran * (int)((long long)nun * c / p.ctas);
    const int T1 = gran * (int)((long long)nun * (c + 1) / p.ctas);
    nku = p.nku;
    rowb = p.rowb;
    ntl = T1 - T0;
    n = ntl * nku;
    ring = smem_u32(smem) + warp * S * q4k::kStageBytes;
    float* slots = reinterpret_cast<float*>(smem + p.slot_off);  // [ntl][W][16]
    for (int i = threadIdx.x; i < ntl * W * 16; i += W * 32) slots[i] = 0.f;
    ltile = warp / nku;
    lku = warp - ltile * nku;
    next = warp;
    fast_end = 0;
    pa = nullptr;
    pb = nullptr;
    if (next < n) seek(p);
    step15 = 15 * rowb;
    dst0 = ring + g * 128 + 16u * ((2u * (uint32_t)t) ^ (uint32_t)g);
    dst1 = ring + g * 128 + 16u * ((2u * (uint32_t)t + 1u) ^ (uint32_t)g);
    dsth = ring + 2048 + (g + 8 * (t & 1)) * 16;
#pragma unroll
    for (int s = 0; s < S; ++s) request(p, s);
  }

  GI_DEVINL void run(const q4k::Params& p, uint8_t* smem) {
    if (!active) return;
    uint8_t* xs = smem + p.x_off;
    const uint32_t xs_s = smem_u32(xs);
    float* slots = reinterpret_cast<float*>(smem + p.slot_off);
    // ends with a CTA barrier (also orders the slot zeroing)
    q4k::stage_x<W, true, true>(xs, reinterpret_cast<float*>(smem + p.red_off), p);

    const uint32_t sh8 = 8u * (uint32_t)t;
    const uint32_t selE = 0x4440u | (t >= 2 ? 1u : 0u), selO = 0x4440u | (t >= 2 ? 3u : 2u);
    const float W0 = t == 0 ? 16777216.f : (t == 1 ? 256.f : (t == 2 ? 1048576.f : 16.f));
    const float W1 = t == 0 ? 65536.f : (t == 1 ? 1.f : (t == 2 ? 4096.f : 0.0625f));
    const uint32_t xlo = (uint32_t)((g & 3) * 32 + 8 * t + (g >= 4 ? 128 : 0));
    const uint32_t lrow = (uint32_t)((lane & 7) + 8 * ((lane >> 3) & 1));
    const uint32_t lofs = lrow * 128u + 16u * ((uint32_t)(lane >> 4) ^ (lrow & 7u));
    int ctile = warp / nku, cku = warp - ctile * nku;
    uint32_t cx = xs_s + cku * q4k::kUnitX;
    float yA = 0.f, yB = 0.f;
    int stage = 0;
    for (int i = warp; i < n; i += W) {
      cp_async_wait<S - 1>();
      __syncwarp();
      q4k::compute_unit(ring + stage * q4k::kStageBytes, lofs, cx, cx + xlo, g, t, sh8, selE, selO, W0, W1, yA, yB);
      __syncwarp();
      request(p, stage);
      stage = stage + 1 == S ? 0 : stage + 1;
      const int tile = ctile;
      cku += W;
      if (cku < nku) {
        cx += W * q4k::kUnitX;
      } else {
        do {
          cku -= nku;
          ++ctile;
        } while (cku >= nku);
        cx = xs_s + cku * q4k::kUnitX;
      }
      if (ctile != tile || i + W >= n) {  // this warp is done with `tile`
        float vA = yA + __shfl_xor_sync(0xffffffffu, yA, 1);
        float vB = yB + __shfl_xor_sync(0xffffffffu, yB, 1);
        vA += __shfl_xor_sync(0xffffffffu, vA, 2);
        vB += __shfl_xor_sync(0xffffffffu, vB, 2);
        yA = 0.f;
        yB = 0.f;
        if (t == 0) {
          float* sl = slots + (tile * W + warp) * 16;
          sl[g] = vA;
          sl[g + 8] = vB;
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();
    // Each tile's partials, summed in fixed warp order (deterministic).
    for (int tl = warp; tl < ntl; tl += W) {
      if (lane < 16) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) sum += slots[(tl * W + w) * 16 + lane];
        int m, lt;
        q4k::tile_of<true>(p, T0 + tl, m, lt);
        const int row = lt * 16 + lane;
        if (p.ymode == kYSwiGLU) {
          if ((tl & 1) == 0 && row < p.rows[0]) {
            float up = 0.f;
#pragma unroll
            for (int w = 0; w < W; ++w) up += slots[((tl + 1) * W + w) * 16 + lane];
            const float silu = __fdiv_rn(sum, __fadd_rn(1.0f, (float)exp(-(double)sum)));
            p.y[0][row] = __fmul_rn(silu, up);
          }
        } else if (p.ymode == kYPush) {
          if (row < p.rows[m]) {
            const uint32_t seq = *(volatile const uint32_t*)p.tp.seq;
            const size_t off = ((size_t)(seq & 1u) * p.tp.world + p.tp.rank) * p.tp.max_dim + row;
            for (int r = 0; r < p.tp.world; ++r) st_ll(p.tp.ll[r] + off, sum, seq);
          }
        } else if (row < p.rows[m]) {
          p.y[m][row] = p.ymode == kYAdd ? __fadd_rn(p.y[m][row], sum) : sum;
        }
      }
    }
    if (p.ymode == kYPush) {
      const uint32_t seq = *(volatile const uint32_t*)p.tp.seq;
      const int world = p.tp.world;
      const unsigned long long* rv = p.tp.ll[p.tp.rank] + (size_t)(seq & 1u) * world * p.tp.max_dim;
      for (int tl = warp; tl < ntl; tl += W) {
        const int row = (T0 + tl) * 16 + lane;
        if (lane < 16 && row < p.rows[0]) {
          // four ranks' words at a time (eight cost this kernel registers)
          float sum = 0.f;
          const bool ok = tp_sum_ll<4>(rv + row, p.tp.max_dim, world, seq, p.tp.error, &sum);
          if (ok)
            p.y[0][row] = __fadd_rn(p.y[0][row], sum);
          else
            atomicExch(p.tp.error, 1);
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.tp.done, 1u) == (unsigned)p.ctas - 1) {
          *(volatile unsigned*)p.tp.done = 0u;
          *(volatile uint32_t*)p.tp.seq = seq + 1;
        }
      }
    }
  }
};

template <int S>
__global__ void __launch_bounds__(kLThreads, 1) layers_kernel(const LayersCfg a, const PlanDev d) {
  extern __shared__ __align__(16) uint8_t smem[];
  q4k::Params* p = reinterpret_cast<q4k::Params*>(smem + d.prm_off);
  int* flag = reinterpret_cast<int*>(smem + d.flag_off);
  float* att_sm = reinterpret_cast<float*>(smem + d.x_off);
  const int c = blockIdx.x;
  const unsigned nct = gridDim.x;
  unsigned nbar = 0;
  auto arrive = [&]() {
    ++nbar;
    grid_arrive(a.bar);
  };
  auto wait = [&]() { return grid_wait(a.bar, nbar * nct, a.error, flag); };
  auto sync = [&]() {
    arrive();
    return wait();
  };
  GemvPhase<kLW, S> G;
  G.init();
  load_params(p, d.ph);
  G.begin(*p, smem, c);
  // Phase k of the step is projection k % 4 of layer k / 4: Q/K/V of
  // RMSNorm(x) (forward.go:200-209); x += Wo att (forward.go:269-273; under
  // tensor parallelism the rank-ordered sum of the ranks' partials); gate
  // and up of RMSNorm(x) with SwiGLU (forward.go:275-283); x += Wdown h
  // (forward.go:284-287).  Between Q/K/V and O run the attention partials
  // (RoPE, this step's cache write, scores and partial softmax sums per
  // (kv head, query-head group, chunk), forward.go:226-266) and their
  // combination.  One code
  // path for all four projections keeps a single copy of the GEMV inlined.
  // attention items: (kv head, head group of hq query heads, chunk), chunk fastest
  const int ng = a.kv_mul / a.hq, items = a.n_kv_heads * ng * a.splits, nph = 4 * a.n_layers;
  for (int k = 0; k < nph; ++k) {
    G.run(*p, smem);
    arrive();
    if (k + 1 < nph) {
      load_params(p, d.ph + k + 1);
      G.begin(*p, smem, c);  // the next projection's first units, while the barrier completes
    }
    if (!wait()) break;
    if ((k & 3) == 0) {
      const int l = k >> 2;
      float* kc = a.kcache + (size_t)l * a.layer_kv;
      float* vc = a.vcache + (size_t)l * a.layer_kv;
      for (int it = c; it < items; it += (int)nct) {
        const int gh = it / a.splits;  // g * ng + hg
        attn_partial_item(a.st, a.q, a.k, a.v, a.rope, kc, vc, a.part, a.kv_mul, a.hd, a.kv_dim, a.splits, a.scale,
                          a.max_pos, a.error, gh / ng, it % a.splits, gh % ng, a.hq, att_sm);
        __syncthreads();
      }
      if (!sync()) break;
      for (int i = c * kLThreads + (int)threadIdx.x; i < a.n_heads * a.hd; i += (int)nct * kLThreads)
        attn_combine_one(a.part, a.att, a.hd, a.splits, i / a.hd, i % a.hd);
      if (!sync()) break;
    }
  }
  cp_async_wait<0>();  // copies requested before a barrier that gave up
}

// Shared-memory layout common to every phase (W = 16, S stages).
struct Layout {
  int stages = 0, slot_off = 0, red_off = 0, prm_off = 0, flag_off = 0, x_off = 0, smem = 0;
};

bool make_layout(int stages, int max_tiles, int max_nku, size_t att_bytes, Layout* o) {
  auto up = [](int v, int a) { return (v + a - 1) / a * a; };
  o->stages = stages;
  o->slot_off = kLW * stages * q4k::kStageBytes;
  o->red_off = o->slot_off + max_tiles * kLW * 16 * 4;
  o->prm_off = up(o->red_off + 4 * kLW, 16);
  o->flag_off = o->prm_off + (int)sizeof(PhaseSlot);
  o->x_off = up(o->flag_off + 16, 128);
  const size_t xbytes = std::max((size_t)max_nku * q4k::kUnitX, att_bytes);
  const size_t total = (size_t)o->x_off + xbytes;
  o->smem = (int)total;
  return total <= (size_t)q4k::kSmemMax;
}

// The GEMV parameters of one projection (q4k::launch's rules).
int fill_phase(const LayersMat& M, int64_t cols, int sm_count, q4k::Params* p, int* max_tiles) {
  if (M.nmat < 1 || M.nmat > q4k::kMaxMats) return -4;
  if (cols < 256 || cols % 256 || cols > q4k::kMaxCols) return -4;
  const GemvFuse& f = M.fuse;
  if (f.ymode == kYSwiGLU && (M.nmat != 2 || M.rows[0] != M.rows[1])) return -4;
  *p = q4k::Params();
  p->tstart[0] = 0;
  for (int m = 0; m < q4k::kMaxMats; ++m) {
    const bool on = m < M.nmat;
    if (on && (!M.w[m] || !M.y[m] || M.rows[m] < 1 || M.rows[m] > (1 << 24))) return -4;
    p->w[m] = on ? static_cast<const uint8_t*>(M.w[m]) : nullptr;
    p->y[m] = on ? M.y[m] : nullptr;
    p->rows[m] = on ? (int)M.rows[m] : 0;
    p->tstart[m + 1] = p->tstart[m] + (on ? (int)((M.rows[m] + 15) / 16) : 0);
  }
  const int gran = f.ymode == kYSwiGLU ? 2 : 1;
  p->ntiles = p->tstart[q4k::kMaxMats];
  const int nun = p->ntiles / gran;
  p->ctas = nun < sm_count ? nun : sm_count;
  *max_tiles = gran * ((nun + p->ctas - 1) / p->ctas);
  p->x2 = f.x2;
  p->eps = f.eps;
  p->xmode = f.xmode;
  p->ymode = f.ymode;
  if (f.ymode == kYPush) {
    if (!f.tp || f.tp->world < 1 || M.rows[0] > f.tp->max_dim || M.nmat != 1 || !f.tp->error) return -4;
    p->tp = *f.tp;
  }
  p->rowb = row_bytes(kTypeQ4_K, cols);
  p->nku = (int)(cols / 256);
  return 0;
}

template <int S>
cudaError_t prepare_one() {
  cudaError_t e = cudaFuncSetAttribute(layers_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, q4k::kSmemMax);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(layers_kernel<S>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
  return e;
}

}  // namespace

struct LayersPlan {
  PhaseSlot* ph = nullptr;  // device
  unsigned* bar = nullptr;  // device
  Layout lay;
  int sm_count = 0;
  size_t bytes = 0;
};

int layers_prepare_device() {
  return prepare_one<3>() == cudaSuccess && prepare_one<2>() == cudaSuccess ? 0 : -5;
}

void layers_plan_free(LayersPlan* plan) {
  if (!plan) return;
  if (plan->ph) cudaFree(plan->ph);
  if (plan->bar) cudaFree(plan->bar);
  delete plan;
}

size_t layers_plan_bytes(const LayersPlan* plan) { return plan ? plan->bytes : 0; }

int layers_plan_build(const LayerRef* layers, int n_layers, const ModelCfg& c, float* x, float* q, float* k, float* v,
                      float* att, float* gate, float* up, const TpDev* tp, int sm_count, LayersPlan** out) {
  *out = nullptr;
  if (n_layers < 1 || sm_count < 1) return -4;
  if (c.tp_world > 1 && !tp) return -4;
  const int hd = c.head_dim, q_dim = c.n_heads * hd, kv_dim = c.n_kv_heads * hd;
  std::vector<PhaseSlot> tab((size_t)n_layers * 4);
  int max_tiles = 1, max_nku = 1;
  for (int l = 0; l < n_layers; ++l) {
    const LayerRef& L = layers[l];
    for (const MatRef* m : {&L.wq, &L.wk, &L.wv, &L.wo, &L.gate, &L.up, &L.down})
      if (m->qtype != kTypeQ4_K || !m->w) return -2;
    if (L.bq || L.bk || L.bv) return -2;
    LayersMat M[4];
    M[0].nmat = 3;
    M[0].w[0] = L.wq.w, M[0].w[1] = L.wk.w, M[0].w[2] = L.wv.w;
    M[0].y[0] = q, M[0].y[1] = k, M[0].y[2] = v;
    M[0].rows[0] = q_dim, M[0].rows[1] = kv_dim, M[0].rows[2] = kv_dim;
    M[0].fuse.xmode = kXNorm, M[0].fuse.x2 = L.attn_norm, M[0].fuse.eps = c.eps;
    M[1].nmat = 1;
    M[1].w[0] = L.wo.w, M[1].y[0] = x, M[1].rows[0] = c.dim;
    M[2].nmat = 2;
    M[2].w[0] = L.gate.w, M[2].w[1] = L.up.w, M[2].y[0] = gate, M[2].y[1] = up;
    M[2].rows[0] = c.hidden, M[2].rows[1] = c.hidden;
    M[2].fuse.xmode = kXNorm, M[2].fuse.x2 = L.ffn_norm, M[2].fuse.eps = c.eps, M[2].fuse.ymode = kYSwiGLU;
    M[3].nmat = 1;
    M[3].w[0] = L.down.w, M[3].y[0] = x, M[3].rows[0] = c.dim;
    for (int j : {1, 3}) {
      if (c.tp_world > 1) {
        M[j].fuse.ymode = kYPush;
        M[j].fuse.tp = tp;
      } else {
        M[j].fuse.ymode = kYAdd;
      }
    }
    const int64_t cols[4] = {c.dim, q_dim, c.dim, c.hidden};
    const float* xin[4] = {x, att, x, gate};
    // the bytes each matrix must hold (the stand-alone launch checks them too)
    const MatRef* mats[4][3] = {{&L.wq, &L.wk, &L.wv}, {&L.wo, nullptr, nullptr}, {&L.gate, &L.up, nullptr},
                                {&L.down, nullptr, nullptr}};
    for (int j = 0; j < 4; ++j) {
      for (int m = 0; m < M[j].nmat; ++m)
        if (mats[j][m]->bytes < (size_t)(row_bytes(kTypeQ4_K, cols[j]) * M[j].rows[m])) return -4;
      q4k::Params& p = tab[(size_t)l * 4 + j].p;
      int mt = 0;
      if (int rc = fill_phase(M[j], cols[j], sm_count, &p, &mt)) return rc;
      p.x = xin[j];
      max_tiles = std::max(max_tiles, mt);
      max_nku = std::max(max_nku, p.nku);
    }
  }
  const size_t att_bytes = attn_smem_bytes(c.n_heads / c.n_kv_heads, hd);
  Layout lay;
  if (!make_layout(3, max_tiles, max_nku, att_bytes, &lay) && !make_layout(2, max_tiles, max_nku, att_bytes, &lay))
    return -4;
  for (PhaseSlot& s : tab) {
    s.p.x_off = lay.x_off;
    s.p.slot_off = lay.slot_off;
    s.p.red_off = lay.red_off;
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      &per_sm, lay.stages == 3 ? layers_kernel<3> : layers_kernel<2>, kLThreads, lay.smem);
  if (e != cudaSuccess) return -5;
  if (per_sm < 1) return -4;  // one CTA per SM must fit for the cooperative launch
  LayersPlan* plan = new LayersPlan;
  plan->lay = lay;
  plan->sm_count = sm_count;
  plan->bytes = sizeof(PhaseSlot) * tab.size() + 256;
  if (cudaMalloc(reinterpret_cast<void**>(&plan->ph), sizeof(PhaseSlot) * tab.size()) != cudaSuccess ||
      cudaMalloc(reinterpret_cast<void**>(&plan->bar), 256) != cudaSuccess ||
      cudaMemcpy(plan->ph, tab.data(), sizeof(PhaseSlot) * tab.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(plan->bar, 0, 256) != cudaSuccess) {
    layers_plan_free(plan);
    return -5;
  }
  *out = plan;
  return 0;
}

int layers_enqueue(const LayersPlan* plan, LayersCfg a, cudaStream_t s) {
  if (!plan) return -4;
  a.bar = plan->bar;
  PlanDev d;
  d.ph = plan->ph;
  d.x_off = plan->lay.x_off;
  d.prm_off = plan->lay.prm_off;
  d.flag_off = plan->lay.flag_off;
  if (cudaMemsetAsync(plan->bar, 0, sizeof(unsigned), s) != cudaSuccess) return -5;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)plan->sm_count);
  cfg.blockDim = dim3(kLThreads);
  cfg.dynamicSmemBytes = (size_t)plan->lay.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = plan->lay.stages == 3 ? cudaLaunchKernelEx(&cfg, layers_kernel<3>, a, d)
                                              : cudaLaunchKernelEx(&cfg, layers_kernel<2>, a, d);
  return e == cudaSuccess ? 0 : -5;
}

}  // namespace gi
