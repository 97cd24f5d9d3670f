// gemv.cu -- decode-time quantised GEMV kernels (batch 1) for sm_100a.
//
// These replace GEMVEngine.MatMul{Q8_0,Q4_K,Q6_K} (pkg/math/gemv.go:98-203
// of go-infer) and the per-row DotVec* they call (pkg/quant/quant.go:320-339,
// 536-545).  Weights are the raw GGUF blocks, row-major, rows = output
// features; x and y are fp32 (go-infer never quantises activations).
//
// Q4_K kernel: at most one CTA per SM, each owning a contiguous run of
// 16-row tiles.  Its 8 or 16 warps stream their units' raw super-blocks into
// per-warp shared-memory rings with cp.async (up to 4 units ahead, the first
// ones requested before the kernel waits on its predecessor) and take exact
// integer dot products on the int8 tensor cores (see namespace q4k).
//
// Q8_0 kernel (rows of whole 256-column groups): the Q4_K structure with one
// exact int8 tensor-core MMA per 32-element block (see namespace q80m).
//
// Q6_K kernels and the remaining Q8_0 rows: 2 or 4 rows per warp, fp32
// CUDA-core dot products.  Their 34- and 210-byte blocks are only 2-byte
// aligned; rows whose length keeps 32-block (Q8_0) or 8-super-block (Q6_K)
// chunks 16-byte aligned are streamed through per-warp two-stage cp.async
// rings, other rows are staged with aligned 128-bit loads; words are
// realigned with funnel shifts.
#include "common.cuh"
#include "gemv.cuh"
#include "q4k.cuh"

namespace gi {

// Every kernel of the library runs with the same (maximum) shared-memory
// carveout, so that kernels that follow each other under programmatic
// dependent launch can share an SM without a carveout change draining it.
template <typename K>
cudaError_t set_max_shared_carveout(K kernel) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                              (int)cudaSharedmemCarveoutMaxShared);
}

int64_t row_bytes(int qtype, int64_t cols) {
  switch (qtype) {
    case kTypeQ8_0: return (cols / 32) * 34;
    case kTypeQ4_K: return (cols / 256) * 144;
    case kTypeQ6_K: return (cols / 256) * 210;
    case kTypeF32: return cols * 4;
    default: return -1;
  }
}

namespace q4k {

// F: the decode-step fusions (RMSNorm staging, residual / SwiGLU / push
// epilogues) are compiled in; without them the kernel is the plain GEMV.
template <int W, int S, bool F>
__global__ void __launch_bounds__(W * 32, W == kWarpsSmall ? 2 : 1) gemv_q4k_kernel(const Params p) {
  constexpr int kWarps = W;
  extern __shared__ __align__(16) uint8_t smem[];
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int c = blockIdx.x;
  // CTA c owns tiles [T0, T1); in kYSwiGLU mode whole (gate, up) pairs.
  const int gran = (F && p.ymode == kYSwiGLU) ? 2 : 1, nun = p.ntiles / gran;
  const int T0 = gran * (int)((long long)nun * c / p.ctas), T1 = gran * (int)((long long)nun * (c + 1) / p.ctas);
  const int ntl = T1 - T0, n = ntl * p.nku;  // the CTA's units, tile-major
  const uint32_t ring = smem_u32(smem) + warp * S * kStageBytes;
  uint8_t* xs = smem + p.x_off;
  const uint32_t xs_s = smem_u32(xs);
  float* slots = reinterpret_cast<float*>(smem + p.slot_off);  // [ntl][kWarps][16]
  const uint64_t pol = l2_evict_first_policy();
  // each warp zeroes its own partial slots (other warps read them only
  // after the CTA barrier that ends the streaming loop)
  for (int i = lane; i < ntl * 16; i += 32) slots[((i >> 4) * kWarps + warp) * 16 + (i & 15)] = 0.f;

  // Warp w takes the CTA's units w, w + kWarps, ...: at any moment the warps
  // stream neighbouring super-blocks of the same 16 rows (one long run of
  // bytes per row), which keeps DRAM pages open.  Request cursor: unit
  // `next` = (tile ltile, column block lku); pa, pb: its super-blocks in
  // rows g and g + 8, advanced in place, also across tiles while they stay
  // whole tiles of one matrix (global tiles below fast_end); seek() places
  // them anew (first unit, a new matrix, a tile whose last rows are clamped,
  // interleaved SwiGLU tiles).
  int ltile = warp / p.nku, lku = warp - ltile * p.nku;
  int next = warp, fast_end = 0;
  const uint8_t* pa = nullptr;
  const uint8_t* pb = nullptr;
  auto seek = [&]() {
    int m, lt;
    tile_of<F>(p, T0 + ltile, m, lt);
    const int r0 = lt * 16, rl = p.rows[m] - 1;
    pa = p.w[m] + (long long)min(r0 + g, rl) * p.rowb + lku * 144;
    pb = p.w[m] + (long long)min(r0 + g + 8, rl) * p.rowb + lku * 144;
    fast_end = (F && p.ymode == kYSwiGLU) ? 0 : p.tstart[m] + (p.rows[m] >> 4);
  };
  if (next < n) seek();
  // Moving from column block lku + kWarps - dt*nku of a row to column block
  // lku of the row 16*dt further on is dt * 15 rows of bytes.
  const long long step15 = 15 * p.rowb;
  // this lane's destinations in a stage: 16-byte pieces 2t, 2t+1 of rows g,
  // g + 8 (piece q of row r at slot q ^ (r & 7)) and, for t < 2, the header
  // of row g + 8t
  const uint32_t dst0 = ring + g * 128 + 16u * ((2u * (uint32_t)t) ^ (uint32_t)g);
  const uint32_t dst1 = ring + g * 128 + 16u * ((2u * (uint32_t)t + 1u) ^ (uint32_t)g);
  const uint32_t dsth = ring + 2048 + (g + 8 * (t & 1)) * 16;
  auto request = [&](int stage) {  // always commits one group (possibly empty)
    if (next < n) {
      const uint32_t o = (uint32_t)stage * kStageBytes;
      cp_async16_hint(dst0 + o, pa + 16 + 32 * t, pol);
      cp_async16_hint(dst1 + o, pa + 32 + 32 * t, pol);
      cp_async16_hint(dst0 + o + 1024, pb + 16 + 32 * t, pol);
      cp_async16_hint(dst1 + o + 1024, pb + 32 + 32 * t, pol);
      if (t < 2) cp_async16_hint(dsth + o, t ? pb : pa, pol);
      next += kWarps;
      lku += kWarps;
      pa += kWarps * 144;
      pb += kWarps * 144;
      if (lku >= p.nku) {
        int dt = 0;
        do {
          lku -= p.nku;
          ++dt;
        } while (lku >= p.nku);
        ltile += dt;
        if (next < n) {
          if (T0 + ltile < fast_end) {
            pa += dt * step15;
            pb += dt * step15;
          } else {
            seek();
          }
        }
      }
    }
    cp_async_commit();
  };
  // Weights never depend on the previous kernel: request S units first.
#pragma unroll
  for (int s = 0; s < S; ++s) request(s);
  griddep_wait();
  // When the column blocks are a multiple of the warps, warp w computes
  // only the blocks w, w + kWarps, ... that it staged itself: no CTA
  // barrier between staging and streaming.  (A runtime choice inside one
  // kernel body: as a template parameter, two bodies, the decode step ran
  // 1.5 % slower on B200 with the same stand-alone GEMV times.)
  stage_x<W, F>(xs, reinterpret_cast<float*>(smem + p.red_off), p, p.nku % kWarps != 0);

  const uint32_t sh8 = 8u * (uint32_t)t;
  // byte selectors of this lane's sub-block scale (even / odd chunk c)
  const uint32_t selE = 0x4440u | (t >= 2 ? 1u : 0u), selO = 0x4440u | (t >= 2 ? 3u : 2u);
  // Limb weights 256^(3-n) of this lane's two columns (lanes 2, 3: divided
  // by the 16 their high-nibble sums carry).
  const float W0 = t == 0 ? 16777216.f : (t == 1 ? 256.f : (t == 2 ? 1048576.f : 16.f));
  const float W1 = t == 0 ? 65536.f : (t == 1 ? 1.f : (t == 2 ? 4096.f : 0.0625f));
  const uint32_t xlo = (uint32_t)((g & 3) * 32 + 8 * t + (g >= 4 ? 128 : 0));
  // ldmatrix rows: lanes 8i..8i+7 address matrix i = (rows 0-7 | 8-15) x
  // (bytes 0-15 | 16-31) of a chunk
  const uint32_t lrow = (uint32_t)((lane & 7) + 8 * ((lane >> 3) & 1));
  const uint32_t lofs = lrow * 128u + 16u * ((uint32_t)(lane >> 4) ^ (lrow & 7u));
  int ctile = warp / p.nku, cku = warp - ctile * p.nku;
  uint32_t cx = xs_s + cku * kUnitX;  // the computed unit's staged activations
  float yA = 0.f, yB = 0.f;
  int stage = 0;
  for (int i = warp; i < n; i += kWarps) {
    cp_async_wait<S - 1>();
    __syncwarp();
    compute_unit(ring + stage * kStageBytes, lofs, cx, cx + xlo, g, t, sh8, selE, selO, W0, W1, yA, yB);
    __syncwarp();
    request(stage);
    stage = stage + 1 == S ? 0 : stage + 1;
    const int tile = ctile;
    cku += kWarps;
    if (cku < p.nku) {
      cx += kWarps * kUnitX;
    } else {
      do {
        cku -= p.nku;
        ++ctile;
      } while (cku >= p.nku);
      cx = xs_s + cku * kUnitX;
    }
    if (ctile != tile || i + kWarps >= n) {  // this warp is done with `tile`
      float vA = yA + __shfl_xor_sync(0xffffffffu, yA, 1);
      float vB = yB + __shfl_xor_sync(0xffffffffu, yB, 1);
      vA += __shfl_xor_sync(0xffffffffu, vA, 2);
      vB += __shfl_xor_sync(0xffffffffu, vB, 2);
      yA = 0.f;
      yB = 0.f;
      if (t == 0) {
        float* sl = slots + (tile * kWarps + warp) * 16;
        sl[g] = vA;
        sl[g + 8] = vB;
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  // Each tile's partials, summed in fixed warp order (deterministic).
  for (int tl = warp; tl < ntl; tl += kWarps) {
    if (lane < 16) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) sum += slots[(tl * kWarps + w) * 16 + lane];
      int m, lt;
      tile_of<F>(p, T0 + tl, m, lt);
      const int row = lt * 16 + lane;
      if (F && p.ymode == kYSwiGLU) {
        // gate tile (even) pairs with the next (up) tile: SwiGLU
        // (kernels.go:39-46), silu = g / (1 + float32(exp(float64(-g)))).
        if ((tl & 1) == 0 && row < p.rows[0]) {
          float up = 0.f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) up += slots[((tl + 1) * kWarps + w) * 16 + lane];
          const float silu = __fdiv_rn(sum, __fadd_rn(1.0f, (float)exp(-(double)sum)));
          p.y[0][row] = __fmul_rn(silu, up);
        }
      } else if (F && p.ymode == kYPush) {
        if (row < p.rows[m]) {  // this rank's tagged partial into slot `rank` of every rank's region
          const uint32_t seq = *p.tp.seq;
          const size_t off = ((size_t)(seq & 1u) * p.tp.world + p.tp.rank) * p.tp.max_dim + row;
          for (int r = 0; r < p.tp.world; ++r) st_ll(p.tp.ll[r] + off, sum, seq);
        }
      } else if (row < p.rows[m]) {
        p.y[m][row] = (F && p.ymode == kYAdd) ? __fadd_rn(p.y[m][row], sum) : sum;  // residual: y += W x
      }
    }
  }
  if (F && p.ymode == kYPush) {
    // Every rank's CTA c computes and pushes the same tiles; this CTA waits
    // for the tagged partials of its own rows from every rank and adds their
    // rank-ordered sum into the residual p.y[0]: the same x on every rank.
    // The last CTA to finish advances the exchange count (every CTA read it
    // before counting itself).
    const uint32_t seq = *p.tp.seq;
    const int world = p.tp.world;
    const unsigned long long* rv = p.tp.ll[p.tp.rank] + (size_t)(seq & 1u) * world * p.tp.max_dim;
    for (int tl = warp; tl < ntl; tl += kWarps) {
      const int row = (T0 + tl) * 16 + lane;
      if (lane < 16 && row < p.rows[0]) {
        float sum = 0.f;
        const bool ok = tp_sum_ll(rv + row, p.tp.max_dim, world, seq, p.tp.error, &sum);
        if (ok)
          p.y[0][row] = __fadd_rn(p.y[0][row], sum);
        else
          atomicExch(p.tp.error, 1);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(p.tp.done, 1u) == gridDim.x - 1) {
        *p.tp.done = 0u;
        *p.tp.seq = seq + 1;
      }
    }
  }
}

struct Layout {
  int warps, ctas, ntiles, stages, x_off, slot_off, red_off, smem;
};

Layout layout(int64_t ntiles, int64_t cols, const GemvLaunch& L, int gran = 1) {
  Layout o;
  const int nku = (int)(cols / 256);
  o.ntiles = (int)ntiles;
  const int nun = o.ntiles / gran;
  o.ctas = nun < L.sm_count ? nun : L.sm_count;
  const int max_tiles = gran * ((nun + o.ctas - 1) / o.ctas);
  // 16 warps when the CTAs are fewer than the SMs or hold 64+ units on
  // average; below that the extra warps would idle (measured on B200:
  // 16 warps gain 7-19 % on 4096-28672-column layers and lose 5-17 % on the
  // 1024-3584-column row splits of a tensor-parallel shard).
  bool large = o.ctas < L.sm_count || (long long)o.ntiles * nku >= 64LL * o.ctas;
  const int xbytes = nku * kUnitX;
  // 16 warps need 2 x 16 ring stages next to the staged activations: for
  // the longest rows that does not fit, and 8 warps are used.
  if (large && xbytes + max_tiles * kWarpsLarge * 64 + 4 * kWarpsLarge + kWarpsLarge * 2 * kStageBytes > kSmemMax)
    large = false;
  o.warps = large ? kWarpsLarge : kWarpsSmall;
  const int slot_bytes = max_tiles * o.warps * 16 * 4;
  const int fixed = xbytes + slot_bytes + 4 * o.warps;
  // As many stages as fit next to a co-resident CTA (8 warps: up to 4; 16
  // warps: up to 3), at least 2.
  o.stages = large ? 3 : 4;
  while (o.stages > 2 && fixed + o.warps * o.stages * kStageBytes > kCoresidentSmem) --o.stages;
  o.x_off = o.warps * o.stages * kStageBytes;
  o.slot_off = o.x_off + xbytes;
  o.red_off = o.slot_off + slot_bytes;  // RMSNorm reduction (one float per warp)
  o.smem = o.red_off + 4 * o.warps;
  return o;
}

int launch(int nmat, float* const* y, const float* x, const void* const* w, const int64_t* rows, int64_t cols,
           const GemvLaunch& L, cudaStream_t stream, const GemvFuse& f = GemvFuse()) {
  if (nmat < 1 || nmat > kMaxMats) return -4;
  if (f.ymode == kYSwiGLU && (nmat != 2 || rows[0] != rows[1])) return -4;
  Params p;
  p.tstart[0] = 0;
  for (int m = 0; m < kMaxMats; ++m) {
    const bool on = m < nmat;
    p.w[m] = on ? static_cast<const uint8_t*>(w[m]) : nullptr;
    p.y[m] = on ? y[m] : nullptr;
    p.rows[m] = on ? (int)rows[m] : 0;
    p.tstart[m + 1] = p.tstart[m] + (on ? (int)((rows[m] + 15) / 16) : 0);
  }
  // unused slots repeat the total so tile_of never selects them
  const int gran = f.ymode == kYSwiGLU ? 2 : 1;
  const Layout o = layout(p.tstart[kMaxMats], cols, L, gran);
  if (o.smem > kSmemMax) return -4;
  p.x = x;
  p.x2 = f.x2;
  p.eps = f.eps;
  p.xmode = f.xmode;
  p.ymode = f.ymode;
  if (f.ymode == kYPush) {
    if (!f.tp || f.tp->world < 1 || rows[0] > f.tp->max_dim || nmat != 1 || !f.tp->error)
      return -4;
    p.tp = *f.tp;
  }
  p.rowb = row_bytes(kTypeQ4_K, cols);
  p.nku = (int)(cols / 256);
  p.ntiles = o.ntiles;
  p.ctas = o.ctas;
  p.x_off = o.x_off;
  p.slot_off = o.slot_off;
  p.red_off = o.red_off;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(o.ctas);
  cfg.blockDim = dim3(o.warps * 32);
  cfg.dynamicSmemBytes = o.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  cudaError_t e;
  const bool fused = f.xmode != kXPlain || f.ymode != kYStore;
  // tile counts past nmat equal the total: tile_of stays < nmat
  const int key = (o.warps == kWarpsLarge ? 100 : 0) + o.stages * 2 + (fused ? 1 : 0);
  switch (key) {
    case 8: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsSmall, 4, false>, p); break;
    case 9: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsSmall, 4, true>, p); break;
    case 6: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsSmall, 3, false>, p); break;
    case 7: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsSmall, 3, true>, p); break;
    case 4: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsSmall, 2, false>, p); break;
    case 5: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsSmall, 2, true>, p); break;
    case 106: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsLarge, 3, false>, p); break;
    case 107: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsLarge, 3, true>, p); break;
    case 104: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsLarge, 2, false>, p); break;
    case 105: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<kWarpsLarge, 2, true>, p); break;
    default: return -4;
  }
  return e == cudaSuccess ? 0 : -5;
}

template <int W, int S, bool F>
cudaError_t prepare_one() {
  cudaError_t e =
      cudaFuncSetAttribute(gemv_q4k_kernel<W, S, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  return e == cudaSuccess ? set_max_shared_carveout(gemv_q4k_kernel<W, S, F>) : e;
}

template <int W, int S>
cudaError_t prepare_both() {
  cudaError_t e = prepare_one<W, S, false>();
  return e == cudaSuccess ? prepare_one<W, S, true>() : e;
}

int prepare() {
  cudaError_t e = prepare_both<kWarpsSmall, 4>();
  if (e == cudaSuccess) e = prepare_both<kWarpsSmall, 3>();
  if (e == cudaSuccess) e = prepare_both<kWarpsSmall, 2>();
  if (e == cudaSuccess) e = prepare_both<kWarpsLarge, 3>();
  if (e == cudaSuccess) e = prepare_both<kWarpsLarge, 2>();
  return e == cudaSuccess ? 0 : -5;
}
}  // namespace q4k

// ------------------------ Q8_0 on the int8 tensor cores ---------------------
// Rows of whole 256-column groups (every row and every 8-block unit is then
// 16-byte aligned: 8 x 34 = 272 = 17 x 16).  The structure is the Q4_K
// kernel's: a unit is 16 rows x 256 columns (8 blocks per row, 4352 bytes),
// each CTA owns whole 16-row tiles, units are dealt to the warps round-robin
// and streamed through per-warp cp.async rings, and every tile's per-warp
// partials are summed in fixed warp order.
//
// Arithmetic: one m16n8k32 s8 MMA per block computes the exact int32 dot
// products of its 32 int8 quants (A) with the four balanced base-256 limbs
// of the 30-bit fixed-point activation (B, columns 0-3; one exponent per 256
// columns, as for Q4_K).  The contraction order inside a block is free, so a
// block's 32 quants are read as eight aligned words: odd blocks start on a
// word boundary (34b + 2 = 0 mod 4); even blocks use seven aligned words
// (quants 2..29) and one word assembled from quants 0, 1, 30, 31; the staged
// activation uses the same order.  Per block and row the limb sums are
// combined exactly in int32 (|sum| < 2^27), converted once to float and
// scaled by the block's d, as DotVecQ8_0 scales its block sums
// (pkg/quant/quant.go:320-339).
namespace q80m {
constexpr int kUnitBytes = 16 * 272;  // one 16-row x 256-column unit of raw blocks
constexpr int kUnitX = 1040;          // staged activation bytes per unit: 8 blocks x 128 + scale
constexpr int kSmemMax = 227 * 1024 - 256;
constexpr int kCoresidentSmem = 110 * 1024;

struct Params {
  const uint8_t* w;
  float* y;
  const float* x;
  long long rowb;
  int rows, nku, ntiles, ctas;
  int x_off, slot_off;
};

// Element of block b carried by byte j of slot word i (see above).
GI_DEVINL int kslot(int b, int i, int j) {
  if (b & 1) return 4 * i + j;
  if (i < 7) return 2 + 4 * i + j;
  return j < 2 ? j : 28 + j;
}

// Stage one unit (256 columns) of x at xu: per block b, [limb n][t][slot t,
// slot 4+t][4 bytes] (128 bytes), then float 2^-e at 1024.  Lane L owns
// block L/4 and the slot words t = L%4 and 4+t.
GI_DEVINL void stage_unit(uint8_t* xu, const float* xunit, int lane) {
  const int b = lane >> 2, t = lane & 3;
  float v[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = xunit[32 * b + kslot(b, t, j)];
    v[4 + j] = xunit[32 * b + kslot(b, 4 + t, j)];
  }
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
  m = warp_max(m);
  int e = 0;
  if (m > 0.f && m <= 3.0e38f) e = min(126, max(-126, 29 - ilogbf(m)));  // max |x| * 2^e < 2^30
  const float s = exp2i(e);
  uint32_t u[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) u[j] = ((uint32_t)__float2int_rn(v[j] * s) + 0x80808080u) ^ 0x80808080u;
  const uint32_t base = smem_u32(xu) + b * 128 + t * 8;
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const uint32_t k = 3u - (uint32_t)n;  // limb n is byte 3-n
    const uint32_t lo = q4k::gather_byte(u[0], u[1], u[2], u[3], k);
    const uint32_t hi = q4k::gather_byte(u[4], u[5], u[6], u[7], k);
    sts64(base + n * 32, (uint64_t)lo | ((uint64_t)hi << 32));
  }
  if (lane == 0) reinterpret_cast<float*>(xu + 1024)[0] = exp2i(-e);
}

// Warp w stages the column blocks w, w + W, ...; with cta_sync false it
// waits only for its own stores (its caller's warps read no other blocks).
template <int W>
__device__ void stage_x(uint8_t* xs, const Params& p, bool cta_sync) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int u = warp; u < p.nku; u += W) stage_unit(xs + u * kUnitX, p.x + 256 * u, lane);
  if (cta_sync)
    __syncthreads();
  else
    __syncwarp();
}

GI_DEVINL float h2f(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// One unit: rows g and g+8 of a 16-row tile.  stage: [16 rows][272 bytes];
// xu: the unit's staged activations.  Wt: this lane's limb weight (lanes 0,
// 1 hold limbs 0-1 and 2-3; lanes 2, 3 hold the zero columns 4-7).
GI_DEVINL void compute_unit(uint32_t stage, uint32_t xu, int g, int t, float Wt, float& yA, float& yB) {
  const uint32_t rowA = stage + g * 272, rowB = rowA + 8 * 272;
  float aA = 0.f, aB = 0.f;
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    uint32_t a0, a1, a2, a3;  // rows g, g+8: slot t; rows g, g+8: slot 4+t
    if (b & 1) {
      const uint32_t o = 34 * b + 2;
      a0 = lds32(rowA + o + 4 * t);
      a1 = lds32(rowB + o + 4 * t);
      a2 = lds32(rowA + o + 16 + 4 * t);
      a3 = lds32(rowB + o + 16 + 4 * t);
    } else {
      const uint32_t o = 34 * b;  // word u_i at o + 4i; quants 0..31 at o + 2 ..
      a0 = lds32(rowA + o + 4 + 4 * t);
      a1 = lds32(rowB + o + 4 + 4 * t);
      const uint32_t i2 = t < 3 ? 20 + 4 * t : 0;  // u_{5+t}, or u_0 for the assembled word
      const uint32_t wA = lds32(rowA + o + i2), wB = lds32(rowB + o + i2);
      const uint32_t eA = lds32(rowA + o + 32), eB = lds32(rowB + o + 32);
      a2 = t < 3 ? wA : prmt(wA, eA, 0x5432u);
      a3 = t < 3 ? wB : prmt(wB, eB, 0x5432u);
    }
    uint64_t xb = 0;
    if (g < 4) xb = lds64(xu + b * 128 + g * 32 + t * 8);
    int d[4] = {0, 0, 0, 0};
    imma_16832s(d, a0, a1, a2, a3, (uint32_t)xb, (uint32_t)(xb >> 32));
    const float dA = h2f(lds16(rowA + 34 * b)), dB = h2f(lds16(rowB + 34 * b));
    aA = fmaf((float)(d[0] * 256 + d[1]), dA, aA);
    aB = fmaf((float)(d[2] * 256 + d[3]), dB, aB);
  }
  const float inv = __uint_as_float(lds32(xu + 1024));
  yA = fmaf(aA * Wt, inv, yA);
  yB = fmaf(aB * Wt, inv, yB);
}

template <int W, int S>
__global__ void __launch_bounds__(W * 32, W == 8 ? 2 : 1) gemv_q80m_kernel(const Params p) {
  constexpr int kWarps = W;
  extern __shared__ __align__(16) uint8_t smem[];
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int c = blockIdx.x;
  const int T0 = (int)((long long)p.ntiles * c / p.ctas), T1 = (int)((long long)p.ntiles * (c + 1) / p.ctas);
  const int ntl = T1 - T0, n = ntl * p.nku;
  const uint32_t ring = smem_u32(smem) + warp * S * kUnitBytes;
  uint8_t* xs = smem + p.x_off;
  const uint32_t xs_s = smem_u32(xs);
  float* slots = reinterpret_cast<float*>(smem + p.slot_off);  // [ntl][kWarps][16]
  const uint64_t pol = l2_evict_first_policy();
  // each warp zeroes its own partial slots (other warps read them only
  // after the CTA barrier that ends the streaming loop)
  for (int i = lane; i < ntl * 16; i += 32) slots[((i >> 4) * kWarps + warp) * 16 + (i & 15)] = 0.f;

  // Request cursor: lane L copies row L/2 of the unit, chunks L%2, L%2 + 2,
  // ... (adjacent lanes fetch adjacent 16-byte chunks of a row).
  const int crow = lane >> 1, cpar = lane & 1;
  int ltile = warp / p.nku, lku = warp - ltile * p.nku;
  int next = warp;
  const uint8_t* src = nullptr;
  auto seek = [&]() {
    src = p.w + (long long)min((T0 + ltile) * 16 + crow, p.rows - 1) * p.rowb + lku * 272;
  };
  if (next < n) seek();
  const uint32_t dst = ring + crow * 272 + 16 * cpar;
  auto request = [&](int stage) {  // always commits one group (possibly empty)
    if (next < n) {
      const uint32_t o = (uint32_t)stage * kUnitBytes;
#pragma unroll
      for (int i = 0; i < 9; ++i)
        if (cpar + 2 * i < 17) cp_async16_hint(dst + o + 32 * i, src + 16 * cpar + 32 * i, pol);
      next += kWarps;
      lku += kWarps;
      if (lku < p.nku) {
        src += kWarps * 272;
      } else {
        do {
          lku -= p.nku;
          ++ltile;
        } while (lku >= p.nku);
        if (next < n) seek();
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s = 0; s < S; ++s) request(s);
  griddep_wait();
  // no CTA barrier when warp w computes only the blocks it staged (the
  // column blocks a multiple of the warps), as in the Q4_K kernel
  stage_x<W>(xs, p, p.nku % kWarps != 0);

  const float Wt = t == 0 ? 65536.f : (t == 1 ? 1.f : 0.f);
  int ctile = warp / p.nku, cku = warp - ctile * p.nku;
  uint32_t cx = xs_s + cku * kUnitX;
  float yA = 0.f, yB = 0.f;
  int stage = 0;
  for (int i = warp; i < n; i += kWarps) {
    cp_async_wait<S - 1>();
    __syncwarp();
    compute_unit(ring + stage * kUnitBytes, cx, g, t, Wt, yA, yB);
    __syncwarp();
    request(stage);
    stage = stage + 1 == S ? 0 : stage + 1;
    const int tile = ctile;
    cku += kWarps;
    if (cku < p.nku) {
      cx += kWarps * kUnitX;
    } else {
      do {
        cku -= p.nku;
        ++ctile;
      } while (cku >= p.nku);
      cx = xs_s + cku * kUnitX;
    }
    if (ctile != tile || i + kWarps >= n) {  // this warp is done with `tile`
      float vA = yA + __shfl_xor_sync(0xffffffffu, yA, 1);
      float vB = yB + __shfl_xor_sync(0xffffffffu, yB, 1);
      vA += __shfl_xor_sync(0xffffffffu, vA, 2);
      vB += __shfl_xor_sync(0xffffffffu, vB, 2);
      yA = 0.f;
      yB = 0.f;
      if (t == 0) {
        float* sl = slots + (tile * kWarps + warp) * 16;
        sl[g] = vA;
        sl[g + 8] = vB;
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  for (int tl = warp; tl < ntl; tl += kWarps) {
    if (lane < 16) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) sum += slots[(tl * kWarps + w) * 16 + lane];
      const int row = (T0 + tl) * 16 + lane;
      if (row < p.rows) p.y[row] = sum;
    }
  }
}

struct Layout {
  int warps, ctas, stages, x_off, slot_off, smem;
};

Layout layout(int64_t rows, int64_t cols, const GemvLaunch& L) {
  Layout o;
  const int nku = (int)(cols / 256), ntiles = (int)((rows + 15) / 16);
  o.ctas = ntiles < L.sm_count ? ntiles : L.sm_count;
  const int max_tiles = (ntiles + o.ctas - 1) / o.ctas;
  bool large = o.ctas < L.sm_count || (long long)ntiles * nku >= 64LL * o.ctas;
  const int xbytes = nku * kUnitX;
  if (large && xbytes + max_tiles * 16 * 64 + 16 * 2 * kUnitBytes > kSmemMax) large = false;
  o.warps = large ? 16 : 8;
  const int fixed = xbytes + max_tiles * o.warps * 64;
  o.stages = 3;
  while (o.stages > 2 && fixed + o.warps * o.stages * kUnitBytes > kCoresidentSmem) --o.stages;
  o.x_off = o.warps * o.stages * kUnitBytes;
  o.slot_off = o.x_off + xbytes;
  o.smem = o.slot_off + max_tiles * o.warps * 64;
  return o;
}

int launch(float* y, const float* x, const uint8_t* w, int64_t rows, int64_t cols, const GemvLaunch& L,
           cudaStream_t stream) {
  const Layout o = layout(rows, cols, L);
  if (o.smem > kSmemMax) return -4;
  Params p;
  p.w = w;
  p.y = y;
  p.x = x;
  p.rowb = (cols / 32) * 34;
  p.rows = (int)rows;
  p.nku = (int)(cols / 256);
  p.ntiles = (int)((rows + 15) / 16);
  p.ctas = o.ctas;
  p.x_off = o.x_off;
  p.slot_off = o.slot_off;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(o.ctas);
  cfg.blockDim = dim3(o.warps * 32);
  cfg.dynamicSmemBytes = o.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  cudaError_t e;
  switch ((o.warps == 16 ? 10 : 0) + o.stages) {
    case 2: e = cudaLaunchKernelEx(&cfg, gemv_q80m_kernel<8, 2>, p); break;
    case 3: e = cudaLaunchKernelEx(&cfg, gemv_q80m_kernel<8, 3>, p); break;
    case 12: e = cudaLaunchKernelEx(&cfg, gemv_q80m_kernel<16, 2>, p); break;
    case 13: e = cudaLaunchKernelEx(&cfg, gemv_q80m_kernel<16, 3>, p); break;
    default: return -4;
  }
  return e == cudaSuccess ? 0 : -5;
}

template <int W, int S>
cudaError_t prepare_one() {
  cudaError_t e = cudaFuncSetAttribute(gemv_q80m_kernel<W, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  return e == cudaSuccess ? set_max_shared_carveout(gemv_q80m_kernel<W, S>) : e;
}

int prepare() {
  cudaError_t e = prepare_one<8, 2>();
  if (e == cudaSuccess) e = prepare_one<8, 3>();
  if (e == cudaSuccess) e = prepare_one<16, 2>();
  if (e == cudaSuccess) e = prepare_one<16, 3>();
  return e == cudaSuccess ? 0 : -5;
}
}  // namespace q80m

// ---------------------------------------------------------------------------
// Shared helpers of the 4-rows-per-warp fp32 kernels (Q8_0, Q6_K).
namespace rowwarp {
constexpr int kWarps = 8;
constexpr int kRows = 4;  // rows per warp: each activation load serves 4 rows
constexpr uint32_t kF32Magic = 0x4B000000u;  // 2^23 as float bits

// Copy bytes [g, g+n) of a weight buffer ending at `end` into smem `dst`,
// starting at the 16-byte boundary at or below g.  Returns g's offset in
// dst.  dst must hold ((g&15) + n + 15)/16 + 1 vectors.
GI_DEVINL int stage_bytes(uint4* dst, const uint8_t* gp, int n, const uint8_t* end,
                          int lane) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(gp);
  const uint8_t* base = reinterpret_cast<const uint8_t*>(a & ~(uintptr_t)15);
  const int off = (int)(a & 15);
  const int nvec = (off + n + 15) >> 4;
  for (int v = lane; v < nvec; v += 32) {
    const uint8_t* src = base + 16 * v;
    if (src + 16 <= end) {
      dst[v] = ldg_stream(src);
    } else {
      uint8_t tmp[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) tmp[i] = src + i < end ? src[i] : 0;
      dst[v] = *reinterpret_cast<const uint4*>(tmp);
    }
  }
  return off;
}

// 32-bit little-endian read at any byte offset of a staged buffer.
GI_DEVINL uint32_t lds_u32(const uint32_t* s, int ofs) {
  const uint32_t w0 = s[ofs >> 2], w1 = s[(ofs >> 2) + 1];
  return __funnelshift_r(w0, w1, (ofs & 3) * 8);
}
GI_DEVINL uint32_t lds_u16(const uint8_t* s, int ofs) {
  return *reinterpret_cast<const uint16_t*>(s + ofs);
}
GI_DEVINL float f16bits_to_f32(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// Byte i of v as an exact float, minus `bias` (v's bytes are unsigned).
GI_DEVINL float byte_as_float(uint32_t v, uint32_t sel, float bias) {
  return __uint_as_float(prmt(v, kF32Magic, sel)) - bias;
}
}  // namespace rowwarp

// ------------------------------- Q8_0 ------------------------------------
namespace q80 {
using namespace rowwarp;
constexpr int kChunkBlocks = 32;                         // blocks staged per row
constexpr int kVecPerRow = (15 + kChunkBlocks * 34 + 15) / 16 + 1;  // 70

__global__ void __launch_bounds__(kWarps * 32) gemv_q80_kernel(
    float* __restrict__ y, const float* __restrict__ x, const uint8_t* __restrict__ w,
    const uint8_t* wend, long long rowb, int rows, int nb) {
  __shared__ uint4 stage[kWarps][kRows][kVecPerRow];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = (blockIdx.x * kWarps + warp) * kRows;
  griddep_wait();
  griddep_launch_dependents();
  if (r0 >= rows) return;
  const int bq = lane >> 2, j = lane & 3;  // block within an 8-block group, quarter of it
  float acc[kRows];
#pragma unroll
  for (int i = 0; i < kRows; ++i) acc[i] = 0.f;
  for (int c0 = 0; c0 < nb; c0 += kChunkBlocks) {
    const int nblk = min(kChunkBlocks, nb - c0);
    int off[kRows];
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int r = min(r0 + i, rows - 1);
      off[i] = stage_bytes(stage[warp][i], w + (long long)r * rowb + 34LL * c0, nblk * 34, wend, lane);
    }
    __syncwarp();
#pragma unroll
    for (int sub = 0; sub < kChunkBlocks / 8; ++sub) {
      const int bl = sub * 8 + bq;
      if (bl < nblk) {
        const float4* xp = reinterpret_cast<const float4*>(x + 32LL * (c0 + bl) + 8 * j);
        const float4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
#pragma unroll
        for (int i = 0; i < kRows; ++i) {
          const uint8_t* sb = reinterpret_cast<const uint8_t*>(stage[warp][i]);
          const uint32_t* sw = reinterpret_cast<const uint32_t*>(stage[warp][i]);
          const int base = off[i] + 34 * bl;
          const float d = f16bits_to_f32(lds_u16(sb, base));
          const uint32_t q0 = lds_u32(sw, base + 2 + 8 * j) ^ 0x80808080u;
          const uint32_t q1 = lds_u32(sw, base + 6 + 8 * j) ^ 0x80808080u;
          const float bias = 8388736.f;  // 2^23 + 128
          float s = byte_as_float(q0, 0x7440u, bias) * x0.x;
          s = fmaf(byte_as_float(q0, 0x7441u, bias), x0.y, s);
          s = fmaf(byte_as_float(q0, 0x7442u, bias), x0.z, s);
          s = fmaf(byte_as_float(q0, 0x7443u, bias), x0.w, s);
          s = fmaf(byte_as_float(q1, 0x7440u, bias), x1.x, s);
          s = fmaf(byte_as_float(q1, 0x7441u, bias), x1.y, s);
          s = fmaf(byte_as_float(q1, 0x7442u, bias), x1.z, s);
          s = fmaf(byte_as_float(q1, 0x7443u, bias), x1.w, s);
          acc[i] = fmaf(s, d, acc[i]);
        }
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    const float v = warp_sum(acc[i]);
    if (lane == 0 && r0 + i < rows) y[r0 + i] = v;
  }
}

// Ring variant for rows of whole 256-column groups (nb % 8 == 0, so every
// row and every 32-block chunk starts on a 16-byte boundary): each warp owns
// R rows and streams them chunk by chunk through a two-stage cp.async ring,
// the first two chunks requested before the kernel waits on its
// predecessor; the arithmetic is the staged kernel's.
constexpr int kRingChunkBytes = kChunkBlocks * 34;  // 1088
// Slot stride: lds_u32 reads the word after a misaligned offset, up to 4
// bytes past the chunk, so every slot carries 16 bytes of padding.
constexpr int kRingSlot = kRingChunkBytes + 16;
template <int R>
__global__ void __launch_bounds__(kWarps * 32) gemv_q80_ring_kernel(float* __restrict__ y, const float* __restrict__ x,
                                                                    const uint8_t* __restrict__ w, long long rowb,
                                                                    int rows, int nb) {
  extern __shared__ __align__(16) uint8_t smem[];  // [warp][stage][R][kRingSlot]
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = (blockIdx.x * kWarps + warp) * R;
  const int nchunks = (nb + kChunkBlocks - 1) / kChunkBlocks;
  uint8_t* ring = smem + (size_t)warp * 2 * R * kRingSlot;
  const uint64_t pol = l2_evict_first_policy();
  auto request = [&](int ch) {  // always commits one group (possibly empty)
    if (ch < nchunks && r0 < rows) {
      const int nvec = min(kChunkBlocks, nb - ch * kChunkBlocks) * 34 / 16;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const uint8_t* src = w + (long long)min(r0 + i, rows - 1) * rowb + (long long)ch * kRingChunkBytes;
        const uint32_t dst = smem_u32(ring + ((ch & 1) * R + i) * kRingSlot);
        for (int v = lane; v < nvec; v += 32) cp_async16_hint(dst + 16 * v, src + 16 * v, pol);
      }
    }
    cp_async_commit();
  };
  request(0);
  request(1);
  griddep_wait();
  if (r0 >= rows) return;  // nothing was requested
  const int bq = lane >> 2, j = lane & 3;  // block within an 8-block group, quarter of it
  float acc[R];
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = 0.f;
  for (int ch = 0; ch < nchunks; ++ch) {
    cp_async_wait<1>();
    __syncwarp();
    const int c0 = ch * kChunkBlocks, nblk = min(kChunkBlocks, nb - c0);
#pragma unroll
    for (int sub = 0; sub < kChunkBlocks / 8; ++sub) {
      const int bl = sub * 8 + bq;
      if (bl < nblk) {
        const float4* xp = reinterpret_cast<const float4*>(x + 32LL * (c0 + bl) + 8 * j);
        const float4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const uint8_t* sb = ring + ((ch & 1) * R + i) * kRingSlot;
          const uint32_t* sw = reinterpret_cast<const uint32_t*>(sb);
          const int base = 34 * bl;
          const float d = f16bits_to_f32(lds_u16(sb, base));
          const uint32_t q0 = lds_u32(sw, base + 2 + 8 * j) ^ 0x80808080u;
          const uint32_t q1 = lds_u32(sw, base + 6 + 8 * j) ^ 0x80808080u;
          const float bias = 8388736.f;  // 2^23 + 128
          float s = byte_as_float(q0, 0x7440u, bias) * x0.x;
          s = fmaf(byte_as_float(q0, 0x7441u, bias), x0.y, s);
          s = fmaf(byte_as_float(q0, 0x7442u, bias), x0.z, s);
          s = fmaf(byte_as_float(q0, 0x7443u, bias), x0.w, s);
          s = fmaf(byte_as_float(q1, 0x7440u, bias), x1.x, s);
          s = fmaf(byte_as_float(q1, 0x7441u, bias), x1.y, s);
          s = fmaf(byte_as_float(q1, 0x7442u, bias), x1.z, s);
          s = fmaf(byte_as_float(q1, 0x7443u, bias), x1.w, s);
          acc[i] = fmaf(s, d, acc[i]);
        }
      }
    }
    __syncwarp();
    request(ch + 2);
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const float v = warp_sum(acc[i]);
    if (lane == 0 && r0 + i < rows) y[r0 + i] = v;
  }
}

// R = 4 rows per warp, or 2 when 4 would leave SMs without a CTA.
int launch_ring(float* y, const float* x, const uint8_t* w, int64_t rows, int64_t cols, const GemvLaunch& L,
                cudaStream_t stream) {
  const int per_cta4 = kWarps * 4;
  const int R = (rows + per_cta4 - 1) / per_cta4 >= L.sm_count ? 4 : 2;
  const int64_t ctas = (rows + (int64_t)kWarps * R - 1) / ((int64_t)kWarps * R);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = (size_t)kWarps * 2 * R * kRingSlot;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  const long long rowb = (cols / 32) * 34;
  const cudaError_t e = R == 4 ? cudaLaunchKernelEx(&cfg, gemv_q80_ring_kernel<4>, y, x, w, rowb, (int)rows,
                                                    (int)(cols / 32))
                               : cudaLaunchKernelEx(&cfg, gemv_q80_ring_kernel<2>, y, x, w, rowb, (int)rows,
                                                    (int)(cols / 32));
  return e == cudaSuccess ? 0 : -5;
}

int prepare_ring() {
  const int smem4 = kWarps * 2 * 4 * kRingSlot;
  if (cudaFuncSetAttribute(gemv_q80_ring_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem4) != cudaSuccess)
    return -5;
  if (set_max_shared_carveout(gemv_q80_ring_kernel<4>) != cudaSuccess) return -5;
  return set_max_shared_carveout(gemv_q80_ring_kernel<2>) == cudaSuccess ? 0 : -5;
}
}  // namespace q80

// ------------------------------- Q6_K ------------------------------------
namespace q6k {
using namespace rowwarp;
constexpr int kChunkSB = 4;                                  // super-blocks staged per row
constexpr int kVecPerRow = (15 + kChunkSB * 210 + 15) / 16 + 1;  // 55

__global__ void __launch_bounds__(kWarps * 32) gemv_q6k_kernel(
    float* __restrict__ y, const float* __restrict__ x, const uint8_t* __restrict__ w,
    const uint8_t* wend, long long rowb, int rows, int nsb) {
  __shared__ uint4 stage[kWarps][kRows][kVecPerRow];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = (blockIdx.x * kWarps + warp) * kRows;
  griddep_wait();
  griddep_launch_dependents();
  if (r0 >= rows) return;
  const int q = lane >> 3, j = lane & 7;  // super-block within the chunk, l-quad 4j..4j+3
  const uint32_t jsel = (uint32_t)(j >> 2);
  float acc[kRows];
#pragma unroll
  for (int i = 0; i < kRows; ++i) acc[i] = 0.f;
  for (int s0 = 0; s0 < nsb; s0 += kChunkSB) {
    const int n4 = min(kChunkSB, nsb - s0);
    int off[kRows];
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int r = min(r0 + i, rows - 1);
      off[i] = stage_bytes(stage[warp][i], w + (long long)r * rowb + 210LL * s0, n4 * 210, wend, lane);
    }
    __syncwarp();
    if (q < n4) {
      const float* xb = x + 256LL * (s0 + q) + 4 * j;
      float4 xv[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int k = 0; k < 4; ++k) xv[n][k] = __ldg(reinterpret_cast<const float4*>(xb + 128 * n + 32 * k));
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const uint8_t* sb = reinterpret_cast<const uint8_t*>(stage[warp][i]);
        const uint32_t* sw = reinterpret_cast<const uint32_t*>(stage[warp][i]);
        const int base = off[i] + 210 * q;
        const float d = f16bits_to_f32(lds_u16(sb, base + 208));
        uint32_t S[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) S[m] = lds_u32(sw, base + 192 + 4 * m) ^ 0x80808080u;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          const uint32_t L0 = lds_u32(sw, base + 64 * n + 4 * j);
          const uint32_t L1 = lds_u32(sw, base + 64 * n + 32 + 4 * j);
          const uint32_t Q = lds_u32(sw, base + 128 + 32 * n + 4 * j);
          uint32_t V[4];
          V[0] = (L0 & 0x0F0F0F0Fu) | ((Q << 4) & 0x30303030u);
          V[1] = (L1 & 0x0F0F0F0Fu) | ((Q << 2) & 0x30303030u);
          V[2] = ((L0 >> 4) & 0x0F0F0F0Fu) | (Q & 0x30303030u);
          V[3] = ((L1 >> 4) & 0x0F0F0F0Fu) | ((Q >> 2) & 0x30303030u);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // scale of sub-block 8n + 2k + (l/16), l = 4j..4j+3
            const uint32_t scw = S[2 * n + (k >> 1)];
            const float sc = byte_as_float(scw, 0x7440u + 2u * (k & 1) + jsel, 8388736.f);
            const float ds = d * sc;  // (d * sc) as DequantizeQ6_K forms it
            const float bias = 8388640.f;  // 2^23 + 32
            float s = byte_as_float(V[k], 0x7440u, bias) * xv[n][k].x;
            s = fmaf(byte_as_float(V[k], 0x7441u, bias), xv[n][k].y, s);
            s = fmaf(byte_as_float(V[k], 0x7442u, bias), xv[n][k].z, s);
            s = fmaf(byte_as_float(V[k], 0x7443u, bias), xv[n][k].w, s);
            acc[i] = fmaf(ds, s, acc[i]);
          }
        }
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    const float v = warp_sum(acc[i]);
    if (lane == 0 && r0 + i < rows) y[r0 + i] = v;
  }
}

// Ring variant for rows of whole 2048-column groups (nsb % 8 == 0, so rows
// and 8-super-block chunks start on 16-byte boundaries): each warp owns R
// rows and streams them through a two-stage cp.async ring, the first two
// chunks requested before the kernel waits on its predecessor; the
// arithmetic is the staged kernel's.
constexpr int kRingSB = 8;
constexpr int kRingChunkBytes = kRingSB * 210;  // 1680
constexpr int kRingSlot = kRingChunkBytes + 16;  // padded like Q8_0's slots
template <int R>
__global__ void __launch_bounds__(kWarps * 32) gemv_q6k_ring_kernel(float* __restrict__ y, const float* __restrict__ x,
                                                                    const uint8_t* __restrict__ w, long long rowb,
                                                                    int rows, int nsb) {
  extern __shared__ __align__(16) uint8_t smem[];  // [warp][stage][R][kRingSlot]
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = (blockIdx.x * kWarps + warp) * R;
  const int nchunks = (nsb + kRingSB - 1) / kRingSB;
  uint8_t* ring = smem + (size_t)warp * 2 * R * kRingSlot;
  const uint64_t pol = l2_evict_first_policy();
  auto request = [&](int ch) {  // always commits one group (possibly empty)
    if (ch < nchunks && r0 < rows) {
      const int nvec = min(kRingSB, nsb - ch * kRingSB) * 210 / 16;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const uint8_t* src = w + (long long)min(r0 + i, rows - 1) * rowb + (long long)ch * kRingChunkBytes;
        const uint32_t dst = smem_u32(ring + ((ch & 1) * R + i) * kRingSlot);
        for (int v = lane; v < nvec; v += 32) cp_async16_hint(dst + 16 * v, src + 16 * v, pol);
      }
    }
    cp_async_commit();
  };
  request(0);
  request(1);
  griddep_wait();
  if (r0 >= rows) return;  // nothing was requested
  const int q = lane >> 3, j = lane & 7;  // super-block within a 4-block group, l-quad 4j..4j+3
  const uint32_t jsel = (uint32_t)(j >> 2);
  float acc[R];
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = 0.f;
  for (int ch = 0; ch < nchunks; ++ch) {
    cp_async_wait<1>();
    __syncwarp();
    const int s0 = ch * kRingSB, n8 = min(kRingSB, nsb - s0);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int sbk = q + 4 * half;
      if (sbk < n8) {
        const float* xb = x + 256LL * (s0 + sbk) + 4 * j;
        float4 xv[2][4];
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int k = 0; k < 4; ++k) xv[n][k] = __ldg(reinterpret_cast<const float4*>(xb + 128 * n + 32 * k));
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const uint8_t* sb = ring + ((ch & 1) * R + i) * kRingSlot;
          const uint32_t* sw = reinterpret_cast<const uint32_t*>(sb);
          const int base = 210 * sbk;
          const float d = f16bits_to_f32(lds_u16(sb, base + 208));
          uint32_t S[4];
#pragma unroll
          for (int m = 0; m < 4; ++m) S[m] = lds_u32(sw, base + 192 + 4 * m) ^ 0x80808080u;
#pragma unroll
          for (int n = 0; n < 2; ++n) {
            const uint32_t L0 = lds_u32(sw, base + 64 * n + 4 * j);
            const uint32_t L1 = lds_u32(sw, base + 64 * n + 32 + 4 * j);
            const uint32_t Q = lds_u32(sw, base + 128 + 32 * n + 4 * j);
            uint32_t V[4];
            V[0] = (L0 & 0x0F0F0F0Fu) | ((Q << 4) & 0x30303030u);
            V[1] = (L1 & 0x0F0F0F0Fu) | ((Q << 2) & 0x30303030u);
            V[2] = ((L0 >> 4) & 0x0F0F0F0Fu) | (Q & 0x30303030u);
            V[3] = ((L1 >> 4) & 0x0F0F0F0Fu) | ((Q >> 2) & 0x30303030u);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              // scale of sub-block 8n + 2k + (l/16), l = 4j..4j+3
              const uint32_t scw = S[2 * n + (k >> 1)];
              const float sc = byte_as_float(scw, 0x7440u + 2u * (k & 1) + jsel, 8388736.f);
              const float ds = d * sc;  // (d * sc) as DequantizeQ6_K forms it
              const float bias = 8388640.f;  // 2^23 + 32
              float sum = byte_as_float(V[k], 0x7440u, bias) * xv[n][k].x;
              sum = fmaf(byte_as_float(V[k], 0x7441u, bias), xv[n][k].y, sum);
              sum = fmaf(byte_as_float(V[k], 0x7442u, bias), xv[n][k].z, sum);
              sum = fmaf(byte_as_float(V[k], 0x7443u, bias), xv[n][k].w, sum);
              acc[i] = fmaf(ds, sum, acc[i]);
            }
          }
        }
      }
    }
    __syncwarp();
    request(ch + 2);
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const float v = warp_sum(acc[i]);
    if (lane == 0 && r0 + i < rows) y[r0 + i] = v;
  }
}

// R = 4 rows per warp, or 2 when 4 would leave SMs without a CTA.
int launch_ring(float* y, const float* x, const uint8_t* w, int64_t rows, int64_t cols, const GemvLaunch& L,
                cudaStream_t stream) {
  const int R = (rows + kWarps * 4 - 1) / (kWarps * 4) >= L.sm_count ? 4 : 2;
  const int64_t ctas = (rows + (int64_t)kWarps * R - 1) / ((int64_t)kWarps * R);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = (size_t)kWarps * 2 * R * kRingSlot;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  const long long rowb = (cols / 256) * 210;
  const cudaError_t e = R == 4 ? cudaLaunchKernelEx(&cfg, gemv_q6k_ring_kernel<4>, y, x, w, rowb, (int)rows,
                                                    (int)(cols / 256))
                               : cudaLaunchKernelEx(&cfg, gemv_q6k_ring_kernel<2>, y, x, w, rowb, (int)rows,
                                                    (int)(cols / 256));
  return e == cudaSuccess ? 0 : -5;
}

int prepare_ring() {
  for (int R : {2, 4}) {
    const int smem = kWarps * 2 * R * kRingSlot;
    auto k = R == 4 ? gemv_q6k_ring_kernel<4> : gemv_q6k_ring_kernel<2>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -5;
    if (set_max_shared_carveout(k) != cudaSuccess) return -5;
  }
  return 0;
}
}  // namespace q6k

// ------------------------ Q6_K on the int8 tensor cores ---------------------
// Rows of whole 2048-column groups (rows then start on 16-byte boundaries:
// 8 x 210 = 1680 = 105 x 16).  The Q4_K / Q8_0 structure: a unit is 16 rows
// x 256 columns (one super-block per row), each CTA owns whole 16-row tiles,
// units are dealt to the warps round-robin and streamed through per-warp
// cp.async rings, every tile's per-warp partials are summed in fixed warp
// order.  A super-block is only 2-byte aligned: a unit stages, per row, the
// 14 aligned 16-byte chunks that cover it (224 bytes), so the block starts
// at byte (2 b) mod 16 of its row slot (b = the column block); odd b leave
// it 2 bytes off a word, and its words are read as two aligned words joined
// by a funnel shift.
//
// Arithmetic (DequantizeQ6_K, pkg/quant/quant.go:256-291): element 128n +
// 32j + l (n < 2, j < 4, l < 32) has q = 4 bits of ql[64n + 32(j&1) + l]
// (low nibble for j < 2) | 2 bits of qh[32n + l] (shift 2j) << 4, weight
// d * sc[8n + 2j + l/16] * (q - 32).  One m16n8k32 MMA (u8 x s8) per
// chunk (n, j): A = the unsigned 6-bit q of 16 rows x 32 elements in their
// natural order; B = the four balanced base-256 limbs of the 30-bit
// fixed-point activation, columns 0-3 carrying the limbs of the chunk's
// first sub-block (l < 16, zeros elsewhere), columns 4-7 those of the second
// (l >= 16); the accumulator starts at -32 x the column's limb sum, so the
// MMA yields the exact sum of (q - 32) * limb per (row, sub-block, limb).
// Each lane holds two limb columns of one sub-block and scales them by that
// sub-block's int8 scale in int32 (exact); a super-block leaves the integer
// domain through 4 int->float conversions per lane, scaled by d and 2^-e.
namespace q6m {
constexpr int kRowSlot = 224;                 // 14 aligned 16-byte chunks cover a 210-byte block
constexpr int kUnitBytes = 16 * kRowSlot;     // 3584
constexpr int kUnitX = 1296;                  // [chunk][limb][32 B] 1024, limb sums 256, 2^-e 16
constexpr int kSmemMax = 227 * 1024 - 256;
constexpr int kCoresidentSmem = 110 * 1024;

struct Params {
  const uint8_t* w;
  float* y;
  const float* x;
  long long rowb;
  int rows, nku, ntiles, ctas;
  int x_off, slot_off;
};

// Stage one unit (256 columns) of x at xu.  Chunk c = 4n + j holds the
// elements 128n + 32j + l; lane L owns chunk L/4 and its elements 4t..4t+3
// and 16+4t..16+4t+3 (t = L%4).  Layout: [c][limb][32 bytes, element order]
// at c*128; at 1024 + 32c + 8t the int32 pair (-32 x limb sum) of the
// chunk's columns 2t, 2t+1 (column k < 4: limb k over l < 16; k >= 4: limb
// k-4 over l >= 16); the float 2^-e at 1280.
GI_DEVINL void stage_unit(uint8_t* xu, const float* xunit, int lane) {
  const int c = lane >> 2, t = lane & 3;
  const int e0 = 128 * (c >> 2) + 32 * (c & 3);
  const float4 a = *reinterpret_cast<const float4*>(xunit + e0 + 4 * t);
  const float4 b = *reinterpret_cast<const float4*>(xunit + e0 + 16 + 4 * t);
  float m = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))),
                  fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
  m = warp_max(m);
  int e = 0;
  if (m > 0.f && m <= 3.0e38f) e = min(126, max(-126, 29 - ilogbf(m)));  // max |x| * 2^e < 2^30
  const float s = exp2i(e);
  uint32_t u[8];
  u[0] = ((uint32_t)__float2int_rn(a.x * s) + 0x80808080u) ^ 0x80808080u;
  u[1] = ((uint32_t)__float2int_rn(a.y * s) + 0x80808080u) ^ 0x80808080u;
  u[2] = ((uint32_t)__float2int_rn(a.z * s) + 0x80808080u) ^ 0x80808080u;
  u[3] = ((uint32_t)__float2int_rn(a.w * s) + 0x80808080u) ^ 0x80808080u;
  u[4] = ((uint32_t)__float2int_rn(b.x * s) + 0x80808080u) ^ 0x80808080u;
  u[5] = ((uint32_t)__float2int_rn(b.y * s) + 0x80808080u) ^ 0x80808080u;
  u[6] = ((uint32_t)__float2int_rn(b.z * s) + 0x80808080u) ^ 0x80808080u;
  u[7] = ((uint32_t)__float2int_rn(b.w * s) + 0x80808080u) ^ 0x80808080u;
  const uint32_t base = smem_u32(xu) + c * 128 + 4 * t;
  int sa[4], sb[4];  // this lane's limb sums over its 4 + 4 elements
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const uint32_t k = 3u - (uint32_t)n;  // limb n is byte 3-n
    const uint32_t lo = q4k::gather_byte(u[0], u[1], u[2], u[3], k);
    const uint32_t hi = q4k::gather_byte(u[4], u[5], u[6], u[7], k);
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(base + n * 32), "r"(lo) : "memory");
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(base + n * 32 + 16), "r"(hi) : "memory");
    sa[n] = (int)(int8_t)(lo) + (int)(int8_t)(lo >> 8) + (int)(int8_t)(lo >> 16) + (int)(int8_t)(lo >> 24);
    sb[n] = (int)(int8_t)(hi) + (int)(int8_t)(hi >> 8) + (int)(int8_t)(hi >> 16) + (int)(int8_t)(hi >> 24);
  }
#pragma unroll
  for (int n = 0; n < 4; ++n) {  // sums over the chunk's four lanes (lanes 4c..4c+3)
    sa[n] += __shfl_xor_sync(0xffffffffu, sa[n], 1);
    sa[n] += __shfl_xor_sync(0xffffffffu, sa[n], 2);
    sb[n] += __shfl_xor_sync(0xffffffffu, sb[n], 1);
    sb[n] += __shfl_xor_sync(0xffffffffu, sb[n], 2);
  }
  // lane t writes columns 2t, 2t+1: t < 2 -> limbs 2t, 2t+1 of the first
  // sub-block; t >= 2 -> limbs 2(t-2), 2(t-2)+1 of the second
  const int c0 = t < 2 ? (t == 0 ? sa[0] : sa[2]) : (t == 2 ? sb[0] : sb[2]);
  const int c1 = t < 2 ? (t == 0 ? sa[1] : sa[3]) : (t == 2 ? sb[1] : sb[3]);
  sts64(smem_u32(xu) + 1024 + 32 * c + 8 * t, (uint64_t)(uint32_t)(-32 * c0) | ((uint64_t)(uint32_t)(-32 * c1) << 32));
  if (lane == 0) reinterpret_cast<float*>(xu + 1280)[0] = exp2i(-e);
}

// Warp w stages the column blocks w, w + W, ...; with cta_sync false it
// waits only for its own stores (its caller's warps read no other blocks).
template <int W>
__device__ void stage_x(uint8_t* xs, const Params& p, bool cta_sync) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int u = warp; u < p.nku; u += W) stage_unit(xs + u * kUnitX, p.x + 256 * u, lane);
  if (cta_sync)
    __syncthreads();
  else
    __syncwarp();
}

// Word at a 2-byte-aligned shared address: one load, or (odd) two aligned
// loads joined by a funnel shift.
template <bool Odd>
GI_DEVINL uint32_t ldw(uint32_t a) {
  if (!Odd) return lds32(a);
  return __funnelshift_r(lds32(a - 2), lds32(a + 2), 16);
}

// Signed byte k of w, sign-extended.
GI_DEVINL int sbyte(uint32_t w, uint32_t k) { return (int)prmt(w, 0u, k | ((k | 8u) * 0x1110u)); }

// One unit: rows g and g+8 of a 16-row tile.  blk: row g's block in the
// stage (row g+8's is 8 slots on); xu: the unit's staged activations.
template <bool Odd>
GI_DEVINL void compute_unit(uint32_t blk, uint32_t xu, int g, int t, float W0, float W1, float& yA, float& yB) {
  const uint32_t bA = blk, bB = blk + 8 * kRowSlot;
  // scales of the two rows (16 signed bytes at 192)
  uint32_t sA[4], sB[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sA[i] = ldw<Odd>(bA + 192 + 4 * i);
    sB[i] = ldw<Odd>(bB + 192 + 4 * i);
  }
  const uint32_t hsel = t >= 2 ? 1u : 0u;  // this lane's sub-block within a chunk
  int iA0 = 0, iA1 = 0, iB0 = 0, iB1 = 0;
  const uint32_t xb_off = (uint32_t)((g & 3) * 32 + (g < 4 ? 0 : 16) + 4 * t);
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    // ql words (j even: L0, j odd: L1) and the qh word at quads 4t and 16+4t
    const uint32_t L0A = ldw<Odd>(bA + 64 * n + 4 * t), L0A2 = ldw<Odd>(bA + 64 * n + 16 + 4 * t);
    const uint32_t L1A = ldw<Odd>(bA + 64 * n + 32 + 4 * t), L1A2 = ldw<Odd>(bA + 64 * n + 48 + 4 * t);
    const uint32_t QA = ldw<Odd>(bA + 128 + 32 * n + 4 * t), QA2 = ldw<Odd>(bA + 128 + 32 * n + 16 + 4 * t);
    const uint32_t L0B = ldw<Odd>(bB + 64 * n + 4 * t), L0B2 = ldw<Odd>(bB + 64 * n + 16 + 4 * t);
    const uint32_t L1B = ldw<Odd>(bB + 64 * n + 32 + 4 * t), L1B2 = ldw<Odd>(bB + 64 * n + 48 + 4 * t);
    const uint32_t QB = ldw<Odd>(bB + 128 + 32 * n + 4 * t), QB2 = ldw<Odd>(bB + 128 + 32 * n + 16 + 4 * t);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // q = 4 bits of ql | 2 bits of qh << 4 (quant.go:270-282)
      auto q6 = [j](uint32_t L0, uint32_t L1, uint32_t Q) {
        const uint32_t L = (j & 1) ? L1 : L0;
        const uint32_t lo = (j >> 1) ? (L >> 4) & 0x0F0F0F0Fu : L & 0x0F0F0F0Fu;
        return lo | (((Q >> (2 * j)) << 4) & 0x30303030u);
      };
      const uint32_t a0 = q6(L0A, L1A, QA), a1 = q6(L0B, L1B, QB);
      const uint32_t a2 = q6(L0A2, L1A2, QA2), a3 = q6(L0B2, L1B2, QB2);
      const int c = 4 * n + j;
      const uint32_t xw = lds32(xu + c * 128 + xb_off);
      const uint64_t cs = lds64(xu + 1024 + 32 * c + 8 * t);
      int d[4] = {(int)(uint32_t)cs, (int)(uint32_t)(cs >> 32), (int)(uint32_t)cs, (int)(uint32_t)(cs >> 32)};
      imma_16832(d, a0, a1, a2, a3, g < 4 ? xw : 0u, g < 4 ? 0u : xw);
      // sub-block 8n + 2j + hsel: byte (2j + hsel) & 3 of scale word 2n + (2j + hsel) / 4
      const uint32_t sbk = 2u * (uint32_t)j + hsel;
      const int scA = sbyte(sA[2 * n + (sbk >> 2)], sbk & 3u), scB = sbyte(sB[2 * n + (sbk >> 2)], sbk & 3u);
      iA0 += d[0] * scA;
      iA1 += d[1] * scA;
      iB0 += d[2] * scB;
      iB1 += d[3] * scB;
    }
  }
  const float inv = __uint_as_float(lds32(xu + 1280));
  const float dA = __half2float(__ushort_as_half((unsigned short)lds16(bA + 208)));
  const float dB = __half2float(__ushort_as_half((unsigned short)lds16(bB + 208)));
  yA = fmaf(fmaf((float)iA0, W0, (float)iA1 * W1) * dA, inv, yA);
  yB = fmaf(fmaf((float)iB0, W0, (float)iB1 * W1) * dB, inv, yB);
}

template <int W, int S>
__global__ void __launch_bounds__(W * 32, W == 8 ? 2 : 1) gemv_q6m_kernel(const Params p) {
  constexpr int kWarps = W;
  extern __shared__ __align__(16) uint8_t smem[];
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int c = blockIdx.x;
  const int T0 = (int)((long long)p.ntiles * c / p.ctas), T1 = (int)((long long)p.ntiles * (c + 1) / p.ctas);
  const int ntl = T1 - T0, n = ntl * p.nku;
  const uint32_t ring = smem_u32(smem) + warp * S * kUnitBytes;
  uint8_t* xs = smem + p.x_off;
  const uint32_t xs_s = smem_u32(xs);
  float* slots = reinterpret_cast<float*>(smem + p.slot_off);  // [ntl][kWarps][16]
  const uint64_t pol = l2_evict_first_policy();
  // each warp zeroes its own partial slots (other warps read them only
  // after the CTA barrier that ends the streaming loop)
  for (int i = lane; i < ntl * 16; i += 32) slots[((i >> 4) * kWarps + warp) * 16 + (i & 15)] = 0.f;

  // Request cursor: lane L copies row L/2 of the unit, chunks L%2, L%2 + 2,
  // ..., L%2 + 12 of the 14 that cover the row's block.
  const int crow = lane >> 1, cpar = lane & 1;
  int ltile = warp / p.nku, lku = warp - ltile * p.nku;
  int next = warp;
  const uint8_t* src = nullptr;
  auto seek = [&]() {
    src = p.w + (long long)min((T0 + ltile) * 16 + crow, p.rows - 1) * p.rowb + ((210 * lku) & ~15);
  };
  if (next < n) seek();
  const uint32_t dst = ring + crow * kRowSlot + 16 * cpar;
  auto request = [&](int stage) {  // always commits one group (possibly empty)
    if (next < n) {
      const uint32_t o = (uint32_t)stage * kUnitBytes;
#pragma unroll
      for (int i = 0; i < 7; ++i) cp_async16_hint(dst + o + 32 * i, src + 16 * cpar + 32 * i, pol);
      next += kWarps;
      lku += kWarps;
      if (lku < p.nku) {
        src += (210 * lku & ~15) - (210 * (lku - kWarps) & ~15);
      } else {
        do {
          lku -= p.nku;
          ++ltile;
        } while (lku >= p.nku);
        if (next < n) seek();
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s = 0; s < S; ++s) request(s);
  griddep_wait();
  // no CTA barrier when warp w computes only the blocks it staged (the
  // column blocks a multiple of the warps), as in the Q4_K kernel
  stage_x<W>(xs, p, p.nku % kWarps != 0);

  // limb weights of this lane's two columns: limbs 2(t&1), 2(t&1)+1
  const float W0 = (t & 1) ? 256.f : 16777216.f, W1 = (t & 1) ? 1.f : 65536.f;
  int ctile = warp / p.nku, cku = warp - ctile * p.nku;
  uint32_t cx = xs_s + cku * kUnitX;
  float yA = 0.f, yB = 0.f;
  int stage = 0;
  for (int i = warp; i < n; i += kWarps) {
    cp_async_wait<S - 1>();
    __syncwarp();
    const uint32_t blk = ring + stage * kUnitBytes + g * kRowSlot + ((2 * cku) & 15);
    if (cku & 1)
      compute_unit<true>(blk, cx, g, t, W0, W1, yA, yB);
    else
      compute_unit<false>(blk, cx, g, t, W0, W1, yA, yB);
    __syncwarp();
    request(stage);
    stage = stage + 1 == S ? 0 : stage + 1;
    const int tile = ctile;
    cku += kWarps;
    if (cku < p.nku) {
      cx += kWarps * kUnitX;
    } else {
      do {
        cku -= p.nku;
        ++ctile;
      } while (cku >= p.nku);
      cx = xs_s + cku * kUnitX;
    }
    if (ctile != tile || i + kWarps >= n) {  // this warp is done with `tile`
      float vA = yA + __shfl_xor_sync(0xffffffffu, yA, 1);
      float vB = yB + __shfl_xor_sync(0xffffffffu, yB, 1);
      vA += __shfl_xor_sync(0xffffffffu, vA, 2);
      vB += __shfl_xor_sync(0xffffffffu, vB, 2);
      yA = 0.f;
      yB = 0.f;
      if (t == 0) {
        float* sl = slots + (tile * kWarps + warp) * 16;
        sl[g] = vA;
        sl[g + 8] = vB;
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  for (int tl = warp; tl < ntl; tl += kWarps) {
    if (lane < 16) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) sum += slots[(tl * kWarps + w) * 16 + lane];
      const int row = (T0 + tl) * 16 + lane;
      if (row < p.rows) p.y[row] = sum;
    }
  }
}

struct Layout {
  int warps, ctas, stages, x_off, slot_off, smem;
};

Layout layout(int64_t rows, int64_t cols, const GemvLaunch& L) {
  Layout o;
  const int nku = (int)(cols / 256), ntiles = (int)((rows + 15) / 16);
  o.ctas = ntiles < L.sm_count ? ntiles : L.sm_count;
  const int max_tiles = (ntiles + o.ctas - 1) / o.ctas;
  bool large = o.ctas < L.sm_count || (long long)ntiles * nku >= 64LL * o.ctas;
  const int xbytes = nku * kUnitX;
  if (large && xbytes + max_tiles * 16 * 64 + 16 * 2 * kUnitBytes > kSmemMax) large = false;
  o.warps = large ? 16 : 8;
  const int fixed = xbytes + max_tiles * o.warps * 64;
  o.stages = 3;
  while (o.stages > 2 && fixed + o.warps * o.stages * kUnitBytes > kCoresidentSmem) --o.stages;
  o.x_off = o.warps * o.stages * kUnitBytes;
  o.slot_off = o.x_off + xbytes;
  o.smem = o.slot_off + max_tiles * o.warps * 64;
  return o;
}

int launch(float* y, const float* x, const uint8_t* w, int64_t rows, int64_t cols, const GemvLaunch& L,
           cudaStream_t stream) {
  if (cols % 2048 != 0 || (reinterpret_cast<uintptr_t>(w) & 15) != 0) return -4;
  const Layout o = layout(rows, cols, L);
  if (o.smem > kSmemMax) return -4;
  Params p;
  p.w = w;
  p.y = y;
  p.x = x;
  p.rowb = (cols / 256) * 210;
  p.rows = (int)rows;
  p.nku = (int)(cols / 256);
  p.ntiles = (int)((rows + 15) / 16);
  p.ctas = o.ctas;
  p.x_off = o.x_off;
  p.slot_off = o.slot_off;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(o.ctas);
  cfg.blockDim = dim3(o.warps * 32);
  cfg.dynamicSmemBytes = o.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  cudaError_t e;
  switch ((o.warps == 16 ? 10 : 0) + o.stages) {
    case 2: e = cudaLaunchKernelEx(&cfg, gemv_q6m_kernel<8, 2>, p); break;
    case 3: e = cudaLaunchKernelEx(&cfg, gemv_q6m_kernel<8, 3>, p); break;
    case 12: e = cudaLaunchKernelEx(&cfg, gemv_q6m_kernel<16, 2>, p); break;
    case 13: e = cudaLaunchKernelEx(&cfg, gemv_q6m_kernel<16, 3>, p); break;
    default: return -4;
  }
  return e == cudaSuccess ? 0 : -5;
}

template <int W, int S>
cudaError_t prepare_one() {
  cudaError_t e = cudaFuncSetAttribute(gemv_q6m_kernel<W, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  return e == cudaSuccess ? set_max_shared_carveout(gemv_q6m_kernel<W, S>) : e;
}

int prepare() {
  cudaError_t e = prepare_one<8, 2>();
  if (e == cudaSuccess) e = prepare_one<8, 3>();
  if (e == cudaSuccess) e = prepare_one<16, 2>();
  if (e == cudaSuccess) e = prepare_one<16, 3>();
  return e == cudaSuccess ? 0 : -5;
}
}  // namespace q6m

int gemv_prepare_device() {
  if (q4k::prepare() != 0) return -5;
  if (set_max_shared_carveout(q80::gemv_q80_kernel) != cudaSuccess) return -5;
  if (q80::prepare_ring() != 0) return -5;
  if (q80m::prepare() != 0) return -5;
  if (q6k::prepare_ring() != 0) return -5;
  if (set_max_shared_carveout(q6k::gemv_q6k_kernel) != cudaSuccess) return -5;
  return 0;
}

int gemv_check(int qtype, int64_t rows, int64_t cols) {
  if (rows < 1 || cols < 1 || rows > (1LL << 30)) return -4;
  switch (qtype) {
    case kTypeQ4_K:
      return (cols % 256 == 0 && cols <= q4k::kMaxCols) ? 0 : -4;
    case kTypeQ6_K:
      return cols % 256 == 0 ? 0 : -4;
    case kTypeQ8_0:
      return cols % 32 == 0 ? 0 : -4;
    case kTypeF32:
      return cols % 4 == 0 ? 0 : -4;
    default:
      return -2;
  }
}

namespace f32 {
// float32 rows (GEMVEngine.MatMulF32, pkg/math/gemv.go:27-60): one warp per
// row, 16-byte loads, warp-shuffle sum.
__global__ void __launch_bounds__(256) gemv_f32_kernel(float* __restrict__ y, const float* __restrict__ x,
                                                       const float* __restrict__ w, int rows, int cols) {
  griddep_launch_dependents();
  griddep_wait();
  const int row = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* wr = reinterpret_cast<const float4*>(w + (size_t)row * cols);
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float s = 0.f;
  for (int i = lane; i < cols / 4; i += 32) {
    const float4 a = __ldg(wr + i), b = __ldg(x4 + i);
    s = fmaf(a.x, b.x, s);
    s = fmaf(a.y, b.y, s);
    s = fmaf(a.z, b.z, s);
    s = fmaf(a.w, b.w, s);
  }
  s = warp_sum(s);
  if (lane == 0) y[row] = s;
}
}  // namespace f32

template <typename K, typename... Args>
static int launch_rowwarp(K kernel, int64_t rows, const GemvLaunch& L, cudaStream_t stream,
                          Args... args) {
  const int64_t groups = (rows + rowwarp::kRows - 1) / rowwarp::kRows;
  const int64_t ctas = (groups + rowwarp::kWarps - 1) / rowwarp::kWarps;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(rowwarp::kWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess ? 0 : -5;
}

int gemv_launch(int qtype, float* y, const float* x, const void* w, size_t w_bytes, int64_t rows,
                int64_t cols, const GemvScratch& s, const GemvLaunch& L, cudaStream_t stream) {
  const int rc = gemv_check(qtype, rows, cols);
  if (rc) return rc;
  const int64_t rb = row_bytes(qtype, cols);
  if (w_bytes < (size_t)(rb * rows)) return -4;
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return -4;
  const uint8_t* wb = static_cast<const uint8_t*>(w);
  switch (qtype) {
    case kTypeQ4_K:
      if ((reinterpret_cast<uintptr_t>(w) & 15) != 0) return -4;
      return q4k::launch(1, &y, x, &w, &rows, cols, L, stream);
    case kTypeQ8_0:
      if (cols % 256 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
        const int r = q80m::launch(y, x, wb, rows, cols, L, stream);
        if (r != -4) return r;  // -4: the activation staging does not fit; the ring kernel takes it
        return q80::launch_ring(y, x, wb, rows, cols, L, stream);
      }
      return launch_rowwarp(q80::gemv_q80_kernel, rows, L, stream, y, x, wb, wb + w_bytes,
                            (long long)rb, (int)rows, (int)(cols / 32));
    case kTypeQ6_K:
      if (L.q6k_mma && cols % 2048 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
        static bool prepared[64] = {};  // kernel attributes, set on first use per device
        int dev = -1;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -5;
        if (!prepared[dev]) {
          if (q6m::prepare() != 0) return -5;
          prepared[dev] = true;
        }
        const int r = q6m::launch(y, x, wb, rows, cols, L, stream);
        if (r != -4) return r;  // -4: the activation staging does not fit; the ring kernel takes it
      }
      if (cols % 2048 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) return q6k::launch_ring(y, x, wb, rows, cols, L, stream);
      return launch_rowwarp(q6k::gemv_q6k_kernel, rows, L, stream, y, x, wb, wb + w_bytes,
                            (long long)rb, (int)rows, (int)(cols / 256));
    case kTypeF32: {
      if ((reinterpret_cast<uintptr_t>(w) & 15) != 0) return -4;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)((rows + 7) / 8));
      cfg.blockDim = dim3(256);
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = L.pdl ? 1 : 0;
      return cudaLaunchKernelEx(&cfg, f32::gemv_f32_kernel, y, x, reinterpret_cast<const float*>(w), (int)rows,
                                (int)cols) == cudaSuccess
                 ? 0
                 : -5;
    }
    default:
      return -2;
  }
}

int gemv_q4k_fused(int nmat, float* const* y, const float* x, const void* const* w, const size_t* w_bytes,
                   const int64_t* rows, int64_t cols, const GemvFuse& f, const GemvLaunch& L, cudaStream_t stream) {
  if (nmat < 1 || nmat > q4k::kMaxMats) return -4;
  for (int m = 0; m < nmat; ++m) {
    const int rc = gemv_check(kTypeQ4_K, rows[m], cols);
    if (rc) return rc;
    if (w_bytes[m] < (size_t)(row_bytes(kTypeQ4_K, cols) * rows[m])) return -4;
    if ((reinterpret_cast<uintptr_t>(w[m]) & 15) != 0) return -4;
  }
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return -4;
  if (f.xmode == kXNorm && (!f.x2 || (reinterpret_cast<uintptr_t>(f.x2) & 15) != 0)) return -4;
  return q4k::launch(nmat, y, x, w, rows, cols, L, stream, f);
}

int gemv_multi_launch(int qtype, int nmat, float* const* y, const float* x, const void* const* w,
                      const size_t* w_bytes, const int64_t* rows, int64_t cols, const GemvScratch& s,
                      const GemvLaunch& L, cudaStream_t stream) {
  if (nmat < 1 || nmat > q4k::kMaxMats) return -4;
  for (int m = 0; m < nmat; ++m) {
    const int rc = gemv_check(qtype, rows[m], cols);
    if (rc) return rc;
    if (w_bytes[m] < (size_t)(row_bytes(qtype, cols) * rows[m])) return -4;
  }
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return -4;
  if (qtype == kTypeQ4_K) {
    for (int m = 0; m < nmat; ++m)
      if ((reinterpret_cast<uintptr_t>(w[m]) & 15) != 0) return -4;
    return q4k::launch(nmat, y, x, w, rows, cols, L, stream);
  }
  for (int m = 0; m < nmat; ++m) {  // the CUDA-core kernels take one matrix per launch
    const int rc = gemv_launch(qtype, y[m], x, w[m], w_bytes[m], rows[m], cols, s, L, stream);
    if (rc) return rc;
  }
  return 0;
}

}  // namespace gi
