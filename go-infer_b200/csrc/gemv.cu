// gemv.cu -- decode-time quantised GEMV kernels (batch 1) for sm_100a.
//
// These replace GEMVEngine.MatMul{Q8_0,Q4_K,Q6_K} (pkg/math/gemv.go:98-203
// of go-infer) and the per-row DotVec* they call (pkg/quant/quant.go:320-339,
// 536-545).  Weights are the raw GGUF blocks, row-major, rows = output
// features; x and y are fp32 (go-infer never quantises activations).
//
// Q4_K kernel: one small CTA per SM, each owning a contiguous run of 16-row
// tiles.  Its 8 warps stream their units' raw super-blocks into per-warp
// shared-memory rings with cp.async (up to 4 units ahead, the first ones
// requested before the kernel waits on its predecessor), turn the 4-bit quants and 6-bit
// sub-block scales into exact fp16 products q*sc with one HFMA2 per two
// weights and multiply them on the tensor cores (mma.m16n8k16, fp32
// accumulate) against the activation split into exact fp16 hi+lo halves.
// The 6-bit mins ride along as a 17th MMA against per-half-sub-block
// activation sums.  Tiles split between warps are summed in fixed warp
// order through shared memory (deterministic).
//
// Q8_0 / Q6_K kernels: 4 rows per warp, fp32 CUDA-core dot products.  Their
// 34- and 210-byte blocks are only 2-byte aligned, so each warp stages its
// rows' bytes through shared memory with aligned 128-bit loads and realigns
// words with funnel shifts.
#include "common.cuh"
#include "gemv.cuh"

namespace gi {

int64_t row_bytes(int qtype, int64_t cols) {
  switch (qtype) {
    case kTypeQ8_0: return (cols / 32) * 34;
    case kTypeQ4_K: return (cols / 256) * 144;
    case kTypeQ6_K: return (cols / 256) * 210;
    default: return -1;
  }
}

namespace q4k {
// Work decomposition: a unit is 16 rows x 256 columns (one super-block per
// row, 2304 bytes).  Each CTA owns a contiguous run of whole 16-row tiles,
// so no reduction crosses CTAs; its units (tile-major) are split into
// contiguous ranges, one per warp, and tiles shared by two warps are summed
// in fixed warp order through shared memory (deterministic).  Each warp
// streams its units through a private ring of shared-memory stages with
// cp.async (16 bytes per lane, L1-bypassing, S units in flight, the first
// ones issued before the kernel waits on its predecessor); every lane
// stages exactly the quants it later reads, so a per-thread wait suffices
// (plus one warp barrier for the row headers).  Keeping the prefetch out of
// registers leaves the compiler room to interleave the decode/MMA chains.
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kUnitVec = 68;      // uint4 of staged activations per 256 columns
constexpr int kStageBytes = 2304;  // q: 4 x [32 lanes][16 B], headers: [16 rows][16 B]
constexpr int kMaxCols = 45056;
constexpr int kSmemMax = 227 * 1024;
constexpr int kCoresidentSmem = 110 * 1024;  // fits two CTAs (this kernel and the next) per SM
constexpr uint32_t kMagic = 0x64006400u;  // f16x2 (1024, 1024)
constexpr uint32_t kMul = 0x2C003C00u;    // f16x2 (1, 1/16)
constexpr uint32_t kAdd = 0xD400E400u;    // f16x2 (-1024, -64)

struct Params {
  const uint8_t* w;
  const float* x;
  float* y;
  long long rowb;
  int rows, nku, ntiles, ctas;
  int x_off, slot_off;  // dynamic smem byte offsets (rings at 0)
};

struct Raw {
  uint4 hA, qA0, qA1, hB, qB0, qB1;
};

// Activations for the MMAs, per 256-column unit (68 x 16 B):
//   [i=0..7][g=0..1][t=0..3] 16 B: the B fragments of thread (g,t) for
//     MMA pair i (g=0: hi halves, g=1: lo halves), in the k order the
//     weight decode produces (see compute_unit);
//   [64..67]: the min-MMA fragments, 8 B per (g-2, t): sums of x over the
//     16-element half sub-blocks thread t covers, hi/lo split.
// Each unit's activations are scaled by their own power of two 2^e (2^(e-4)
// for the sums) so that max|x| < 2^15 keeps the fp16 halves exact; the
// unit's 2^-e goes to s_inv[u] and into the epilogue multiplier.  One warp
// stages a unit: lane (i, tt) loads the 8 values of its fragments; a warp
// requests up to 4 units' values before converting any.
GI_DEVINL void stage_unit(uint4* xs, float* s_inv, int u, float4 a, float4 b, int lane) {
  const int i = lane >> 2, tt = lane & 3;
  float m = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))),
                  fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
  m = warp_max(m);
  int e = 0;
  if (m > 0.f && m <= 3.0e38f) e = min(100, max(-100, 14 - ilogbf(m)));
  const float s = exp2i(e);
  float ah[4], al[4], bh[4], bl[4];
  split_hi_lo(a.x * s, ah[0], al[0]);
  split_hi_lo(a.y * s, ah[1], al[1]);
  split_hi_lo(a.z * s, ah[2], al[2]);
  split_hi_lo(a.w * s, ah[3], al[3]);
  split_hi_lo(b.x * s, bh[0], bl[0]);
  split_hi_lo(b.y * s, bh[1], bl[1]);
  split_hi_lo(b.z * s, bh[2], bl[2]);
  split_hi_lo(b.w * s, bh[3], bl[3]);
  uint4 hi, lo;
  hi.x = pack_h2(ah[0], ah[2]);
  hi.y = pack_h2(bh[0], bh[2]);
  hi.z = pack_h2(ah[1], ah[3]);
  hi.w = pack_h2(bh[1], bh[3]);
  lo.x = pack_h2(al[0], al[2]);
  lo.y = pack_h2(bl[0], bl[2]);
  lo.z = pack_h2(al[1], al[3]);
  lo.w = pack_h2(bl[1], bl[3]);
  xs[u * kUnitVec + i * 8 + tt] = hi;
  xs[u * kUnitVec + i * 8 + 4 + tt] = lo;
  // Half-sub-block sums: this lane's 4 values, then over w (lane bits 2-3).
  float sa = (a.x + a.y) + (a.z + a.w);
  float sb = (b.x + b.y) + (b.z + b.w);
  sa += __shfl_xor_sync(0xffffffffu, sa, 4);
  sb += __shfl_xor_sync(0xffffffffu, sb, 4);
  sa += __shfl_xor_sync(0xffffffffu, sa, 8);
  sb += __shfl_xor_sync(0xffffffffu, sb, 8);
  const float sa1 = __shfl_down_sync(0xffffffffu, sa, 16);  // v = 1 half sums
  const float sb1 = __shfl_down_sync(0xffffffffu, sb, 16);
  if (lane < 4) {
    const float sm = exp2i(e - 4);
    float Xh[4], Xl[4];
    split_hi_lo(sa * sm, Xh[0], Xl[0]);
    split_hi_lo(sb * sm, Xh[1], Xl[1]);
    split_hi_lo(sa1 * sm, Xh[2], Xl[2]);
    split_hi_lo(sb1 * sm, Xh[3], Xl[3]);
    uint2* m2 = reinterpret_cast<uint2*>(xs + u * kUnitVec + 64);
    m2[tt] = make_uint2(pack_h2(Xh[0], Xh[1]), pack_h2(Xh[2], Xh[3]));
    m2[4 + tt] = make_uint2(pack_h2(Xl[0], Xl[1]), pack_h2(Xl[2], Xl[3]));
  }
  if (lane == 0) s_inv[u] = exp2i(-e);
}

__device__ void stage_x(uint4* xs, float* s_inv, const float* __restrict__ x, int nku) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int i = lane >> 2, tt = lane & 3;
  const int off = 64 * ((tt >> 1) + 2 * (i >> 2)) + 16 * (tt & 1) + 4 * (i & 3);
  for (int u0 = warp; u0 < nku; u0 += 4 * kWarps) {
    float4 a[4], b[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int u = u0 + k * kWarps;
      if (u < nku) {
        a[k] = __ldg(reinterpret_cast<const float4*>(x + u * 256 + off));
        b[k] = __ldg(reinterpret_cast<const float4*>(x + u * 256 + off + 32));
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int u = u0 + k * kWarps;
      if (u < nku) stage_unit(xs, s_inv, u, a[k], b[k], lane);
    }
  }
  __syncthreads();
}

// Scales and mins of the four sub-blocks thread t covers, as exact f16x2:
// (sc[p], sc[p+1]), (sc[p+4], sc[p+5]) and the same for the mins, with
// p = 2*(t>>1).  This is getScaleMin (pkg/quant/quant.go:228-235) for two
// sub-blocks at a time.
GI_DEVINL void decode_scales(const uint4& h, uint32_t sh, uint32_t& sc0, uint32_t& sc1,
                             uint32_t& mn0, uint32_t& mn1) {
  const uint32_t a = h.y >> sh, b = h.z >> sh, c = h.w >> sh;
  const uint32_t s01 = a & 0x3F3Fu, n01 = b & 0x3F3Fu;
  const uint32_t s45 = (c & 0x0F0Fu) | ((a >> 2) & 0x3030u);
  const uint32_t n45 = ((c >> 4) & 0x0F0Fu) | ((b >> 2) & 0x3030u);
  sc0 = hsub2_u32(prmt(s01, 0x6464u, 0x5140u), kMagic);
  sc1 = hsub2_u32(prmt(s45, 0x6464u, 0x5140u), kMagic);
  mn0 = hsub2_u32(prmt(n01, 0x6464u, 0x5140u), kMagic);
  mn1 = hsub2_u32(prmt(n45, 0x6464u, 0x5140u), kMagic);
}

// One unit: 16 rows (g, g+8 for this thread) x 256 columns.
GI_DEVINL void compute_unit(const Raw& r, const uint4* __restrict__ xsu, int g, int t,
                            uint32_t sh, uint32_t fshift, float fmul, float& yA, float& yB) {
  uint32_t scA[2], scB[2], mnA[2], mnB[2];
  decode_scales(r.hA, sh, scA[0], scA[1], mnA[0], mnA[1]);
  decode_scales(r.hB, sh, scB[0], scB[1], mnB[0], mnB[1]);
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // one MMA chain per v
#pragma unroll
  for (int v = 0; v < 2; ++v) {
    const uint32_t kA = hmul2_u32(scA[v], kMul), aA = hmul2_u32(scA[v], kAdd);
    const uint32_t kB = hmul2_u32(scB[v], kMul), aB = hmul2_u32(scB[v], kAdd);
    const uint32_t mlA = prmt(kA, kA, 0x1010u), mhA = prmt(kA, kA, 0x3232u);
    const uint32_t alA = prmt(aA, aA, 0x1010u), ahA = prmt(aA, aA, 0x3232u);
    const uint32_t mlB = prmt(kB, kB, 0x1010u), mhB = prmt(kB, kB, 0x3232u);
    const uint32_t alB = prmt(aB, aB, 0x1010u), ahB = prmt(aB, aB, 0x3232u);
    const uint4 qa = v ? r.qA1 : r.qA0;
    const uint4 qb = v ? r.qB1 : r.qB0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t wa = (&qa.x)[w], wb = (&qb.x)[w];
      uint4 bf = make_uint4(0u, 0u, 0u, 0u);
      if (g < 2) bf = xsu[(4 * v + w) * 8 + g * 4 + t];
      // bytes 0 and 2: low nibbles -> elements e0, e0+2; high -> e0+32, e0+34
      const uint32_t p0a = hfma2_u32(and_or(wa, 0x000F000Fu, kMagic), mlA, alA);
      const uint32_t p0b = hfma2_u32(and_or(wb, 0x000F000Fu, kMagic), mlB, alB);
      const uint32_t p1a = hfma2_u32(and_or(wa, 0x00F000F0u, kMagic), mhA, ahA);
      const uint32_t p1b = hfma2_u32(and_or(wb, 0x00F000F0u, kMagic), mhB, ahB);
      mma_16816(acc[v], p0a, p0b, p1a, p1b, bf.x, bf.y);
      // bytes 1 and 3: elements e0+1, e0+3, e0+33, e0+35
      const uint32_t wa8 = wa >> 8, wb8 = wb >> 8;
      const uint32_t p2a = hfma2_u32(and_or(wa8, 0x000F000Fu, kMagic), mlA, alA);
      const uint32_t p2b = hfma2_u32(and_or(wb8, 0x000F000Fu, kMagic), mlB, alB);
      const uint32_t p3a = hfma2_u32(and_or(wa8, 0x00F000F0u, kMagic), mhA, ahA);
      const uint32_t p3b = hfma2_u32(and_or(wb8, 0x00F000F0u, kMagic), mhB, ahB);
      mma_16816(acc[v], p2a, p2b, p3a, p3b, bf.z, bf.w);
    }
  }
  uint2 bm = make_uint2(0u, 0u);
  if (g == 2 || g == 3) bm = reinterpret_cast<const uint2*>(xsu + 64)[(g - 2) * 4 + t];
  mma_16816(acc[0], mnA[0], mnB[0], mnA[1], mnB[1], bm.x, bm.y);
  // Lane t=0 holds columns 0,1 (sum q*sc*x as hi+lo), lane t=1 columns 2,3
  // (sum m*X); f = d for t=0 and -16*dmin for t=1 (the sums were staged at
  // 2^-4 the activation scale).  Lanes t>=2 hold zero columns.
  const float fA = __half2float(__ushort_as_half((unsigned short)(r.hA.x >> fshift))) * fmul;
  const float fB = __half2float(__ushort_as_half((unsigned short)(r.hB.x >> fshift))) * fmul;  // fmul carries the unit's 2^-e
  yA = fmaf(fA, (acc[0][0] + acc[0][1]) + (acc[1][0] + acc[1][1]), yA);
  yB = fmaf(fB, (acc[0][2] + acc[0][3]) + (acc[1][2] + acc[1][3]), yB);
}

template <int S>
__global__ void __launch_bounds__(kThreads, 2) gemv_q4k_kernel(const Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int c = blockIdx.x;
  const int T0 = (int)((long long)p.ntiles * c / p.ctas), T1 = (int)((long long)p.ntiles * (c + 1) / p.ctas);
  const int c0 = T0 * p.nku, n = (T1 - T0) * p.nku;  // the CTA's units [c0, c0 + n)
  auto range_of = [&](int w, int& a, int& b) {
    a = c0 + (int)((long long)n * w / kWarps);
    b = c0 + (int)((long long)n * (w + 1) / kWarps);
  };
  int u0, u1;
  range_of(warp, u0, u1);
  const uint32_t ring = smem_u32(smem) + warp * S * kStageBytes;
  uint4* xs = reinterpret_cast<uint4*>(smem + p.x_off);
  float* s_inv = reinterpret_cast<float*>(xs + p.nku * kUnitVec);
  float* slots = reinterpret_cast<float*>(smem + p.slot_off);  // [kWarps][2][16]
  const uint64_t pol = l2_evict_first_policy();

  // Producer state: (tile, ku) of the next unit to request.
  int ltile = u0 / p.nku, lku = u0 - ltile * p.nku;
  int next = u0;
  auto request = [&](int stage) {  // always commits one group (possibly empty)
    if (next < u1) {
      const int rA = min(ltile * 16 + g, p.rows - 1);
      const int rB = min(ltile * 16 + g + 8, p.rows - 1);
      const uint8_t* a = p.w + (long long)rA * p.rowb + lku * 144;
      const uint8_t* b = p.w + (long long)rB * p.rowb + lku * 144;
      const uint32_t base = ring + stage * kStageBytes;
      cp_async16_hint(base + lane * 16, a + 16 + 16 * t, pol);
      cp_async16_hint(base + 512 + lane * 16, a + 80 + 16 * t, pol);
      cp_async16_hint(base + 1024 + lane * 16, b + 16 + 16 * t, pol);
      cp_async16_hint(base + 1536 + lane * 16, b + 80 + 16 * t, pol);
      if (t < 2) cp_async16_hint(base + 2048 + (g + 8 * t) * 16, t ? b : a, pol);
      if (++lku == p.nku) {
        lku = 0;
        ++ltile;
      }
      ++next;
    }
    cp_async_commit();
  };
  // Weights never depend on the previous kernel: request S units first.
#pragma unroll
  for (int s = 0; s < S; ++s) request(s);
  griddep_wait();
  stage_x(xs, s_inv, p.x, p.nku);

  const uint32_t sh = (uint32_t)(t >> 1) * 16u;
  const uint32_t fshift = t == 0 ? 0u : 16u;
  const float fmul = t == 0 ? 1.f : -16.f;
  const int first_tile = u0 / p.nku;
  int ctile = first_tile, cku = u0 - first_tile * p.nku;
  float yA = 0.f, yB = 0.f;
  int stage = 0;
  for (int u = u0; u < u1; ++u) {
    cp_async_wait<S - 1>();
    __syncwarp();
    const uint32_t base = ring + stage * kStageBytes;
    Raw r;
    r.qA0 = lds128(base + lane * 16);
    r.qA1 = lds128(base + 512 + lane * 16);
    r.qB0 = lds128(base + 1024 + lane * 16);
    r.qB1 = lds128(base + 1536 + lane * 16);
    r.hA = lds128(base + 2048 + g * 16);
    r.hB = lds128(base + 2048 + (g + 8) * 16);
    compute_unit(r, xs + cku * kUnitVec, g, t, sh, fshift, fmul * s_inv[cku], yA, yB);
    __syncwarp();
    request(stage);
    stage = stage + 1 == S ? 0 : stage + 1;
    const int tile = ctile;
    const bool tile_end = cku == p.nku - 1;
    if (++cku == p.nku) {
      cku = 0;
      ++ctile;
    }
    if (tile_end || u == u1 - 1) {
      const float vA = yA + __shfl_xor_sync(0xffffffffu, yA, 1);
      const float vB = yB + __shfl_xor_sync(0xffffffffu, yB, 1);
      yA = 0.f;
      yB = 0.f;
      if (t == 0) {
        const int tu0 = tile * p.nku;
        if (tu0 >= u0 && tu0 + p.nku <= u1) {  // this warp owns the whole tile
          const int rA = tile * 16 + g;
          if (rA < p.rows) p.y[rA] = vA;
          if (rA + 8 < p.rows) p.y[rA + 8] = vB;
        } else {
          float* sl = slots + (warp * 2 + (tile == first_tile ? 0 : 1)) * 16;
          sl[g] = vA;
          sl[g + 8] = vB;
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  // Tiles split between warps of this CTA: sum their partials in warp order.
  for (int T = T0 + warp; T < T1; T += kWarps) {
    const int tu0 = T * p.nku, tu1 = tu0 + p.nku;
    float sum = 0.f;
    bool owned = false;
    for (int w = 0; w < kWarps; ++w) {
      int a, b;
      range_of(w, a, b);
      if (a >= b || a >= tu1 || b <= tu0) continue;
      if (a <= tu0 && b >= tu1) owned = true;
      if (lane < 16) sum += slots[(w * 2 + (T == a / p.nku ? 0 : 1)) * 16 + lane];
    }
    const int row = T * 16 + lane;
    if (!owned && lane < 16 && row < p.rows) p.y[row] = sum;
  }
}

struct Layout {
  int ctas, ntiles, stages, x_off, slot_off, smem;
};

Layout layout(int64_t rows, int64_t cols, const GemvLaunch& L) {
  Layout o;
  const int nku = (int)(cols / 256);
  o.ntiles = (int)((rows + 15) / 16);
  o.ctas = o.ntiles < L.sm_count ? o.ntiles : L.sm_count;
  const int xbytes = ((nku * (kUnitVec * 16 + 4)) + 15) & ~15;
  const int fixed = xbytes + kWarps * 2 * 16 * 4;
  // As many stages as fit next to a co-resident CTA, at least 2.
  o.stages = 4;
  while (o.stages > 2 && fixed + kWarps * o.stages * kStageBytes > kCoresidentSmem) --o.stages;
  o.x_off = kWarps * o.stages * kStageBytes;
  o.slot_off = o.x_off + xbytes;
  o.smem = o.slot_off + kWarps * 2 * 16 * 4;
  return o;
}

int launch(float* y, const float* x, const void* w, int64_t rows, int64_t cols, const GemvScratch& s,
           const GemvLaunch& L, cudaStream_t stream) {
  (void)s;
  const Layout o = layout(rows, cols, L);
  if (o.smem > kSmemMax) return -4;
  Params p;
  p.w = static_cast<const uint8_t*>(w);
  p.x = x;
  p.y = y;
  p.rowb = row_bytes(kTypeQ4_K, cols);
  p.rows = (int)rows;
  p.nku = (int)(cols / 256);
  p.ntiles = o.ntiles;
  p.ctas = o.ctas;
  p.x_off = o.x_off;
  p.slot_off = o.slot_off;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(o.ctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = o.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  cudaError_t e;
  switch (o.stages) {
    case 4: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<4>, p); break;
    case 3: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<3>, p); break;
    default: e = cudaLaunchKernelEx(&cfg, gemv_q4k_kernel<2>, p); break;
  }
  return e == cudaSuccess ? 0 : -5;
}

int prepare() {
  cudaError_t e = cudaFuncSetAttribute(gemv_q4k_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_q4k_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_q4k_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  return e == cudaSuccess ? 0 : -5;
}
}  // namespace q4k

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
}  // namespace q6k

int gemv_prepare_device() { return q4k::prepare(); }

int gemv_check(int qtype, int64_t rows, int64_t cols) {
  if (rows < 1 || cols < 1 || rows > (1LL << 30)) return -4;
  switch (qtype) {
    case kTypeQ4_K:
      return (cols % 256 == 0 && cols <= q4k::kMaxCols) ? 0 : -4;
    case kTypeQ6_K:
      return cols % 256 == 0 ? 0 : -4;
    case kTypeQ8_0:
      return cols % 32 == 0 ? 0 : -4;
    default:
      return -2;
  }
}

void gemv_scratch_need(int qtype, int64_t rows, int64_t cols, const GemvLaunch& L, int* warps,
                       int* tiles) {
  *warps = 0;
  *tiles = 0;
  (void)qtype;
  (void)rows;
  (void)cols;
  (void)L;
}

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
      return q4k::launch(y, x, w, rows, cols, s, L, stream);
    case kTypeQ8_0:
      return launch_rowwarp(q80::gemv_q80_kernel, rows, L, stream, y, x, wb, wb + w_bytes,
                            (long long)rb, (int)rows, (int)(cols / 32));
    case kTypeQ6_K:
      return launch_rowwarp(q6k::gemv_q6k_kernel, rows, L, stream, y, x, wb, wb + w_bytes,
                            (long long)rb, (int)rows, (int)(cols / 256));
    default:
      return -2;
  }
}

}  // namespace gi
