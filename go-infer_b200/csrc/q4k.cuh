// q4k.cuh -- device code of the Q4_K decode GEMV: the work decomposition,
// the activation staging and the per-unit tensor-core arithmetic, shared by
// the stand-alone GEMV kernel (gemv.cu) and the persistent decode-layer
// kernel (layers.cu).
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace gi {
namespace q4k {
// Work decomposition: a unit is 16 rows x 256 columns (one super-block per
// row, 2304 bytes).  Each CTA owns a contiguous run of whole 16-row tiles,
// so no reduction crosses CTAs; its units (tile-major) are dealt to the
// warps round-robin and every tile's per-warp partials are summed in fixed
// warp order through shared memory (deterministic).  Each warp
// streams its units through a private ring of shared-memory stages with
// cp.async (16 bytes per lane, L1-bypassing, S units in flight, the first
// ones requested before the kernel waits on its predecessor).
//
// Arithmetic: integer tensor cores.  The 4-bit quants enter an int8 MMA
// (m16n8k32) unchanged except for one mask per 4 weights (low nibbles as
// q, high nibbles as 16*q); the activations enter as four balanced base-256
// limbs of a 30-bit fixed-point value per 256-column unit
// (x = 2^-e * sum_n L_n 256^(3-n), |x| < 2^(30-e); exact for every value
// within 7 binades of the unit's largest, absolute error <= 2^-31 of it
// otherwise).  Every product and sum of a sub-block is therefore exact in
// int32; the 6-bit sub-block scales are applied with integer multiply-adds,
// and a unit's total leaves the integer domain once, through 4 int->float
// conversions per lane.  The 6-bit mins ride on one fp16 MMA against the
// per-sub-block activation sums (hi+lo fp16 split).
// Warps per CTA, W: 16 when each CTA has enough units to keep them busy
// (more warps hide more of the per-warp dependency chains), else 8.
constexpr int kWarpsSmall = 8, kWarpsLarge = 16;
constexpr int kUnitX = 1104;       // staged activation bytes per unit (see stage_unit)
constexpr int kStageBytes = 2304;  // qs: [16 rows][8 x 16 B, piece q at slot q ^ (row & 7)], headers: [16 rows][16 B]
constexpr int kMaxCols = 45056;
constexpr int kSmemMax = 227 * 1024 - 256;  // dynamic; the rest is static (the RMSNorm reduction)
constexpr int kCoresidentSmem = 110 * 1024;  // fits two CTAs (this kernel and the next) per SM
constexpr uint32_t kMagic = 0x64006400u;     // f16x2 (1024, 1024)

constexpr int kMaxMats = 3;  // matrices sharing one activation vector per launch

struct Params {
  const uint8_t* w[kMaxMats];
  float* y[kMaxMats];
  int rows[kMaxMats];
  int tstart[kMaxMats + 1];  // first global 16-row tile of each matrix (prefix sums)
  const float* x;
  const float* x2;  // RMSNorm weight (xmode kXNorm)
  float eps;
  int xmode, ymode;
  TpDev tp;  // kYPush
  long long rowb;
  int nku, ntiles, ctas;
  int x_off, slot_off, red_off;  // dynamic smem byte offsets (rings at 0)
};

// Matrix m and its local 16-row tile lt of global tile T: matrices one
// after another (tiles of matrix m are [tstart[m], tstart[m+1])), or in
// kYSwiGLU mode gate and up tiles interleaved (gate tile i = 2i, up = 2i+1)
// so that one CTA holds both halves of every row it finishes.
template <bool F>
GI_DEVINL void tile_of(const Params& p, int T, int& m, int& lt) {
  if (F && p.ymode == kYSwiGLU) {
    m = T & 1;
    lt = T >> 1;
  } else {
    m = (T >= p.tstart[1]) + (T >= p.tstart[2]);
    lt = T - p.tstart[m];
  }
}

// Byte k of each of four words, gathered into one word (byte i from w_i).
GI_DEVINL uint32_t gather_byte(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t k) {
  const uint32_t lo = prmt(w0, w1, k | ((4u + k) << 4));
  const uint32_t hi = prmt(w2, w3, k | ((4u + k) << 4));
  return prmt(lo, hi, 0x5410u);
}

// Activations of one unit (256 columns) in shared memory at xu:
//   [0, 1024)    int8 limbs, [sub-block j][limb n][32 positions], limb 0 the
//                most significant; sub-block j covers columns
//                64*(j/2) + 32*(j%2) + l, as Q4_K's getScaleMin indexes them,
//                and positions 8q..8q+7 hold its elements 4q..4q+3 and
//                16+4q..16+4q+3: the k order of an m16n8k32 B fragment, so
//                lane t of the MMA reads its two B registers with one load;
//   [1024, 1088) min-MMA B fragments: for t = 0..3, 8 bytes:
//                f16 (X_t hi, X_t lo, X_{t+4} hi, X_{t+4} lo), X_j the sum
//                of sub-block j scaled by 2^em;
//   [1088, 1096) float 2^-e, float 2^-em.
// One warp stages a unit; lane L owns elements 4q..4q+3 (a) and
// 16+4q..16+4q+3 (b) of sub-block L/4, q = L%4.
GI_DEVINL void stage_unit(uint8_t* xu, float4 a, float4 b, int lane) {
  float m = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))),
                  fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
  m = warp_max(m);
  int e = 0, em = 0;
  if (m > 0.f && m <= 3.0e38f) {
    const int lg = ilogbf(m);
    e = min(126, max(-126, 29 - lg));  // max |x| * 2^e < 2^30
    em = min(126, max(-126, 9 - lg));  // max |X| <= 32 max |x|: X * 2^em < 2^15
  }
  const float s = exp2i(e);
  // Balanced base-256 digits of v are the bytes of (v + 0x80808080) ^ 0x80808080.
  uint32_t u[8];
  u[0] = ((uint32_t)__float2int_rn(a.x * s) + 0x80808080u) ^ 0x80808080u;
  u[1] = ((uint32_t)__float2int_rn(a.y * s) + 0x80808080u) ^ 0x80808080u;
  u[2] = ((uint32_t)__float2int_rn(a.z * s) + 0x80808080u) ^ 0x80808080u;
  u[3] = ((uint32_t)__float2int_rn(a.w * s) + 0x80808080u) ^ 0x80808080u;
  u[4] = ((uint32_t)__float2int_rn(b.x * s) + 0x80808080u) ^ 0x80808080u;
  u[5] = ((uint32_t)__float2int_rn(b.y * s) + 0x80808080u) ^ 0x80808080u;
  u[6] = ((uint32_t)__float2int_rn(b.z * s) + 0x80808080u) ^ 0x80808080u;
  u[7] = ((uint32_t)__float2int_rn(b.w * s) + 0x80808080u) ^ 0x80808080u;
  const int j = lane >> 2, q = lane & 3;
  const uint32_t base = smem_u32(xu) + j * 128 + 8 * q;
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const uint32_t k = 3u - (uint32_t)n;  // limb n is byte 3-n
    const uint32_t lo = gather_byte(u[0], u[1], u[2], u[3], k);
    const uint32_t hi = gather_byte(u[4], u[5], u[6], u[7], k);
    sts64(base + n * 32, (uint64_t)lo | ((uint64_t)hi << 32));
  }
  float sx = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w));
  sx += __shfl_xor_sync(0xffffffffu, sx, 1);
  sx += __shfl_xor_sync(0xffffffffu, sx, 2);  // sub-block sum, in lanes 4j..4j+3
  const float xs = sx * exp2i(em);
  const float Xa = __shfl_sync(0xffffffffu, xs, 4 * q);       // X_q
  const float Xb = __shfl_sync(0xffffffffu, xs, 16 + 4 * q);  // X_{q+4}
  if (lane < 4) {
    float ah, al, bh, bl;
    split_hi_lo(Xa, ah, al);
    split_hi_lo(Xb, bh, bl);
    sts64(smem_u32(xu) + 1024 + 8 * lane, (uint64_t)pack_h2(ah, al) | ((uint64_t)pack_h2(bh, bl) << 32));
  }
  if (lane == 0) {
    reinterpret_cast<float*>(xu + 1088)[0] = exp2i(-e);
    reinterpret_cast<float*>(xu + 1088)[1] = exp2i(-em);
  }
}

GI_DEVINL float4 mul3(float4 a, float s, float4 w) {  // (a * s) * w, one rounding each
  return make_float4(__fmul_rn(__fmul_rn(a.x, s), w.x), __fmul_rn(__fmul_rn(a.y, s), w.y),
                     __fmul_rn(__fmul_rn(a.z, s), w.z), __fmul_rn(__fmul_rn(a.w, s), w.w));
}

// Load of the activation vector: through the read-only path, or (C) with an
// L2-coherent load (__ldcg) when the vector was written earlier in the same
// kernel by other CTAs (the persistent decode-layer kernel), where the
// read-only path may still hold an older copy.
template <bool C>
GI_DEVINL float4 ld_x4(const float4* p) {
  if (C) return __ldcg(p);
  return __ldg(p);
}

// Stage the activation vector: p.x, or in kXNorm mode RMSNorm(p.x) * p.x2
// (pkg/math/kernels.go:9-19: float32 sum of squares, scale
// float32(1 / sqrt(float64(mean + eps))), out = x * scale * w), computed by
// every CTA from the same data in the same order.  Warp w stages the column
// blocks w, w + W, ...; with cta_sync false it only waits for its own
// stores, for a caller whose warps read nothing but the blocks they staged.
template <int W, bool F, bool C = false>
__device__ void stage_x(uint8_t* xs, float* red, const Params& p, bool cta_sync = true) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = lane >> 2, q = lane & 3;
  const int offA = 64 * (j >> 1) + 32 * (j & 1) + 4 * q, offB = offA + 16;  // stage_unit's a, b
  const int nku = p.nku;
  const float* x = p.x;
  float scale = 1.f;
  if (F && p.xmode == kXNorm) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float s = 0.f;
    for (int i = threadIdx.x; i < nku * 64; i += W * 32) {
      const float4 v = ld_x4<C>(x4 + i);
      s = __fadd_rn(s, __fmul_rn(v.x, v.x));
      s = __fadd_rn(s, __fmul_rn(v.y, v.y));
      s = __fadd_rn(s, __fmul_rn(v.z, v.z));
      s = __fadd_rn(s, __fmul_rn(v.w, v.w));
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) tot = __fadd_rn(tot, red[w]);
    const float mean = __fdiv_rn(tot, (float)(nku * 256));
    scale = (float)(1.0 / sqrt((double)__fadd_rn(mean, p.eps)));
  }
  for (int u0 = warp; u0 < nku; u0 += 4 * W) {
    float4 a[4], b[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int u = u0 + k * W;
      if (u < nku) {
        a[k] = ld_x4<C>(reinterpret_cast<const float4*>(x + u * 256 + offA));
        b[k] = ld_x4<C>(reinterpret_cast<const float4*>(x + u * 256 + offB));
        if (F && p.xmode == kXNorm) {
          a[k] = mul3(a[k], scale, __ldg(reinterpret_cast<const float4*>(p.x2 + u * 256 + offA)));
          b[k] = mul3(b[k], scale, __ldg(reinterpret_cast<const float4*>(p.x2 + u * 256 + offB)));
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int u = u0 + k * W;
      if (u < nku) stage_unit(xs + u * kUnitX, a[k], b[k], lane);
    }
  }
  if (cta_sync)
    __syncthreads();
  else
    __syncwarp();
}

// One unit: rows g and g+8 of a 16-row tile, 256 columns.  stage: the raw
// super-blocks in shared memory (qs of row r at r*128, its 16-byte piece p
// at slot p ^ (r & 7), so the eight rows of one ldmatrix read hit eight
// different bank groups; headers at 2048 + r*16); lofs: this lane's
// ldmatrix row address in a stage for chunk 0 (chunk c: lofs ^ 32c); xu:
// the unit's staged activations; xl: this lane's B fragment in them (limb g
// of sub-block 0, or for g >= 4 limb g-4 of sub-block 1).
//
// Each 64-column chunk c takes two MMAs with the same B: its columns 0-3
// hold the limbs of sub-block 2c (the low nibbles' activations), columns 4-7
// those of sub-block 2c+1 (the high nibbles').  MMA L multiplies the low
// nibbles alone, MMA F the whole bytes (q_lo + 16 q_hi): columns 0-3 of L
// are the low-nibble products, columns 4-7 of F - L are 16 x the
// high-nibble products.  Lanes t = 0, 1 hold columns 0-3 and lanes 2, 3
// columns 4-7; each scales its accumulators by its sub-block's scale, so the
// integer sums stay exact and every column of both MMAs is used.
GI_DEVINL void compute_unit(uint32_t stage, uint32_t lofs, uint32_t xu, uint32_t xl, int g, int t, uint32_t sh8,
                            uint32_t selE, uint32_t selO, float W0, float W1, float& yA, float& yB) {
  const uint4 hA = lds128(stage + 2048 + g * 16);
  const uint4 hB = lds128(stage + 2048 + (g + 8) * 16);
  // 6-bit scales sc0..sc7 as bytes (getScaleMin, pkg/quant/quant.go:228-235)
  const uint32_t sA03 = hA.y & 0x3F3F3F3Fu, sB03 = hB.y & 0x3F3F3F3Fu;
  const uint32_t sA47 = (hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u);
  const uint32_t sB47 = (hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u);
  int lA0 = 0, lA1 = 0, lB0 = 0, lB1 = 0, fA0 = 0, fA1 = 0, fB0 = 0, fB1 = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    // A fragment of chunk c: rows g, g+8 x bytes 4t..4t+3 and 16+4t..16+4t+3
    uint32_t a0, a1, a2, a3;
    ldsm_x4(stage + (lofs ^ (32u * (uint32_t)c)), a0, a1, a2, a3);
    const uint64_t xv = lds64(xl + (2 * c) * 128);
    int dl[4] = {0, 0, 0, 0}, df[4] = {0, 0, 0, 0};
    imma_16832(dl, a0 & 0x0F0F0F0Fu, a1 & 0x0F0F0F0Fu, a2 & 0x0F0F0F0Fu, a3 & 0x0F0F0F0Fu, (uint32_t)xv,
               (uint32_t)(xv >> 32));
    imma_16832(df, a0, a1, a2, a3, (uint32_t)xv, (uint32_t)(xv >> 32));
    // this lane's sub-block scale: byte (2c & 3) + (t >= 2) of the word
    const uint32_t sel = (c & 1) ? selO : selE;
    const int sA = (int)prmt(c < 2 ? sA03 : sA47, 0u, sel), sB = (int)prmt(c < 2 ? sB03 : sB47, 0u, sel);
    lA0 += dl[0] * sA;
    lA1 += dl[1] * sA;
    lB0 += dl[2] * sB;
    lB1 += dl[3] * sB;
    fA0 += df[0] * sA;
    fA1 += df[1] * sA;
    fB0 += df[2] * sB;
    fB1 += df[3] * sB;
  }
  // Mins: A = m_t, m_{t+4} (duplicated for the hi/lo halves of X), B col 4.
  const uint32_t zA = hA.z >> sh8, wA = hA.w >> sh8, zB = hB.z >> sh8, wB = hB.w >> sh8;
  const uint32_t mA0 = zA & 63u, mA4 = ((wA >> 4) & 0xFu) | ((zA >> 2) & 0x30u);
  const uint32_t mB0 = zB & 63u, mB4 = ((wB >> 4) & 0xFu) | ((zB >> 2) & 0x30u);
  const uint32_t gA0 = hsub2_u32((mA0 * 0x10001u) | kMagic, kMagic);
  const uint32_t gA4 = hsub2_u32((mA4 * 0x10001u) | kMagic, kMagic);
  const uint32_t gB0 = hsub2_u32((mB0 * 0x10001u) | kMagic, kMagic);
  const uint32_t gB4 = hsub2_u32((mB4 * 0x10001u) | kMagic, kMagic);
  uint64_t bm = 0;
  if (g == 4) bm = lds64(xu + 1024 + 8 * t);
  float cm[4] = {0.f, 0.f, 0.f, 0.f};
  mma_16816(cm, gA0, gB0, gA4, gB4, (uint32_t)bm, (uint32_t)(bm >> 32));
  // lanes 0, 1: the low-nibble sums; lanes 2, 3: F - L, the high-nibble
  // sums times 16 (W0, W1 divide it out)
  const bool hi = t >= 2;
  const int iA0 = hi ? fA0 - lA0 : lA0, iA1 = hi ? fA1 - lA1 : lA1;
  const int iB0 = hi ? fB0 - lB0 : lB0, iB1 = hi ? fB1 - lB1 : lB1;
  // Scale factors multiply in an order that keeps every intermediate a
  // normal float (2^-e alone can be as small as 2^-126).
  const uint64_t inv = lds64(xu + 1088);
  const float inv_main = __uint_as_float((uint32_t)inv);
  const float inv_min = __uint_as_float((uint32_t)(inv >> 32));
  const float2 dA = __half22float2(*reinterpret_cast<const __half2*>(&hA.x));
  const float2 dB = __half22float2(*reinterpret_cast<const __half2*>(&hB.x));
  yA = fmaf(fmaf((float)iA0, W0, (float)iA1 * W1) * dA.x, inv_main, yA);
  yB = fmaf(fmaf((float)iB0, W0, (float)iB1 * W1) * dB.x, inv_main, yB);
  yA = fmaf((cm[0] + cm[1]) * -dA.y, inv_min, yA);
  yB = fmaf((cm[2] + cm[3]) * -dB.y, inv_min, yB);
}
}  // namespace q4k
}  // namespace gi
