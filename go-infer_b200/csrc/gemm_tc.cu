// gemm_tc.cu -- batched prefill Y[tok][row] = sum_k W[row][k] X[tok][k] over
// raw GGUF Q4_K / Q6_K blocks on the sm_100a tensor cores.
//
// This is the tensor-core counterpart of go-infer's prefill kernels
// gemm_q4_k_batched / gemm_q6_k_batched (pkg/metal/kernels.metal:678,828),
// reached through Weights.MatMulBatch (pkg/engine/weights.go:328-350).  The
// reference computes every product in fp32; these kernels keep that accuracy
// on fp16 tensor cores by making every MMA operand exact:
//
//  * Weights.  A Q4_K weight is d*sc*q - dmin*m (pkg/quant/quant.go:215-253).
//    Within one super-block, sc*q <= 63*15 is an integer that fp16 holds
//    exactly, so the A operand of a super-block is the integer tile sc*q and
//    d is applied afterwards, once per (row, super-block).  The min term
//    dmin * sum_j m_j * (sum of x over sub-block j) is a second, K=16 MMA of
//    the integer mins against the sub-block sums.  A Q6_K weight is
//    d*sc*(q6-32) (quant.go:256-291); sc*q can need 12 bits, so its A
//    operand is the pair fp16(sc*q) + (sc*q - fp16(sc*q)), both exact.
//    A Q8_0 weight is d*q (quant.go:196-212, 32-element blocks): d*q needs
//    19 bits, so its A operand is an exact hi/lo pair too, with each block's
//    d folded in and scaled by a power of two per super-block of 256
//    columns (largest d of the 8 blocks -> [64, 128)) that the epilogue
//    divides out.
//  * Activations.  Each token row is scaled by a power of two (its largest
//    magnitude lands below 2^10) and split into fp16 hi + lo, 22 bits of
//    mantissa.  The staging kernel writes both halves once per call.
//
// Per (row, super-block) the fp32 tensor-memory accumulators of the
// super-block are read back by four epilogue warps, scaled by d (and dmin)
// and added to a running fp32 sum in registers; the tensor core meanwhile
// fills the second accumulator buffer with the next super-block.
//
// The K order of a 64-element chunk is permuted identically in the weight
// tile and in the staged activations (a contraction does not care), so that
// one 32-bit word of packed nibbles becomes one 16-byte row segment of the
// operand tile without byte shuffles.
//
// CTA = 10 warps, one 128-row x 128-token output tile:
//   warp 0      bulk (TMA) copies of the staged activation tiles (one thread)
//   warp 1      TMEM allocation, tcgen05.mma issue (one thread)
//   warps 2-5   weight decode: raw blocks -> fp16 operand rows in tensor memory
//   warps 6-9   epilogue: TMEM -> registers, d/dmin scaling, y stores
// Every wait is bounded in time; on expiry the kernel sets *error, drains its
// own copies and MMAs, frees tensor memory and returns.
//
// CTA pairs (opt-in, gi_cuda_set_prefill_pair): two CTAs of a cluster own
// consecutive 128-row weight tiles of the same token tile, and rank 0
// issues 256-row cta_group::2 MMAs over both.  Each CTA still decodes its
// own rows into its own tensor memory and reads back its own accumulators,
// but copies only its 64-token half of every activation tile: the
// activation traffic from L2 (every 128-row weight tile re-reads the whole
// activation) halves.  No copy reads another CTA's shared memory; the
// tensor core reads both halves.  Measured on B200 the pairs are slower:
// the MMA issuer of a single CTA waits little on its activation copies
// (~3 us per launch), while a pair's decoded-weight hand-off (multicast
// commit to the other CTA, its decode, a remote arrive back) outlasts the
// 4-stage pipeline (~33 us of waiting per launch), so single CTAs are the
// default.
#include <type_traits>

#include "common.cuh"
#include "gemm.cuh"

namespace gi {
namespace tc {

constexpr int kTileRows = 128;  // weight rows per CTA: MMA M, TMEM lanes
constexpr int kTileTok = 128;   // tokens per CTA: MMA N
constexpr int kTileBytes = 128 * 64 * 2;  // 128 x 64 fp16 operand tile, 128-byte swizzle
constexpr int kSmallBytes = 128 * 16 * 2;  // 128 x 16 fp16 operand tile, no swizzle
constexpr int kThreads = 320;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: far beyond any legitimate wait

// Tensor memory (512 columns x 128 lanes of 32 bits): two D1 accumulator
// buffers of 128 columns (one per super-block in flight), for Q4_K one D2
// (min-term) accumulator, and the decoded weight operand A of each pipeline
// stage (64 fp16 of K per row = 32 columns; Q6_K's hi and lo parts 64).
template <int QT>
struct Cfg;
template <>
struct Cfg<kTypeQ4_K> {
  static constexpr int kStages = 4;
  static constexpr bool kMins = true;
  static constexpr int kStageBytes = 2 * kTileBytes + 2 * kSmallBytes;  // B hi, B lo, mins, sums
  static constexpr int kD2Col = 256;
  static constexpr int kACol = 384;
  static constexpr int kAStageCols = 32;
  static constexpr int kPrefetch = 4;  // weight chunks loaded ahead by each decode thread
};
template <>
struct Cfg<kTypeQ6_K> {
  static constexpr int kStages = 4;
  static constexpr bool kMins = false;
  static constexpr int kStageBytes = 2 * kTileBytes;  // B hi, B lo
  static constexpr int kD2Col = 0;
  static constexpr int kACol = 256;
  static constexpr int kAStageCols = 64;  // hi part, then lo part
  static constexpr int kPrefetch = 2;
};
template <>
struct Cfg<kTypeQ8_0> {  // the Q6_K pipeline: hi and lo weight parts, no min term
  static constexpr int kStages = 4;
  static constexpr bool kMins = false;
  static constexpr int kStageBytes = 2 * kTileBytes;  // B hi, B lo
  static constexpr int kD2Col = 0;
  static constexpr int kACol = 256;
  static constexpr int kAStageCols = 64;  // hi part, then lo part
  static constexpr int kPrefetch = 3;
};
constexpr int kTmemCols = 512;

// Bytes of one pipeline stage in shared memory.  A CTA of a pair holds only
// its 64-token half of the activation tiles and of the sub-block sums (the
// mins tile keeps all 128 rows of its own weight tile).
template <int QT, bool P2>
constexpr int stage_bytes() {
  return P2 ? Cfg<QT>::kStageBytes / 2 + (Cfg<QT>::kMins ? kSmallBytes / 2 : 0) : Cfg<QT>::kStageBytes;
}

template <int QT, bool P2 = false>
constexpr int smem_bytes() {
  return Cfg<QT>::kStages * stage_bytes<QT, P2>() + 1024 /* alignment */ + 256 /* barriers */;
}

// ---- tcgen05 / TMA / timer primitives ---------------------------------------

GI_DEVINL uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// mbarrier test with acquire at cluster scope: for barriers that the other
// CTA of a pair arrives on.
GI_DEVINL bool mbar_try_wait_cl(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; "
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of `parity` on an mbarrier, giving up after kWaitNs
// (CL: acquire at cluster scope).
template <bool CL = false>
GI_DEVINL bool wait_phase(uint32_t bar, uint32_t parity) {
  auto test = [&]() { return CL ? mbar_try_wait_cl(bar, parity) : mbar_try_wait(bar, parity); };
  if (test()) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (test()) return true;
    if (globaltimer_ns() - t0 > kWaitNs) return false;
  }
}

// The same for a whole warp: lane 0 polls, every lane gets the outcome, and
// the warp leaves converged (the tcgen05 .sync.aligned forms require it).
template <bool CL = false>
GI_DEVINL bool warp_wait_phase(uint32_t bar, uint32_t parity) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_phase<CL>(bar, parity);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

GI_DEVINL void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Contiguous global -> shared bulk copy into this CTA only; completes `bytes`
// of tx on `bar`.  Both addresses 16-byte aligned, bytes a multiple of 16.
GI_DEVINL void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

GI_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
GI_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, fp16 inputs, fp32 accumulate.
GI_DEVINL void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with A read from tensor memory (lane m = row m of A, 16-bit
// column k = element k: two K values per 32-bit column).
GI_DEVINL void mma_f16_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 columns of 32 bits into tensor memory (the warp's lane
// quarter); completion is awaited with tmem_wait_st.
GI_DEVINL void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
GI_DEVINL void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrive once on `bar` when every MMA this thread issued so far has finished.
GI_DEVINL void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// ---- CTA-pair (cta_group::2) forms ------------------------------------------
// The pair is a cluster of two CTAs; rank 0 issues the MMAs for both.  A
// 256-row MMA reads rows 0-127 of A from rank 0's tensor memory and rows
// 128-255 from rank 1's, tokens 0-63 of B from rank 0's shared memory and
// 64-127 from rank 1's (the same offsets in both), and writes each CTA's
// rows of D into its own tensor memory.

GI_DEVINL uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of shared-memory offset `addr` in CTA `rank`.
GI_DEVINL uint32_t peer_addr(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Arrive on an mbarrier of either CTA of the pair (release at cluster scope).
GI_DEVINL void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Both CTAs of the cluster, every thread: release then acquire.
GI_DEVINL void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

GI_DEVINL void mma_f16_2(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

GI_DEVINL void mma_f16_ts_2(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` (the same offset) in both CTAs of the pair when every
// pair MMA this thread issued so far has finished.
GI_DEVINL void mma_commit_2(uint32_t bar) {
  const uint16_t both = 3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(both)
      : "memory");
}

// 32 lanes x 16 columns of fp32 from tensor memory, waited for in place
// (the wait names the registers, so no use can be scheduled before it).
GI_DEVINL void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptors (K-major).  128-byte swizzle: 8-row x
// 128-byte atoms, 1024 bytes apart (stride byte offset), 16-byte units of a
// row XOR-ed with the row index; the leading byte offset is unused.  No
// swizzle: 8-row x 16-byte core matrices, `sbo` bytes between row groups and
// `lbo` bytes between the two 8-element K halves.
GI_DEVINL uint64_t desc_sw128(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
GI_DEVINL uint64_t desc_plain(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
         ((uint64_t)1 << 46);
}

// Instruction descriptor: fp32 D, fp16 A and B, both K-major, M=128, N=128;
// for a CTA pair M=256 (128 rows in each CTA).
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kTileTok >> 3) << 17) | ((uint32_t)(kTileRows >> 4) << 24);
constexpr uint32_t kIdesc2 = (1u << 4) | ((uint32_t)(kTileTok >> 3) << 17) | ((uint32_t)(2 * kTileRows >> 4) << 24);

GI_DEVINL void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

GI_DEVINL uint4 ldg_nc128(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
GI_DEVINL uint32_t ldg_nc32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
GI_DEVINL uint32_t ldg_nc16(const void* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

GI_DEVINL uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
GI_DEVINL uint32_t h2_splat(float v) { return h2_bits(__float2half2_rn(v)); }
GI_DEVINL float h_lo(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFF))); }
GI_DEVINL float h_hi(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

// Byte offset of 16-byte unit `u` of row `r` in a 128-byte-swizzled tile.
GI_DEVINL uint32_t sw128_off(int r, int u) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((u ^ (r & 7)) << 4));
}
// Byte offset of K half `kh` of row `r` in a 128 x 16 core-matrix tile
// (row groups 128 bytes apart, K halves 2048 bytes apart).
GI_DEVINL uint32_t plain_off(int r, int kh) { return (uint32_t)((r >> 3) * 128 + (r & 7) * 16 + kh * 2048); }

// ---- weight decode ------------------------------------------------------------

// Q4_K chunk c (0..3) of a super-block = qs bytes [32c, 32c+32): low nibbles
// are elements 64c+l (sub-block 2c), high nibbles 64c+32+l (sub-block 2c+1),
// pkg/quant/quant.go:230-250.  Word u of the chunk (bytes 4u..4u+3) fills
// 16-byte unit u of the operand row in K order
//   4u, 4u+2, 4u+1, 4u+3 | 32+4u, 32+4u+2, 32+4u+1, 32+4u+3.
struct Q4kRaw {
  uint4 qa, qb;  // the chunk's 32 quant bytes
  uint4 hdr;     // d, dmin, scales[12] of the super-block
};

GI_DEVINL void q4k_load(Q4kRaw& r, const uint8_t* wrow, int chunk, bool valid) {
  if (!valid) {
    r.qa = r.qb = r.hdr = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint8_t* blk = wrow + (size_t)(chunk >> 2) * 144;
  r.hdr = ldg_nc128(blk);
  r.qa = ldg_nc128(blk + 16 + 32 * (chunk & 3));
  r.qb = ldg_nc128(blk + 32 + 32 * (chunk & 3));
}

// Words 4u..4u+3 of the operand row: unit u (8 fp16 of K) from quant word w.
GI_DEVINL void q4k_word(uint32_t (&o)[32], int u, uint32_t w, uint32_t s_lo, uint32_t c_lo, uint32_t s_hi,
                        uint32_t c_hi) {
  const uint32_t a0 = and_or(w, 0x000F000Fu, 0x64006400u);       // 1024 + q (4u, 4u+2)
  const uint32_t a1 = and_or(w >> 8, 0x000F000Fu, 0x64006400u);  // 1024 + q (4u+1, 4u+3)
  const uint32_t a2 = and_or(w, 0x00F000F0u, 0x64006400u);       // 1024 + 16q (high nibbles)
  const uint32_t a3 = and_or(w >> 8, 0x00F000F0u, 0x64006400u);
  o[4 * u + 0] = hfma2_u32(a0, s_lo, c_lo);
  o[4 * u + 1] = hfma2_u32(a1, s_lo, c_lo);
  o[4 * u + 2] = hfma2_u32(a2, s_hi, c_hi);
  o[4 * u + 3] = hfma2_u32(a3, s_hi, c_hi);
}

// The chunk's operand row (64 fp16 = 32 words of sc*q) in registers.
GI_DEVINL void q4k_decode(const Q4kRaw& r, int chunk, uint32_t (&o)[32]) {
  const int c = chunk & 3;
  // 6-bit scales of sub-blocks 0..3 and 4..7, one per byte (getScaleMin,
  // quant.go:201-212).
  const uint32_t sc03 = r.hdr.y & 0x3F3F3F3Fu;
  const uint32_t sc47 = (r.hdr.w & 0x0F0F0F0Fu) | ((r.hdr.y >> 2) & 0x30303030u);
  const uint32_t scw = c < 2 ? sc03 : sc47;
  const int sh = (c & 1) * 16;
  const float sl = (float)((scw >> sh) & 0xFF), shi = (float)((scw >> (sh + 8)) & 0xFF);
  const uint32_t s_lo = h2_splat(sl), c_lo = h2_splat(-1024.f * sl);
  const uint32_t s_hi = h2_splat(shi * 0.0625f), c_hi = h2_splat(-64.f * shi);
  q4k_word(o, 0, r.qa.x, s_lo, c_lo, s_hi, c_hi);
  q4k_word(o, 1, r.qa.y, s_lo, c_lo, s_hi, c_hi);
  q4k_word(o, 2, r.qa.z, s_lo, c_lo, s_hi, c_hi);
  q4k_word(o, 3, r.qa.w, s_lo, c_lo, s_hi, c_hi);
  q4k_word(o, 4, r.qb.x, s_lo, c_lo, s_hi, c_hi);
  q4k_word(o, 5, r.qb.y, s_lo, c_lo, s_hi, c_hi);
  q4k_word(o, 6, r.qb.z, s_lo, c_lo, s_hi, c_hi);
  q4k_word(o, 7, r.qb.w, s_lo, c_lo, s_hi, c_hi);
}

// Row `row` of the super-block's min operand [m_0..m_7 | m_0..m_7] (fp16).
GI_DEVINL void q4k_store_mins(const Q4kRaw& r, int row, uint32_t mins_tile) {
  const uint32_t m03 = r.hdr.z & 0x3F3F3F3Fu;
  const uint32_t m47 = ((r.hdr.w >> 4) & 0x0F0F0F0Fu) | ((r.hdr.z >> 2) & 0x30303030u);
  const uint32_t k1024 = 0x64006400u;
  // (m_a, m_b) pairs as exact fp16: (1024 + m) - 1024.
  const uint32_t p0 = hsub2_u32(prmt(m03, 0, 0x4140) | k1024, k1024);
  const uint32_t p1 = hsub2_u32(prmt(m03, 0, 0x4342) | k1024, k1024);
  const uint32_t p2 = hsub2_u32(prmt(m47, 0, 0x4140) | k1024, k1024);
  const uint32_t p3 = hsub2_u32(prmt(m47, 0, 0x4342) | k1024, k1024);
  sts128(mins_tile + plain_off(row, 0), p0, p1, p2, p3);
  sts128(mins_tile + plain_off(row, 1), p0, p1, p2, p3);
}

// Q6_K chunk c = 2h + p (h = 128-element half, p = 0/1) of a super-block:
// ql bytes [64h+32p, +32), qh bytes [32h, +32) bit pairs 2p (low nibbles)
// and 4+2p (high nibbles).  Low nibbles are elements 128h+32p+l, high
// nibbles 128h+64+32p+l; element l's scale is sc[8h+2p+l/16] (low) or
// sc[8h+4+2p+l/16] (high), quant.go:256-291.  Word u fills unit u in the same
// K order as Q4_K.  The 210-byte blocks are only 2-byte aligned, so 32-bit
// words are assembled from aligned loads with a funnel shift.
struct Q6kRaw {
  uint32_t ql[9], qh[9], sc[3];
  uint32_t shift;  // 0 or 16: misalignment of the block in bits
};

GI_DEVINL void q6k_load(Q6kRaw& r, const uint8_t* wrow, int chunk, bool valid) {
  if (!valid) {
#pragma unroll
    for (int i = 0; i < 9; ++i) r.ql[i] = r.qh[i] = 0;
    r.sc[0] = r.sc[1] = r.sc[2] = 0;
    r.shift = 0;
    return;
  }
  const int h = (chunk & 3) >> 1, p = chunk & 1;
  const uint8_t* blk = wrow + (size_t)(chunk >> 2) * 210;
  const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
  r.shift = (uint32_t)(a & 3) * 8;
  const uint8_t* base = reinterpret_cast<const uint8_t*>(a & ~(uintptr_t)3);
  // Offsets 64h+32p, 128+32h and 192+8h are multiples of 4, so the aligned
  // base + offset stays aligned.
#pragma unroll
  for (int i = 0; i < 9; ++i) r.ql[i] = ldg_nc32(base + 64 * h + 32 * p + 4 * i);
#pragma unroll
  for (int i = 0; i < 9; ++i) r.qh[i] = ldg_nc32(base + 128 + 32 * h + 4 * i);
  // The third scale word is needed (and inside the block) only when the
  // block is misaligned; aligned, it would lie past the block's last byte.
  r.sc[0] = ldg_nc32(base + 192 + 8 * h);
  r.sc[1] = ldg_nc32(base + 196 + 8 * h);
  r.sc[2] = r.shift ? ldg_nc32(base + 200 + 8 * h) : 0u;
}

// Unit u of the hi and lo operand rows from four packed (1024 + q6) pairs.
GI_DEVINL void q6k_unit(uint32_t (&hi)[32], uint32_t (&lo)[32], int u, uint32_t q0, uint32_t q1, uint32_t q2,
                        uint32_t q3, uint32_t s_lo, uint32_t s_hi) {
  const uint32_t k1056 = 0x64206420u;  // (1056, 1056): 1024 + q6 - 1056 = q6 - 32
  const uint32_t v0 = hsub2_u32(q0, k1056), v1 = hsub2_u32(q1, k1056);
  const uint32_t v2 = hsub2_u32(q2, k1056), v3 = hsub2_u32(q3, k1056);
  const uint32_t h0 = hmul2_u32(v0, s_lo), h1 = hmul2_u32(v1, s_lo);
  const uint32_t h2 = hmul2_u32(v2, s_hi), h3 = hmul2_u32(v3, s_hi);
  const uint32_t sign = 0x80008000u;
  hi[4 * u + 0] = h0;
  hi[4 * u + 1] = h1;
  hi[4 * u + 2] = h2;
  hi[4 * u + 3] = h3;
  // sc*q - fp16(sc*q): an exact small integer.
  lo[4 * u + 0] = hfma2_u32(v0, s_lo, h0 ^ sign);
  lo[4 * u + 1] = hfma2_u32(v1, s_lo, h1 ^ sign);
  lo[4 * u + 2] = hfma2_u32(v2, s_hi, h2 ^ sign);
  lo[4 * u + 3] = hfma2_u32(v3, s_hi, h3 ^ sign);
}

GI_DEVINL void q6k_decode(const Q6kRaw& r, int chunk, uint32_t (&hi)[32], uint32_t (&lo)[32]) {
  const int p = chunk & 1;
  const uint32_t sc0 = __funnelshift_r(r.sc[0], r.sc[1], r.shift);  // sc[8h .. 8h+3]
  const uint32_t sc1 = __funnelshift_r(r.sc[1], r.sc[2], r.shift);  // sc[8h+4 .. 8h+7]
  // Scales as exact fp16 splats: low group (u < 4, u >= 4), high group.
  const int sh = 16 * p;
  const uint32_t sl0 = h2_splat((float)(int8_t)(sc0 >> sh)), sl1 = h2_splat((float)(int8_t)(sc0 >> (sh + 8)));
  const uint32_t sh0 = h2_splat((float)(int8_t)(sc1 >> sh)), sh1 = h2_splat((float)(int8_t)(sc1 >> (sh + 8)));
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const uint32_t ql = __funnelshift_r(r.ql[u], r.ql[u + 1], r.shift);
    const uint32_t qh = __funnelshift_r(r.qh[u], r.qh[u + 1], r.shift) >> (2 * p);
    const uint32_t k = 0x64006400u;
    const uint32_t q0 = (ql & 0x000F000Fu) | ((qh << 4) & 0x00300030u) | k;          // low, (4u, 4u+2)
    const uint32_t q1 = ((ql >> 8) & 0x000F000Fu) | ((qh >> 4) & 0x00300030u) | k;   // low, (4u+1, 4u+3)
    const uint32_t q2 = ((ql >> 4) & 0x000F000Fu) | (qh & 0x00300030u) | k;          // high, (4u, 4u+2)
    const uint32_t q3 = ((ql >> 12) & 0x000F000Fu) | ((qh >> 8) & 0x00300030u) | k;  // high, (4u+1, 4u+3)
    q6k_unit(hi, lo, u, q0, q1, q2, q3, u < 4 ? sl0 : sl1, u < 4 ? sh0 : sh1);
  }
}

// Q8_0 chunk c (64 elements) of a row = blocks 2c and 2c+1: fp16 d at bytes
// 0 and 34, int8 quants at 2..33 and 36..67 (quant.go:37-41).  Word u of
// the operand fills unit u in the Q4_K K order, elements 4u.. of block 2c
// in its low half and 4u.. of block 2c+1 in its high half.  Blocks are
// 2-byte aligned: the 68 bytes are read as aligned words (the last two
// bytes by a 16-bit load when misaligned, so no read passes the chunk)
// and realigned with a funnel shift.  The first chunk of each 256-column
// super-block also carries the super-block's eight d, from which the
// decode and the epilogue derive the same power of two.
struct Q80Raw {
  uint32_t w[18];
  uint32_t shift;  // 0 or 16
  uint32_t dd[4];  // chunk & 3 == 0: the super-block's 8 fp16 d
};

GI_DEVINL void q80_load_d(uint32_t (&dd)[4], const uint8_t* wrow, int sb) {
  const uint8_t* p = wrow + (size_t)sb * 272;
#pragma unroll
  for (int k = 0; k < 4; ++k) dd[k] = ldg_nc16(p + 68 * k) | (ldg_nc16(p + 68 * k + 34) << 16);
}

// 2^E with (largest |d| of the 8) * 2^E in [64, 128) (1 for an all-zero
// super-block): fp16 d * 2^E times an int8 quant is then an fp16 hi part
// below 2^14 plus an exact fp16 residual.
GI_DEVINL float q80_sb_scale(const uint32_t (&dd)[4]) {
  uint32_t m = 0;  // fp16 magnitudes order as unsigned integers
#pragma unroll
  for (int k = 0; k < 4; ++k) m = max(m, max(dd[k] & 0x7FFFu, (dd[k] >> 16) & 0x7FFFu));
  const float f = __half2float(__ushort_as_half((unsigned short)m));
  if (!(f > 0.f) || f > 65504.f) return 1.f;
  return exp2i(6 - ilogbf(f));
}

GI_DEVINL void q80_load(Q80Raw& r, const uint8_t* wrow, int chunk, bool valid) {
  if (!valid) {
#pragma unroll
    for (int i = 0; i < 18; ++i) r.w[i] = 0;
    r.dd[0] = r.dd[1] = r.dd[2] = r.dd[3] = 0;
    r.shift = 0;
    return;
  }
  const uint8_t* blk = wrow + (size_t)chunk * 68;
  const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
  r.shift = (uint32_t)(a & 3) * 8;
  const uint8_t* base = reinterpret_cast<const uint8_t*>(a & ~(uintptr_t)3);
#pragma unroll
  for (int i = 0; i < 17; ++i) r.w[i] = ldg_nc32(base + 4 * i);
  r.w[17] = r.shift ? ldg_nc16(blk + 66) : 0u;
  if ((chunk & 3) == 0) q80_load_d(r.dd, wrow, chunk >> 2);
}

// hi = fp16(q * d), lo = q * d - hi (exact) for the quant pairs of units u.
GI_DEVINL void q80_decode(const Q80Raw& r, float scale, uint32_t (&hi)[32], uint32_t (&lo)[32]) {
  uint32_t W[17];
#pragma unroll
  for (int k = 0; k < 17; ++k) W[k] = __funnelshift_r(r.w[k], r.w[k + 1], r.shift);
  const uint32_t s0 = h2_splat(__half2float(__ushort_as_half((unsigned short)(W[0] & 0xFFFFu))) * scale);
  const uint32_t s1 = h2_splat(__half2float(__ushort_as_half((unsigned short)(W[8] >> 16))) * scale);
  const uint32_t k1152 = 0x64806480u, sign = 0x80008000u, mag = 0x64646464u;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    // quants as unsigned bytes (q + 128), two to an fp16 pair as 1024 + q + 128
    const uint32_t qa = __funnelshift_r(W[u], W[u + 1], 16) ^ 0x80808080u;  // block 2c, 4u..4u+3
    const uint32_t qb = W[9 + u] ^ 0x80808080u;                             // block 2c+1, 4u..4u+3
    const uint32_t v0 = hsub2_u32(prmt(qa, mag, 0x4240u), k1152);  // (4u, 4u+2)
    const uint32_t v1 = hsub2_u32(prmt(qa, mag, 0x4341u), k1152);  // (4u+1, 4u+3)
    const uint32_t v2 = hsub2_u32(prmt(qb, mag, 0x4240u), k1152);
    const uint32_t v3 = hsub2_u32(prmt(qb, mag, 0x4341u), k1152);
    const uint32_t h0 = hmul2_u32(v0, s0), h1 = hmul2_u32(v1, s0);
    const uint32_t h2 = hmul2_u32(v2, s1), h3 = hmul2_u32(v3, s1);
    hi[4 * u + 0] = h0;
    hi[4 * u + 1] = h1;
    hi[4 * u + 2] = h2;
    hi[4 * u + 3] = h3;
    lo[4 * u + 0] = hfma2_u32(v0, s0, h0 ^ sign);
    lo[4 * u + 1] = hfma2_u32(v1, s0, h1 ^ sign);
    lo[4 * u + 2] = hfma2_u32(v2, s1, h2 ^ sign);
    lo[4 * u + 3] = hfma2_u32(v3, s1, h3 ^ sign);
  }
}

// ---- the prefill kernel -----------------------------------------------------------

struct Params {
  const uint8_t* w;    // raw weight rows
  size_t rowb;         // bytes per weight row
  uint32_t rows, tokens, nsb;
  const uint8_t* xs;   // staged activation tiles [token tile][chunk][hi 16 KB | lo 16 KB]
  const uint8_t* sxs;  // staged sub-block sums [token tile][super-block][4 KB] (Q4_K)
  float* y;
  const float* tok_scale;
  int* error;
};

// P2: the kernel runs as CTA pairs (clusters of two along the weight-row
// tiles: the grid is (row tiles, token tiles), blockIdx.x = 2p, 2p + 1; a
// pair's two CTAs are ranks 0 and 1 of the cluster's x dimension, the
// dimension 2-SM MMA pairs are formed along).  Rank 0 issues 256-row MMAs over both
// CTAs' operands; each CTA decodes its own 128 weight rows into its own
// tensor memory, copies its own 64-token half of the activation tiles, and
// reads its own rows of D.  Arrivals meant for rank 0's barriers (decode,
// epilogue, and rank 1's copy completions, relayed by rank 1's warp 1) are
// remote mbarrier arrives; the MMA commits arrive on both CTAs' barriers.
template <int QT, bool P2>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const Params P) {
  using C = Cfg<QT>;
  constexpr int S = C::kStages;
  constexpr int kSB = stage_bytes<QT, P2>();
  constexpr int kBH = P2 ? kTileBytes / 2 : kTileBytes;  // this CTA's activation hi (and lo) tile
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023) & ~1023u;
  const uint32_t bars = sbase + S * kSB;
  // barriers: tma_full[S], prod_full[S], empty[S], acc_full[2], acc_empty[2], d2_empty, done
  auto tma_full = [&](int s) { return bars + 8 * s; };
  auto prod_full = [&](int s) { return bars + 8 * (S + s); };
  auto empty = [&](int s) { return bars + 8 * (2 * S + s); };
  auto acc_full = [&](int b) { return bars + 8 * (3 * S + b); };
  auto acc_empty = [&](int b) { return bars + 8 * (3 * S + 2 + b); };
  const uint32_t d2_empty = bars + 8 * (3 * S + 4);
  const uint32_t done_bar = bars + 8 * (3 * S + 5);
  const uint32_t tmem_slot = bars + 8 * (3 * S + 6);
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(smem_raw + (tmem_slot - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tt = P2 ? blockIdx.y : blockIdx.x;  // token tile
  const uint32_t tok0 = tt * kTileTok;
  const uint32_t row0 = (P2 ? blockIdx.x : blockIdx.y) * kTileRows;
  const int nchunk = (int)P.nsb * 4;
  const uint32_t rank = P2 ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  // Arrive on rank 0's copy of one of this CTA's barrier offsets.
  auto arrive_leader = [&](uint32_t bar) {
    if (P2) mbar_arrive_cluster(peer_addr(bar, 0));
    else mbar_arrive(bar);
  };

  // Stage s: [activation hi tile][activation lo tile][mins (Q4_K)][sub-block sums (Q4_K)].
  auto stage_bh = [&](int s) { return sbase + s * kSB; };
  auto stage_bl = [&](int s) { return stage_bh(s) + kBH; };
  auto stage_a2 = [&](int s) { return stage_bh(s) + 2 * kBH; };
  auto stage_b2 = [&](int s) { return stage_a2(s) + kSmallBytes; };

  if (threadIdx.x == 0) {
    const uint32_t pair = P2 ? 2u : 1u;
    for (int s = 0; s < S; ++s) {
      mbar_init(tma_full(s), (P2 && leader) ? 2u : 1u);  // rank 0: its own copy + rank 1's relay
      mbar_init(prod_full(s), 4 * pair);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 4 * pair);
    }
    mbar_init(d2_empty, 4 * pair);
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (P2) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  if constexpr (P2) cluster_sync();  // both CTAs' barriers initialised before any remote arrive
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot_ptr);

  if (warp == 0) {
    // ---- bulk copies of the staged activation tiles ----
    if (lane == 0) {
      int issued = 0;
      // The staged activations come from the staging kernel just before
      // this one (programmatic dependent launch: the weight decode already
      // runs while it finishes).
      griddep_wait();
      // A pair's workspace holds each chunk as [rank 0's half | rank 1's half].
      constexpr int kSums = P2 ? kSmallBytes / 2 : kSmallBytes;
      for (int i = 0; i < nchunk; ++i) {
        const int s = i % S;
        if (!wait_phase<P2>(empty(s), ((i / S) & 1) ^ 1)) {
          atomicExch(P.error, 1);
          break;
        }
        const bool mins = C::kMins && (i & 3) == 3;
        mbar_arrive_expect_tx(tma_full(s), 2 * kBH + (mins ? kSums : 0));
        // The hi and lo tiles are adjacent in the stage and in the workspace.
        bulk_load(stage_bh(s), P.xs + (((size_t)tt * nchunk + i) * (P2 ? 2 : 1) + rank) * (2 * kBH), 2 * kBH,
                  tma_full(s));
        if (mins)
          bulk_load(stage_b2(s), P.sxs + (((size_t)tt * P.nsb + (i >> 2)) * (P2 ? 2 : 1) + rank) * kSums,
                    kSums, tma_full(s));
        issued = i + 1;
      }
      // Drain: the last S issued copies must have landed before the CTA exits
      // (in a pair, rank 1's relay has observed every one of its copies).
      if (!P2 || leader)
        for (int i = issued - S < 0 ? 0 : issued - S; i < issued; ++i)
          if (!wait_phase<P2>(tma_full(i % S), (i / S) & 1)) atomicExch(P.error, 1);
    }
    __syncwarp();
  } else if (warp == 1 && !leader) {
    // ---- rank 1 of a pair: relay each of its copies' completion to rank 0,
    // then wait for rank 0's MMAs to finish with this CTA's tensor memory ----
    if (lane == 0) {
      for (int i = 0; i < nchunk; ++i) {
        const int s = i % S;
        if (!wait_phase<P2>(tma_full(s), (i / S) & 1)) {
          atomicExch(P.error, 1);
          break;
        }
        arrive_leader(tma_full(s));
      }
      if (!wait_phase<P2>(done_bar, 0)) atomicExch(P.error, 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer (rank 0 of a pair issues for both CTAs) ----
    auto mma_a = [&](uint32_t d, uint32_t a, uint64_t b, uint32_t acc) {
      if constexpr (P2) mma_f16_ts_2(d, a, b, kIdesc2, acc);
      else mma_f16_ts(d, a, b, kIdesc, acc);
    };
    auto commit = [&](uint32_t bar) {
      if constexpr (P2) mma_commit_2(bar);
      else mma_commit(bar);
    };
    if (lane == 0) {
      bool ok = true;
      for (int sb = 0; sb < (int)P.nsb && ok; ++sb) {
        const int b = sb & 1;
        if (!wait_phase<P2>(acc_empty(b), ((sb >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d1 = tmem + b * 128;
        for (int c = 0; c < 4; ++c) {
          const int i = sb * 4 + c, s = i % S;
          const uint32_t par = (i / S) & 1;
          if (!wait_phase<P2>(tma_full(s), par) || !wait_phase<P2>(prod_full(s), par)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = tmem + C::kACol + s * C::kAStageCols;
          const uint64_t bh = desc_sw128(stage_bh(s)), bl = desc_sw128(stage_bl(s));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // K step of 16 fp16: 8 tensor-memory columns of A, 32 bytes (2
            // units of the descriptor's start address) of B.
            mma_a(d1, a + 8 * k, bh + 2 * k, (c | k) != 0);
            mma_a(d1, a + 8 * k, bl + 2 * k, 1);
            if constexpr (!C::kMins) mma_a(d1, a + 32 + 8 * k, bh + 2 * k, 1);
          }
          if constexpr (C::kMins) {
            if (c == 3) {
              // The single D2 accumulator: the epilogue must have read the
              // previous super-block's.
              if (sb > 0 && !wait_phase<P2>(d2_empty, (sb - 1) & 1)) {
                ok = false;
                break;
              }
              tc_fence_after();
              // A pair's sums tile is 64 tokens: its K halves 1024 bytes apart.
              const uint64_t a2 = desc_plain(stage_a2(s), 2048, 128);
              const uint64_t b2 = desc_plain(stage_b2(s), P2 ? 1024 : 2048, 128);
              if constexpr (P2) mma_f16_2(tmem + C::kD2Col, a2, b2, kIdesc2, 0);
              else mma_f16(tmem + C::kD2Col, a2, b2, kIdesc, 0);
            }
          }
          commit(empty(s));
        }
        if (ok) commit(acc_full(b));
      }
      if (!ok) atomicExch(P.error, 1);
      // Every MMA issued must finish before tensor memory is released.
      commit(done_bar);
      if (!wait_phase<P2>(done_bar, 0)) atomicExch(P.error, 1);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ---- weight decode: one weight row per thread, written into the
    // warp's lane quarter of tensor memory ----
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const bool valid = row0 + r < P.rows;
    const uint8_t* wrow = P.w + (size_t)(valid ? row0 + r : 0) * P.rowb;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + C::kACol;
    constexpr int R = C::kPrefetch;
    using Raw = typename std::conditional<QT == kTypeQ4_K, Q4kRaw,
                                          typename std::conditional<QT == kTypeQ6_K, Q6kRaw, Q80Raw>::type>::type;
    float q80_scale = 1.f;  // Q8_0: the current super-block's power of two
    Raw ring[R];
#pragma unroll
    for (int j = 0; j < R; ++j) {
      if (j < nchunk) {
        if constexpr (QT == kTypeQ4_K) q4k_load(ring[j], wrow, j, valid);
        else if constexpr (QT == kTypeQ6_K) q6k_load(ring[j], wrow, j, valid);
        else q80_load(ring[j], wrow, j, valid);
      }
    }
    bool ok = true;
    for (int base = 0; base < nchunk && ok; base += R) {
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const int i = base + j;
        if (i < nchunk && ok) {
          const int s = i % S;
          if (!warp_wait_phase<P2>(empty(s), ((i / S) & 1) ^ 1)) {
            ok = false;
          } else {
            tc_fence_after();
            const uint32_t col = lane_base + s * C::kAStageCols;
            if constexpr (QT == kTypeQ4_K) {
              uint32_t o[32];
              q4k_decode(ring[j], i, o);
              tmem_st32(col, o);
              if ((i & 3) == 3) {
                q4k_store_mins(ring[j], r, stage_a2(s));
                fence_proxy_async_smem();
              }
            } else {
              uint32_t hi[32], lo[32];
              if constexpr (QT == kTypeQ6_K) {
                q6k_decode(ring[j], i, hi, lo);
              } else {
                if ((i & 3) == 0) q80_scale = q80_sb_scale(ring[j].dd);
                q80_decode(ring[j], q80_scale, hi, lo);
              }
              tmem_st32(col, hi);
              tmem_st32(col + 32, lo);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_leader(prod_full(s));
            if (i + R < nchunk) {
              if constexpr (QT == kTypeQ4_K) q4k_load(ring[j], wrow, i + R, valid);
              else if constexpr (QT == kTypeQ6_K) q6k_load(ring[j], wrow, i + R, valid);
              else q80_load(ring[j], wrow, i + R, valid);
            }
          }
        }
      }
    }
    if (!ok) atomicExch(P.error, 1);
    __syncwarp();
  } else {
    // ---- epilogue: lane quarter (warp % 4) of the accumulators ----
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t row = row0 + r;
    const bool valid = row < P.rows;
    const uint8_t* wrow = P.w + (size_t)(valid ? row : 0) * P.rowb;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    float acc[kTileTok];
#pragma unroll
    for (int t = 0; t < kTileTok; ++t) acc[t] = 0.f;
    // d (and dmin) of the row's super-block as an fp16 pair; Q8_0: the
    // float bits of 2^-E, the super-block's power of two divided out.
    auto load_scale = [&](int sb) -> uint32_t {
      if (!valid) return 0u;
      if constexpr (QT == kTypeQ4_K) {
        return ldg_nc32(wrow + (size_t)sb * 144);
      } else if constexpr (QT == kTypeQ6_K) {
        return ldg_nc16(wrow + (size_t)sb * 210 + 208);
      } else {
        uint32_t dd[4];
        q80_load_d(dd, wrow, sb);
        return __float_as_uint(1.f / q80_sb_scale(dd));
      }
    };
    uint32_t dd = load_scale(0);
    bool ok = true;
    for (int sb = 0; sb < (int)P.nsb; ++sb) {
      const int b = sb & 1;
      const uint32_t dd_next = sb + 1 < (int)P.nsb ? load_scale(sb + 1) : 0u;
      if (!warp_wait_phase<P2>(acc_full(b), (sb >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if constexpr (C::kMins) {
        const float ndmin = -h_hi(dd);
#pragma unroll
        for (int cc = 0; cc < kTileTok / 16; ++cc) {
          float v[16];
          tmem_ld16(lane_base + C::kD2Col + 16 * cc, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[16 * cc + i] = fmaf(ndmin, v[i], acc[16 * cc + i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(d2_empty);
      }
      float d;
      if constexpr (QT == kTypeQ8_0) d = __uint_as_float(dd);
      else d = h_lo(dd);
      const uint32_t col = lane_base + b * 128;
#pragma unroll
      for (int cc = 0; cc < kTileTok / 16; ++cc) {
        float v[16];
        tmem_ld16(col + 16 * cc, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[16 * cc + i] = fmaf(d, v[i], acc[16 * cc + i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_leader(acc_empty(b));
      dd = dd_next;
    }
    griddep_wait();  // tok_scale is the staging kernel's
    if (!ok) {
      atomicExch(P.error, 1);
    } else if (valid) {
#pragma unroll
      for (int t = 0; t < kTileTok; ++t) {
        const uint32_t tok = tok0 + t;
        if (tok < P.tokens) P.y[(size_t)tok * P.rows + row] = acc[t] * __ldg(P.tok_scale + tok);
      }
    }
    __syncwarp();
  }

  tc_fence_before();
  if constexpr (P2) cluster_sync();  // no remote arrive or MMA can still reach either CTA
  else __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (P2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                   : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                   : "memory");
  }
}

// ---- activation staging ----------------------------------------------------------
//
// Per token: e such that max|x| * 2^e < 2^10 (clamped to [-120, 120]),
// tok_scale = 2^-e, and x 2^e split into fp16 hi = fp16(x 2^e) and lo =
// fp16(x 2^e - hi).  The halves are written as the exact shared-memory image
// the MMA reads: for token tile tt and chunk i, 32 KB at xs + (tt * nchunk +
// i) * 32 KB = the hi tile then the lo tile, each 128 tokens x 64 fp16 in the
// permuted chunk order of QT, token t's 16-byte unit u at
// (t/8)*1024 + (t%8)*128 + ((u ^ t%8) * 16) (the 128-byte swizzle).  So one
// contiguous bulk copy per stage moves it.  For Q4_K also the sub-block
// sums of each super-block: 4 KB at sxs + (tt * nsb + sb) * 4 KB, 8 x 16-byte
// core matrices per 8 tokens, hi sums in K half 0 and lo sums in K half 1.
// Tokens past the batch (the last tile's padding) are written as zeros.
// P2 (CTA pairs): each 128-token tile is stored as two 64-token halves, the
// half a pair's rank copies: chunk i of tile tt at xs + ((tt * nchunk + i) *
// 2 + h) * 16 KB = [hi 8 KB | lo 8 KB] of tokens 64h .. 64h + 63, and the
// sums as 2 KB halves (K half 1 at 1024 bytes).
template <int QT, bool P2>
__global__ void __launch_bounds__(256) stage_tokens_kernel(const float* __restrict__ x, int cols, uint32_t tokens,
                                                           uint8_t* __restrict__ xs, uint8_t* __restrict__ sxs,
                                                           float* __restrict__ tok_scale) {
  __shared__ float red[8];
  griddep_launch_dependents();  // the GEMM may start: it waits for this grid before reading what it writes
  const uint32_t tok = blockIdx.x;
  const bool live = tok < tokens;
  const int tt = (int)(tok >> 7), t = (int)(tok & 127);
  const int nchunk = cols / 64, nsb = cols / 256;
  const float4* xr4 = reinterpret_cast<const float4*>(x + (size_t)(live ? tok : 0) * cols);
  float m = 0.f;
  if (live)
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) {
      const float4 v = __ldg(xr4 + i);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
  int e = 120;
  if (m >= 0x1p-100f) {
    const int E = (int)((__float_as_uint(m) >> 23) & 0xFF) - 126;  // m < 2^E
    e = min(max(10 - E, -120), 120);
  }
  const float s = live ? exp2i(e) : 0.f;
  if (threadIdx.x == 0 && live) tok_scale[tok] = exp2i(-e);

  const int th = P2 ? (t >> 6) : 0, tl = P2 ? (t & 63) : t;  // half and row within it
  const uint32_t row_off = (uint32_t)((tl >> 3) * 1024 + (tl & 7) * 128);
  for (int g = threadIdx.x; g < cols / 8; g += blockDim.x) {
    const int chunk = g >> 3, u = g & 7;
    const int sb = chunk >> 2, c = chunk & 3;
    int lo_base, hi_off;
    if (QT != kTypeQ6_K) {  // Q4_K and Q8_0: chunk c = elements 64c .. 64c + 63
      lo_base = sb * 256 + 64 * c;
      hi_off = 32;
    } else {
      lo_base = sb * 256 + 128 * (c >> 1) + 32 * (c & 1);
      hi_off = 64;
    }
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (live) {
      a = __ldg(xr4 + (lo_base + 4 * u) / 4);
      b = __ldg(xr4 + (lo_base + hi_off + 4 * u) / 4);
    }
    const float v[8] = {a.x * s, a.z * s, a.y * s, a.w * s, b.x * s, b.z * s, b.y * s, b.w * s};
    uint32_t ph[4], pl[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const __half h0 = __float2half_rn(v[2 * k]), h1 = __float2half_rn(v[2 * k + 1]);
      const __half l0 = __float2half_rn(v[2 * k] - __half2float(h0));
      const __half l1 = __float2half_rn(v[2 * k + 1] - __half2float(h1));
      ph[k] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      pl[k] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    constexpr int kHalf = P2 ? kTileBytes / 2 : kTileBytes;  // one token block's hi tile
    uint8_t* dst = xs + (((size_t)tt * nchunk + chunk) * (P2 ? 2 : 1) + th) * (2 * kHalf) + row_off +
                   ((u ^ (t & 7)) << 4);
    *reinterpret_cast<uint4*>(dst) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
    *reinterpret_cast<uint4*>(dst + kHalf) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
  }
  if (QT == kTypeQ4_K) {
    const float* xr = reinterpret_cast<const float*>(xr4);
    for (int q = threadIdx.x; q < nsb * 8; q += blockDim.x) {
      const int sb = q >> 3, j = q & 7;
      double acc = 0.0;
      if (live) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(xr + sb * 256 + 32 * j) + i);
          acc += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
        }
      }
      const double vs = acc * (double)s;
      const __half hh = __double2half(vs);
      const __half hl = __double2half(vs - (double)__half2float(hh));
      constexpr int kSums = P2 ? kSmallBytes / 2 : kSmallBytes;
      __half* dst = reinterpret_cast<__half*>(sxs + (((size_t)tt * nsb + sb) * (P2 ? 2 : 1) + th) * kSums +
                                              (tl >> 3) * 128 + (tl & 7) * 16);
      dst[j] = hh;
      dst[kSums / 4 + j] = hl;  // K half 1, kSums / 2 bytes on
    }
  }
}

// ---- host side ---------------------------------------------------------------------

struct WsLayout {
  size_t xs, sxs, scale, total;
};

WsLayout ws_layout(int64_t batch, int64_t cols) {
  auto up = [](size_t v) { return (v + 1023) & ~(size_t)1023; };
  const size_t ntt = (size_t)((batch + kTileTok - 1) / kTileTok);
  WsLayout L;
  L.xs = 0;
  L.sxs = up(ntt * (size_t)(cols / 64) * 2 * kTileBytes);
  L.scale = L.sxs + up(ntt * (size_t)(cols / 256) * kSmallBytes);
  L.total = L.scale + up((size_t)batch * 4);
  return L;
}

// CTA pairs (cluster of two, 256-row MMAs) for every launch, or single CTAs
// (the default).
bool g_pair = false;

template <int QT, bool P2>
int launch_typed(float* y, const float* x, const void* w, int64_t batch, int64_t rows, int64_t cols,
                 const GemmWorkspace& ws, int* error, cudaStream_t stream) {
  const WsLayout L = ws_layout(batch, cols);
  uint8_t* base = static_cast<uint8_t*>(ws.ptr);
  const int64_t ntt = (batch + kTileTok - 1) / kTileTok;
  stage_tokens_kernel<QT, P2><<<(unsigned)(ntt * kTileTok), 256, 0, stream>>>(
      x, (int)cols, (uint32_t)batch, base + L.xs, base + L.sxs, reinterpret_cast<float*>(base + L.scale));
  Params P;
  P.w = static_cast<const uint8_t*>(w);
  P.rowb = (size_t)row_bytes(QT, cols);
  P.rows = (uint32_t)rows;
  P.tokens = (uint32_t)batch;
  P.nsb = (uint32_t)(cols / 256);
  P.xs = base + L.xs;
  P.sxs = base + L.sxs;
  P.y = y;
  P.tok_scale = reinterpret_cast<const float*>(base + L.scale);
  P.error = error;
  unsigned row_tiles = (unsigned)((rows + kTileRows - 1) / kTileRows);
  if (!P2) {
    // Programmatic dependent launch: the weight decode of the first stages
    // overlaps the staging kernel; the copies and the scale reads wait for it.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ntt, row_tiles);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes<QT>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, prefill_kernel<QT, false>, P) == cudaSuccess ? 0 : -5;
  }
  // Pairs of row tiles; an odd last tile gets a partner whose rows are all
  // past the matrix (decoded as zeros, never stored).
  row_tiles += row_tiles & 1u;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(row_tiles, (unsigned)ntt);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes<QT, true>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prefill_kernel<QT, true>, P) == cudaSuccess ? 0 : -5;
}

template <int QT>
int launch_typed(float* y, const float* x, const void* w, int64_t batch, int64_t rows, int64_t cols,
                 const GemmWorkspace& ws, int* error, cudaStream_t stream) {
  return g_pair ? launch_typed<QT, true>(y, x, w, batch, rows, cols, ws, error, stream)
                : launch_typed<QT, false>(y, x, w, batch, rows, cols, ws, error, stream);
}

template <int QT>
cudaError_t prepare_typed() {
  cudaError_t e = cudaFuncSetAttribute(prefill_kernel<QT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem_bytes<QT>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(prefill_kernel<QT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_bytes<QT, true>());
  return e;
}

}  // namespace tc

bool gemm_tc_supported(int qtype, int64_t batch, int64_t rows, int64_t cols) {
  (void)rows;
  return (qtype == kTypeQ4_K || qtype == kTypeQ6_K || qtype == kTypeQ8_0) && batch >= kGemmTcMinBatch &&
         cols % 256 == 0 &&
         batch <= 65535 * (int64_t)tc::kTileTok && cols <= (int64_t)1 << 24;
}

size_t gemm_tc_workspace(int64_t batch, int64_t cols) { return tc::ws_layout(batch, cols).total; }

int gemm_tc_prepare_device() {
  if (tc::prepare_typed<kTypeQ4_K>() != cudaSuccess || tc::prepare_typed<kTypeQ6_K>() != cudaSuccess ||
      tc::prepare_typed<kTypeQ8_0>() != cudaSuccess)
    return -5;
  return 0;
}

void gemm_tc_set_pair(bool on) { tc::g_pair = on; }

int gemm_tc_launch(int qtype, float* y, const float* x, const void* w, int64_t batch, int64_t rows, int64_t cols,
                   const GemmWorkspace& ws, int* error, cudaStream_t stream) {
  if (!ws.ptr || ws.bytes < gemm_tc_workspace(batch, cols)) return -3;
  if (reinterpret_cast<uintptr_t>(x) % 16) return -4;
  if (qtype == kTypeQ4_K) {
    if (reinterpret_cast<uintptr_t>(w) % 16 || row_bytes(qtype, cols) % 16) return -4;
    return tc::launch_typed<kTypeQ4_K>(y, x, w, batch, rows, cols, ws, error, stream);
  }
  if (reinterpret_cast<uintptr_t>(w) % 2) return -4;
  if (qtype == kTypeQ8_0) return tc::launch_typed<kTypeQ8_0>(y, x, w, batch, rows, cols, ws, error, stream);
  return tc::launch_typed<kTypeQ6_K>(y, x, w, batch, rows, cols, ws, error, stream);
}

}  // namespace gi
