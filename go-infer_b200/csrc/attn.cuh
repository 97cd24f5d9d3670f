// attn.cuh -- decode attention with GQA over the rolling KV cache
// (pkg/engine/forward.go:226-266), as device functions of one work item:
// called by the attention kernels of model.cu (one CTA per item) and by the
// persistent decode-layer kernel of layers.cu (items looped over its CTAs).
#pragma once

#include <math.h>

#include "common.cuh"
#include "model.cuh"

namespace gi {

constexpr int kAttChunk = 32;  // KV positions per attention work item

inline size_t attn_smem_bytes(int kv_mul, int hd) {
  return sizeof(float) * ((size_t)kv_mul * hd + 2 * (size_t)kAttChunk * hd + (size_t)kv_mul * kAttChunk + 2 * kv_mul);
}

// Query heads per attention item: kv_mul halved while the items (kv heads x
// chunks x head groups) number fewer than `target`.
inline int attn_heads_per_item(int kv_mul, int n_kv_heads, int splits, int target) {
  int hq = kv_mul;
  while (hq > 1 && hq % 2 == 0 && (long long)n_kv_heads * splits * (kv_mul / hq) < target) hq /= 2;
  return hq;
}

// ---- attention with GQA (forward.go:226-266), split over KV positions -------
// Item (kv head g, chunk c, head group hg) handles query heads hg*hq ..
// hg*hq + hq - 1 of g's kv_mul heads against the cache slots [32c, 32c + 32)
// of the active context (hq divides kv_mul; the callers pick it so that the
// items fill the GPU: under tensor parallelism a rank holds few kv heads,
// and each head's arithmetic is the same whatever the grouping).  It applies
// RoPE (kernels.go:22-36; rope[pos][i] = (cos, sin) of pos / theta^(2i/hd),
// computed in double on the host and rounded to float32) to its queries as
// it stages them; the items whose chunk holds this step's slot also rotate
// k, and the one of head group 0 writes k and v into the cache
// (forward.go:226-238) — no other item reads that slot from the cache.  It
// stages the chunk's K and V rows in shared memory (all loads in flight at
// once), then writes, per query head, (max, sum of exp, unnormalised output)
// for attn_combine_one.  Scores use the float64 exp of kernels.go:60.
// One item, by every thread of the calling CTA; sm: attn_smem_bytes(hq, hd)
// of shared memory.
//
// q, k, v and (in attn_combine_one) part may have been written earlier in the
// same launch by other CTAs (the persistent decode-layer kernel rewrites them
// every layer), so they are read with L2-coherent loads (__ldcg), never
// through the read-only path, whose per-SM lines could be stale.
GI_DEVINL void attn_partial_item(const StepState* __restrict__ st, const float* q, const float* k, const float* v,
                                 const float2* __restrict__ rope, float* __restrict__ kc, float* __restrict__ vc,
                                 float* part, int kv_mul, int hd, int kv_dim, int splits, float scale,
                                 uint32_t max_pos, int* error, int g, int c, int hg, int hq, float* sm) {
  const uint32_t pos = st->pos, slot = st->slot;
  if (pos >= max_pos) {  // past the RoPE table: report, touch nothing
    if (g == 0 && c == 0 && hg == 0 && threadIdx.x == 0) atomicExch(error, 1);
    return;
  }
  const int active = (int)st->active;
  const int t0 = c * kAttChunk;
  const int nt = max(0, min(kAttChunk, active - t0));
  const int half = hd >> 1, hd4 = hd >> 2;
  float* qs = sm;                          // [hq][hd]
  float* ks = qs + hq * hd;                // [kAttChunk][hd]
  float* vs = ks + kAttChunk * hd;         // [kAttChunk][hd]
  float* sc = vs + kAttChunk * hd;         // [hq][kAttChunk]
  float* mx = sc + hq * kAttChunk;         // [hq][2]
  const float2* cs = rope + (size_t)pos * half;
  // the item's queries (heads hg*hq .. hg*hq + hq - 1 of g's group), rotated
  // (r0 = v0 c - v1 s, r1 = v0 s + v1 c)
  const int h_first = g * kv_mul + hg * hq;  // the item's first query head
  const float* qg = q + (size_t)h_first * hd;
  for (int i = threadIdx.x; i < hq * half; i += blockDim.x) {
    const int h = i / half, j = i - h * half;
    const float2 r = cs[j];
    const float v0 = __ldcg(qg + h * hd + j), v1 = __ldcg(qg + h * hd + j + half);
    qs[h * hd + j] = __fsub_rn(__fmul_rn(v0, r.x), __fmul_rn(v1, r.y));
    qs[h * hd + j + half] = __fadd_rn(__fmul_rn(v0, r.y), __fmul_rn(v1, r.x));
  }
  const int cur = (int)slot - t0;  // this step's slot in the chunk, if it is here
  float4* ks4 = reinterpret_cast<float4*>(ks);
  float4* vs4 = reinterpret_cast<float4*>(vs);
  for (int i = threadIdx.x; i < nt * hd4; i += blockDim.x) {
    const int t = i / hd4, d4 = i - t * hd4;
    if (t == cur) continue;
    const size_t off = ((size_t)(t0 + t) * kv_dim + (size_t)g * hd) / 4 + d4;
    ks4[i] = __ldg(reinterpret_cast<const float4*>(kc) + off);
    vs4[i] = __ldg(reinterpret_cast<const float4*>(vc) + off);
  }
  if (cur >= 0 && cur < nt) {
    float* krow = kc + (size_t)slot * kv_dim + (size_t)g * hd;
    float* vrow = vc + (size_t)slot * kv_dim + (size_t)g * hd;
    for (int j = threadIdx.x; j < half; j += blockDim.x) {
      const float2 r = cs[j];
      const float v0 = __ldcg(k + g * hd + j), v1 = __ldcg(k + g * hd + j + half);
      const float r0 = __fsub_rn(__fmul_rn(v0, r.x), __fmul_rn(v1, r.y));
      const float r1 = __fadd_rn(__fmul_rn(v0, r.y), __fmul_rn(v1, r.x));
      ks[cur * hd + j] = r0;
      ks[cur * hd + j + half] = r1;
      if (hg == 0) {  // one item of the chunk writes the cache
        krow[j] = r0;
        krow[j + half] = r1;
      }
    }
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      const float val = __ldcg(v + g * hd + d);
      vs[cur * hd + d] = val;
      if (hg == 0) vrow[d] = val;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int p = warp; p < hq * nt; p += nw) {  // one warp per (head, position)
    const int h = p / nt, t = p - h * nt;
    float s = 0.f;
    for (int d = lane; d < hd; d += 32) s = fmaf(qs[h * hd + d], ks[t * hd + d], s);
    s = warp_sum(s);
    if (lane == 0) sc[h * kAttChunk + t] = __fmul_rn(s, scale);
  }
  __syncthreads();
  for (int h = warp; h < hq; h += nw) {  // local softmax statistics per head
    float m = -INFINITY;
    for (int t = lane; t < nt; t += 32) m = fmaxf(m, sc[h * kAttChunk + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < nt; t += 32) {
      const float e = (float)exp((double)__fsub_rn(sc[h * kAttChunk + t], m));
      sc[h * kAttChunk + t] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      mx[2 * h] = m;
      mx[2 * h + 1] = l;
    }
  }
  __syncthreads();
  for (int o = threadIdx.x; o < hq * hd; o += blockDim.x) {  // thread per (head, d)
    const int h = o / hd, d = o - h * hd;
    float a0 = 0.f, a1 = 0.f;
    int t = 0;
    for (; t + 1 < nt; t += 2) {
      a0 = fmaf(sc[h * kAttChunk + t], vs[t * hd + d], a0);
      a1 = fmaf(sc[h * kAttChunk + t + 1], vs[(t + 1) * hd + d], a1);
    }
    if (t < nt) a0 = fmaf(sc[h * kAttChunk + t], vs[t * hd + d], a0);
    float* pp = part + ((size_t)(h_first + h) * splits + c) * (hd + 2);
    pp[2 + d] = a0 + a1;
    if (d == 0) {
      pp[0] = nt > 0 ? mx[2 * h] : -INFINITY;
      pp[1] = nt > 0 ? mx[2 * h + 1] : 0.f;
    }
  }
}

// Output element (head h, dimension d): the splits' partials merged, in
// split order.  The loads of 8 splits are issued before their arithmetic
// (the partials sit in L2: one round trip per 8 splits instead of one per
// split); the operations and their order are those of a plain split loop.
GI_DEVINL void attn_combine_one(const float* part, float* __restrict__ att, int hd, int splits, int h, int d) {
  constexpr int U = 8;
  const float* ph = part + (size_t)h * splits * (hd + 2);
  const int stride = hd + 2, dd = d < hd ? d : 0;  // a thread past the head's dimensions stores nothing
  float M = -INFINITY;
  for (int s0 = 0; s0 < splits; s0 += U) {
    float m[U];
#pragma unroll
    for (int u = 0; u < U; ++u) m[u] = s0 + u < splits ? __ldcg(ph + (size_t)(s0 + u) * stride) : -INFINITY;
#pragma unroll
    for (int u = 0; u < U; ++u) M = fmaxf(M, m[u]);
  }
  float L = 0.f, acc = 0.f;
  for (int s0 = 0; s0 < splits; s0 += U) {
    float m[U], l[U], o[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const bool in = s0 + u < splits;
      const float* ps = ph + (size_t)(in ? s0 + u : 0) * stride;
      m[u] = in ? __ldcg(ps) : -INFINITY;
      l[u] = __ldcg(ps + 1);
      o[u] = __ldcg(ps + 2 + dd);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (m[u] == -INFINITY) continue;
      const float f = (float)exp((double)(m[u] - M));
      L = fmaf(l[u], f, L);
      acc = fmaf(o[u], f, acc);
    }
  }
  if (d < hd) att[(size_t)h * hd + d] = L > 0.f ? acc / L : 0.f;
}

}  // namespace gi
