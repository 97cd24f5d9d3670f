// tp.cuh -- tensor-parallel exchange between the GPUs of one node, the
// device-side counterpart of go-infer's TPCoordinator.AllReduce
// (pkg/distributed/tensor_parallel.go:33-108): every rank contributes a
// partial vector and every rank ends with the same sum.
//
// Each rank owns one exchange region in its own HBM that every peer maps
// through CUDA IPC and writes with plain stores over NVLink:
//   recv  [2 sets][world][max_dim] float   rank r's partial vector in slot r
//   flags [2 sets][world] uint32           sequence number of rank r's push
//   argv  [2 sets][world] float2           rank r's (max logit, index bits)
//   aflag [2 sets][world] uint32           sequence number of rank r's argv
//   seq   uint32                           exchanges completed (same on every rank)
//   done  uint32                           CTAs of a pushing GEMV finished
//   rdone uint32                           CTAs of a reducing kernel finished
//   ll    [2 sets][world][max_dim] uint64  rank r's partial in slot r as
//                                          (float bits | exchange number << 32):
//                                          one 8-byte store carries value and
//                                          tag, so a reader that sees the tag
//                                          has the value (no fence, no flag)
// Exchange k uses set k & 1.  A rank can only be one exchange ahead of a
// peer (exchange k needs every rank's push k), so by the time it writes set
// k & 1 again every peer has finished reading it.  Flags start at
// 0xffffffff and are compared for equality with k, so stale values never
// match.  Sums are taken in rank order, identical on every rank.
#pragma once

#include <stdint.h>

namespace gi {

constexpr int kTpMaxWorld = 8;

struct TpDev {
  int rank = 0, world = 1, max_dim = 0;
  float* recv[kTpMaxWorld] = {};
  uint32_t* flags[kTpMaxWorld] = {};
  float2* argv[kTpMaxWorld] = {};
  uint32_t* aflag[kTpMaxWorld] = {};
  uint32_t* seq = nullptr;  // this rank's copy
  unsigned* done = nullptr;
  unsigned* rdone = nullptr;
  unsigned long long* ll[kTpMaxWorld] = {};
  int* error = nullptr;  // bounded waits that give up set it (mapped host word)
};

// Byte layout of one region.
struct TpLayout {
  size_t recv, flags, argv, aflag, seq, done, rdone, ll, total;
};

inline TpLayout tp_layout(int world, int max_dim) {
  auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
  TpLayout L;
  L.recv = 0;
  L.flags = up(L.recv + sizeof(float) * 2 * (size_t)world * max_dim);
  L.argv = up(L.flags + sizeof(uint32_t) * 2 * world);
  L.aflag = up(L.argv + 8 * 2 * (size_t)world);
  L.seq = up(L.aflag + sizeof(uint32_t) * 2 * world);
  L.done = L.seq + 128;
  L.rdone = L.done + 128;
  L.ll = up(L.rdone + 128);
  L.total = up(L.ll + sizeof(unsigned long long) * 2 * (size_t)world * max_dim);
  return L;
}

#ifdef __CUDACC__
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait (at most 2 s) for a flag to read `want`; false when it never did, or
// soon when an earlier wait has already failed (*error set), so that a
// missing peer costs one timeout, not one per exchange.  The error word is
// mapped host memory, a PCIe round trip per read: it and the clock are
// checked once every 256 polls of the flag.
__device__ __forceinline__ bool tp_wait_flag(const uint32_t* f, uint32_t want, const int* error) {
  if (ld_acquire_sys(f) == want) return true;
  const uint64_t t0 = now_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_sys(f) == want) return true;
    if ((i & 255u) == 0) {
      if (*(volatile const int*)error) return false;
      if (now_ns() - t0 > 2000000000ull) return false;
    }
  }
}
// One tagged partial: 8-byte stores and loads are single-copy atomic.
__device__ __forceinline__ void st_ll(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_ll(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Wait (at most about 2 s; the error word and the clock are read every 256
// polls) for a tagged partial; false when it never came.
__device__ __forceinline__ bool tp_wait_ll(const unsigned long long* p, uint32_t tag, const int* error, float* v) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    const unsigned long long w = ld_ll(p);
    if ((uint32_t)(w >> 32) == tag) {
      *v = __uint_as_float((uint32_t)w);
      return true;
    }
    if ((i & 255u) == 255u) {
      if (*(volatile const int*)error) return false;
      const uint64_t t = now_ns();
      if (t0 == 0)
        t0 = t;
      else if (t - t0 > 2000000000ull)
        return false;
    }
  }
}

// The rank-ordered sum of one row's tagged partials (rank r's word at
// rv + r * stride): the words of B ranks at a time are loaded at once, a
// word not yet tagged is then waited for as tp_wait_ll does, and the values
// are added in rank order.  One round trip per B ranks when the partials
// have arrived, instead of one per rank (B = 8 in the stand-alone GEMV; the
// persistent kernel, short of registers, takes 4).
template <int B = kTpMaxWorld>
__device__ __forceinline__ bool tp_sum_ll(const unsigned long long* rv, size_t stride, int world, uint32_t tag,
                                          const int* error, float* out) {
  float sum = 0.f;
#pragma unroll
  for (int r0 = 0; r0 < kTpMaxWorld; r0 += B) {
    if (r0 < world) {
      unsigned long long w[B];
#pragma unroll
      for (int u = 0; u < B; ++u)
        if (r0 + u < world) w[u] = ld_ll(rv + (size_t)(r0 + u) * stride);
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const int r = r0 + u;
        if (r < world) {
          float v;
          if ((uint32_t)(w[u] >> 32) == tag)
            v = __uint_as_float((uint32_t)w[u]);
          else if (!tp_wait_ll(rv + (size_t)r * stride, tag, error, &v))
            return false;
          sum = r == 0 ? v : __fadd_rn(sum, v);
        }
      }
    }
  }
  *out = sum;
  return true;
}
#endif

}  // namespace gi
