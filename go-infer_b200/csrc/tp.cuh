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
};

// Byte layout of one region.
struct TpLayout {
  size_t recv, flags, argv, aflag, seq, done, rdone, total;
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
  L.total = up(L.rdone + 128);
  return L;
}

}  // namespace gi
