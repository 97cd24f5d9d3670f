// batch_alias.h -- host-range bookkeeping of the batch mode of the C ABI
// (plain C++, no CUDA: unit-tested on the CPU).
//
// metal_begin_batch / metal_end_batch (pkg/metal/metal_bridge.h) queue the
// calls between them on one command buffer over zero-copy host memory, so a
// call inside a batch reads what an earlier call of the same batch wrote to
// the same host slice: go-infer's prefill FFN (pkg/engine/forward.go:607-640)
// runs gate/up into batchGate, the down projection from batchGate and the
// residual add from batchFFNDown in one batch.  Here a call's output stays in
// device memory until the batch ends (one copy back per output, in call
// order), so an input must be looked up among the pending outputs first:
// PendingOutputs::resolve finds the device copy that holds the newest bytes
// of a host range, or reports that the range straddles outputs and has to be
// materialised on the host first.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

namespace gi {

struct PendingOutput {
  const void* host = nullptr;  // caller's buffer, written back at the end of the batch
  size_t bytes = 0;
  const void* dev = nullptr;   // device copy holding the newest bytes
};

enum class Resolve { kHost, kDevice, kFlush };

class PendingOutputs {
 public:
  void add(const void* host, size_t bytes, const void* dev) { list_.push_back({host, bytes, dev}); }
  void clear() { list_.clear(); }
  bool empty() const { return list_.empty(); }
  const std::vector<PendingOutput>& list() const { return list_; }

  // The newest pending output that overlaps [host, host + bytes) decides:
  // none -> the host bytes are current (kHost); it contains the range ->
  // *dev = its device copy at the same offset (kDevice); it covers only part
  // of the range -> kFlush (older outputs can hold other parts, and the host
  // bytes are stale where any output overlaps).
  Resolve resolve(const void* host, size_t bytes, const void** dev) const {
    *dev = nullptr;
    const uintptr_t a = reinterpret_cast<uintptr_t>(host), b = a + bytes;
    for (size_t i = list_.size(); i-- > 0;) {
      const PendingOutput& p = list_[i];
      const uintptr_t pa = reinterpret_cast<uintptr_t>(p.host), pb = pa + p.bytes;
      if (b <= pa || pb <= a) continue;  // disjoint
      if (pa <= a && b <= pb) {
        *dev = static_cast<const uint8_t*>(p.dev) + (a - pa);
        return Resolve::kDevice;
      }
      return Resolve::kFlush;
    }
    return Resolve::kHost;
  }

 private:
  std::vector<PendingOutput> list_;
};

}  // namespace gi
