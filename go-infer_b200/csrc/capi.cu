// capi.cu -- the C ABI of include/goinfer_cuda.h: device context, weight
// buffers, host<->device staging and dispatch to the sm_100a kernels.
//
// The reference seam is pkg/metal/metal_bridge.h (+ metal_bridge_darwin.m):
// a process-wide device/queue, weight buffers created once per tensor, and
// int-returning GEMV/GEMM entry points that block unless a batch is open.
// Here the process-wide state is one CUDA stream on one device plus the
// mapped error word that the kernels' bounded waits report through;
// host-pointer calls stage x/y through a device arena on that stream.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/goinfer_cuda.h"
#include "batch_alias.h"
#include "gemm.cuh"
#include "gemv.cuh"
#include "model.cuh"

namespace gi {
int quantize_host(int qtype, const float* src, int64_t rows, int64_t cols, uint8_t* dst,
                  int threads);
int quantize_seeded(int qtype, uint64_t seed, float stddev, int64_t row0, int64_t rows, int64_t col0, int64_t cols,
                    uint8_t* dst, int threads);
int synth_device(int qtype, uint64_t seed, float stddev, int64_t row0, int64_t rows, int64_t col0, int64_t cols,
                 void* dst, size_t dst_bytes, cudaStream_t stream);
}

namespace {

thread_local std::string t_err;

struct Buffer {
  void* dptr = nullptr;
  size_t bytes = 0;
  int device = -1;
};

struct Ctx {
  std::mutex mu;
  bool ready = false;
  int device = -1;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  gi::GemvScratch scratch;
  gi::GemmWorkspace gemm_ws;  // staged activations of the tensor-core prefill path
  int* err_host = nullptr;  // mapped pinned word the kernels set when a bounded wait gives up
  uint8_t* arena = nullptr;  // device activations of host-pointer calls
  size_t arena_cap = 0, arena_used = 0;
  uint8_t* pinned = nullptr;  // D2H staging of a batch's outputs
  size_t pinned_cap = 0;
  bool batch = false;
  bool pdl = false;
  bool q6k_mma = true;  // gi_cuda_set_q6k_mma
  // Outputs of the open batch: still in device memory, copied back to their
  // host buffers when the batch ends; later calls of the batch read them there.
  gi::PendingOutputs pending;
  std::vector<void*> spill;  // arena overflow blocks of the open batch
  size_t spill_bytes = 0;
};

Ctx g;

int fail(int code, const char* what, cudaError_t e = cudaSuccess) {
  char buf[256];
  if (e != cudaSuccess)
    std::snprintf(buf, sizeof buf, "%s: %s", what, cudaGetErrorString(e));
  else
    std::snprintf(buf, sizeof buf, "%s", what);
  t_err = buf;
  return code;
}

#define GI_CUDA_TRY(call, what)                      \
  do {                                               \
    cudaError_t e_ = (call);                         \
    if (e_ != cudaSuccess) return fail(-5, what, e_); \
  } while (0)


int init_locked(int device) {
  if (g.ready) {
    if (device >= 0 && device != g.device) return fail(-1, "gi_cuda_init: already bound to another device");
    return cudaSetDevice(g.device) == cudaSuccess ? 0 : fail(-5, "cudaSetDevice");
  }
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return fail(-1, "no CUDA device");
  if (device < 0) {
    const char* env = std::getenv("GOINFER_CUDA_DEVICE");
    if (env && *env) device = std::atoi(env);
    else GI_CUDA_TRY(cudaGetDevice(&device), "cudaGetDevice");
  }
  if (device < 0 || device >= n) return fail(-1, "gi_cuda_init: device ordinal out of range");
  GI_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  GI_CUDA_TRY(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major < 10) return fail(-1, "gi_cuda_init: the kernels are built for sm_100a");
  g.sm_count = prop.multiProcessorCount;
  GI_CUDA_TRY(cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking), "cudaStreamCreate");
  if (gi::gemv_prepare_device() != 0 || gi::gemm_prepare_device() != 0)
    return fail(-5, "kernel attribute set-up", cudaGetLastError());
  GI_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&g.err_host), sizeof(int), cudaHostAllocMapped),
              "cudaHostAlloc error word");
  *g.err_host = 0;
  GI_CUDA_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(&g.scratch.error), g.err_host, 0),
              "cudaHostGetDevicePointer");
  g.device = device;
  g.ready = true;
  return 0;
}

int ensure_ready() {
  if (!g.ready) return fail(-1, "gi_cuda_init has not succeeded");
  GI_CUDA_TRY(cudaSetDevice(g.device), "cudaSetDevice");
  return 0;
}

// Device scratch for activations of host-pointer calls (bump allocator,
// reset when the call or the batch completes).
int arena_alloc(size_t bytes, void** out) {
  bytes = (bytes + 255) & ~(size_t)255;
  if (g.arena_used + bytes > g.arena_cap) {
    if (g.arena_used != 0 && g.batch) {
      // Earlier calls of the batch keep their data where it is: a separate
      // block until the batch ends (the arena then grows to the batch's size).
      void* p = nullptr;
      GI_CUDA_TRY(cudaMalloc(&p, bytes), "cudaMalloc batch activations");
      g.spill.push_back(p);
      g.spill_bytes += bytes;
      *out = p;
      return 0;
    }
    if (g.arena_used != 0) return fail(-3, "activation arena exhausted");
    if (g.arena) cudaFree(g.arena);
    g.arena = nullptr;
    size_t cap = g.arena_cap ? g.arena_cap : (size_t)8 << 20;
    while (cap < bytes) cap *= 2;
    GI_CUDA_TRY(cudaMalloc(&g.arena, cap), "cudaMalloc arena");
    g.arena_cap = cap;
  }
  *out = g.arena + g.arena_used;
  g.arena_used += bytes;
  return 0;
}

// Copy the batch's pending outputs back to their host buffers, in call
// order, after everything queued so far; the list is empty afterwards.
int flush_pending_locked() {
  if (g.pending.empty()) return 0;
  const std::vector<gi::PendingOutput> list = g.pending.list();
  g.pending.clear();
  size_t total = 0;
  for (const gi::PendingOutput& p : list) total += (p.bytes + 255) & ~(size_t)255;
  if (total > g.pinned_cap) {
    if (g.pinned) cudaFreeHost(g.pinned);
    g.pinned = nullptr;
    g.pinned_cap = 0;
    size_t cap = (size_t)8 << 20;
    while (cap < total) cap *= 2;
    GI_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&g.pinned), cap, cudaHostAllocDefault), "cudaHostAlloc");
    g.pinned_cap = cap;
  }
  size_t off = 0;
  for (const gi::PendingOutput& p : list) {
    GI_CUDA_TRY(cudaMemcpyAsync(g.pinned + off, p.dev, p.bytes, cudaMemcpyDeviceToHost, g.stream), "copy y to host");
    off += (p.bytes + 255) & ~(size_t)255;
  }
  GI_CUDA_TRY(cudaStreamSynchronize(g.stream), "batched kernels");
  off = 0;
  for (const gi::PendingOutput& p : list) {
    std::memcpy(const_cast<void*>(p.host), g.pinned + off, p.bytes);
    off += (p.bytes + 255) & ~(size_t)255;
  }
  return 0;
}

// A host input of a call inside a batch: *dev = the device copy of the
// pending output holding its newest bytes, or nullptr when the host bytes
// are current (outside a batch, untouched by the batch, or made current by
// flushing outputs that the range straddles).
int batch_input(const void* host, size_t bytes, const void** dev) {
  *dev = nullptr;
  if (!g.batch) return 0;
  switch (g.pending.resolve(host, bytes, dev)) {
    case gi::Resolve::kHost:
    case gi::Resolve::kDevice:
      return 0;
    case gi::Resolve::kFlush:
      *dev = nullptr;
      return flush_pending_locked();
  }
  return 0;
}

// Input x of a batched call on the device: a pending output read in place
// (copied into `slot` when it is not 16-byte aligned), else the host bytes
// copied into `slot`.
int stage_input(const float* x, size_t bytes, void* slot, const float** xd) {
  const void* fwd = nullptr;
  if (int rc = batch_input(x, bytes, &fwd)) return rc;
  if (fwd && (reinterpret_cast<uintptr_t>(fwd) & 15) == 0) {
    *xd = static_cast<const float*>(fwd);
    return 0;
  }
  GI_CUDA_TRY(cudaMemcpyAsync(slot, fwd ? fwd : static_cast<const void*>(x), bytes,
                              fwd ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, g.stream),
              "copy x to device");
  *xd = static_cast<const float*>(slot);
  return 0;
}

// After a batch: nothing is in flight; overflow blocks are freed and the
// arena grows to hold what the batch needed.
void release_batch_memory_locked() {
  cudaStreamSynchronize(g.stream);
  for (void* p : g.spill) cudaFree(p);
  g.spill.clear();
  if (g.spill_bytes) {
    const size_t cap = (g.arena_cap + g.spill_bytes + ((size_t)1 << 20) - 1) & ~(((size_t)1 << 20) - 1);
    if (g.arena) cudaFree(g.arena);
    g.arena = nullptr;
    g.arena_cap = 0;
    if (cudaMalloc(reinterpret_cast<void**>(&g.arena), cap) == cudaSuccess) g.arena_cap = cap;
    else g.arena = nullptr;
    g.spill_bytes = 0;
  }
  g.arena_used = 0;
}

// Finish the host-pointer call: outside a batch wait for the stream.
// A kernel gave up a bounded wait (reported through the mapped error word).
int check_device_error() {
  if (g.err_host && *reinterpret_cast<volatile int*>(g.err_host)) {
    *g.err_host = 0;
    return fail(-6, "a device-side wait timed out");
  }
  return 0;
}

int complete_locked() {
  if (g.batch) return 0;
  GI_CUDA_TRY(cudaStreamSynchronize(g.stream), "kernel execution");
  g.arena_used = 0;
  return check_device_error();
}

gi::GemvLaunch launch_cfg(bool pdl) {
  gi::GemvLaunch L;
  L.sm_count = g.sm_count;
  L.pdl = pdl;
  L.q6k_mma = g.q6k_mma;
  return L;
}

// Grow the prefill workspace to `need` bytes.  Growing waits for the device
// (work queued earlier may still read the old workspace), so a caller that
// captures CUDA graphs makes one call of its largest shape before capturing.
int ensure_gemm_ws(size_t need) {
  if (need <= g.gemm_ws.bytes) return 0;
  GI_CUDA_TRY(cudaDeviceSynchronize(), "synchronize before growing the prefill workspace");
  if (g.gemm_ws.ptr) cudaFree(g.gemm_ws.ptr);
  g.gemm_ws = gi::GemmWorkspace();
  size_t cap = (size_t)16 << 20;
  while (cap < need) cap *= 2;
  GI_CUDA_TRY(cudaMalloc(&g.gemm_ws.ptr, cap), "cudaMalloc prefill workspace");
  g.gemm_ws.bytes = cap;
  return 0;
}

int run_dev(int qtype, float* y, const float* x, const void* w, size_t w_bytes, int64_t batch,
            int64_t rows, int64_t cols, cudaStream_t s, bool pdl) {
  if (batch == 1) {
    return gi::gemv_launch(qtype, y, x, w, w_bytes, rows, cols, g.scratch, launch_cfg(pdl), s);
  }
  const int rc = ensure_gemm_ws(gi::gemm_workspace_need(qtype, batch, rows, cols));
  if (rc) return rc;
  return gi::gemm_launch(qtype, y, x, w, w_bytes, batch, rows, cols, g.scratch, g.gemm_ws, launch_cfg(pdl), s);
}

// y/x on the host, weights on the device.
int run_host_io(int qtype, float* y, const float* x, const void* wdev, size_t w_bytes,
                int64_t batch, int64_t rows, int64_t cols) {
  if (!y || !x) return fail(-4, "null y or x");
  int rc = batch == 1 ? gi::gemv_check(qtype, rows, cols) : gi::gemm_check(qtype, batch, rows, cols);
  if (rc) return fail(rc, rc == -2 ? "unsupported quant type" : "unsupported shape");
  void *xd, *yd;
  // One reservation for x and y (the arena grows only while it is empty;
  // inside a batch an overflow takes a block of its own).
  const size_t xbytes = ((sizeof(float) * batch * cols) + 255) & ~(size_t)255;
  if ((rc = arena_alloc(xbytes + sizeof(float) * batch * rows, &xd))) return rc;
  yd = static_cast<uint8_t*>(xd) + xbytes;
  // A y in page-locked host memory that the device can address (CUDA's
  // unified addressing maps cudaHostAlloc'd buffers) is written by the
  // kernel itself: no device-to-host copy.  Pageable y goes through the
  // copy, as do calls inside a batch (their y is read at EndBatch).
  float* ydirect = nullptr;
  if (!g.batch) {
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, y) == cudaSuccess) {
      if (pa.type == cudaMemoryTypeHost && pa.devicePointer) ydirect = static_cast<float*>(pa.devicePointer);
    } else {
      cudaGetLastError();
    }
  }
  const float* xin = static_cast<const float*>(xd);
  if (g.batch) {  // x may be an output of an earlier call of the batch
    if ((rc = stage_input(x, sizeof(float) * batch * cols, xd, &xin))) return rc;
  } else {
    GI_CUDA_TRY(cudaMemcpyAsync(xd, x, sizeof(float) * batch * cols, cudaMemcpyHostToDevice, g.stream),
                "copy x to device");
  }
  rc = run_dev(qtype, ydirect ? ydirect : static_cast<float*>(yd), xin, wdev, w_bytes, batch, rows, cols,
               g.stream, false);
  if (rc) return fail(rc, rc == -4 ? "unsupported shape or buffer too small" : "kernel launch failed",
                      rc == -5 ? cudaGetLastError() : cudaSuccess);
  if (ydirect) return complete_locked();
  const size_t yb = sizeof(float) * batch * rows;
  if (g.batch) {  // y reaches the host when the batch ends
    g.pending.add(y, yb, yd);
    return 0;
  }
  GI_CUDA_TRY(cudaMemcpyAsync(y, yd, yb, cudaMemcpyDeviceToHost, g.stream), "copy y to host");
  return complete_locked();
}

// Host weights: copy them for this call only (metal_gemv_q4_k wraps them
// per call too, metal_bridge_darwin.m:3424-3437).
int run_host_weights(int qtype, float* y, const float* x, const void* w, int64_t batch, int64_t rows,
                     int64_t cols) {
  if (!w) return fail(-1, "null weights");
  const int64_t rb = gi::row_bytes(qtype, cols);
  if (rb < 0) return fail(-2, "unsupported quant type");
  const size_t wb = (size_t)(rb * rows);
  void* wd = nullptr;
  GI_CUDA_TRY(cudaMalloc(&wd, wb + 64), "cudaMalloc weights");
  cudaError_t e = cudaMemcpyAsync(wd, w, wb, cudaMemcpyHostToDevice, g.stream);
  int rc = e == cudaSuccess ? run_host_io(qtype, y, x, wd, wb, batch, rows, cols) : fail(-5, "copy weights", e);
  if (g.batch) cudaStreamSynchronize(g.stream);  // the weights die with this call
  cudaFree(wd);
  return rc;
}

// ---- whole-model decode -----------------------------------------------------

// Sizes recorded by gi_cuda_alloc_buffers and the model that
// gi_cuda_forward_transformer runs on them.
struct Mirror {
  bool set = false;
  uint32_t dim = 0, hidden = 0, kv_dim = 0, vocab = 0, layers = 0, max_seq = 0;
  gi::DecodeModel* m = nullptr;
  int n_heads = 0, n_kv_heads = 0, head_dim = 0;
  float eps = 0.f, theta = 0.f, scale = 0.f;
};
Mirror g_mirror;

// Tensor-parallel exchange region of this process and its peers' mappings.
struct TpCtx {
  int world = 0, rank = -1, max_dim = 0;
  bool connected = false;
  uint8_t* region = nullptr;
  void* peer[gi::kTpMaxWorld] = {};
  gi::TpDev dev;
};
TpCtx g_tp;

void tp_release() {
  for (int r = 0; r < gi::kTpMaxWorld; ++r)
    if (g_tp.peer[r]) cudaIpcCloseMemHandle(g_tp.peer[r]);
  if (g_tp.region) cudaFree(g_tp.region);
  g_tp = TpCtx();
}

struct ModelHandle {
  gi::DecodeModel m;
  uint32_t* pinned = nullptr;  // prompt tokens staged for the per-step copies
  size_t pinned_cap = 0;
  gi::StepState* pinned_state = nullptr;
  ~ModelHandle() {
    if (pinned) cudaFreeHost(pinned);
    if (pinned_state) cudaFreeHost(pinned_state);
  }
};

const Buffer* as_buffer(gi_cuda_buffer_t b) { return static_cast<const Buffer*>(b); }

// A weight matrix of `rows` x `cols`: present, of a supported type, large enough.
int mat_ref(gi_cuda_buffer_t b, int qtype, int64_t rows, int64_t cols, gi::MatRef* out, const char* what) {
  const Buffer* B = as_buffer(b);
  if (!B || !B->dptr) return fail(-3, what);
  const int64_t rb = gi::row_bytes(qtype, cols);
  if (rb < 0) return fail(-2, what);
  if (B->bytes < (size_t)(rb * rows)) return fail(-4, what);
  out->w = B->dptr;
  out->bytes = B->bytes;
  out->qtype = qtype;
  return 0;
}

int vec_ref(gi_cuda_buffer_t b, int64_t n, const float** out, bool optional, const char* what) {
  const Buffer* B = as_buffer(b);
  if (!B || !B->dptr) {
    if (optional) {
      *out = nullptr;
      return 0;
    }
    return fail(-3, what);
  }
  if (B->bytes < sizeof(float) * (size_t)n) return fail(-4, what);
  *out = static_cast<const float*>(B->dptr);
  return 0;
}

int layer_refs(const gi_cuda_layer_weights_t* lw, uint32_t n_layers, int64_t dim, int64_t q_dim, int64_t kv_dim,
               int64_t hidden, std::vector<gi::LayerRef>* out) {
  if (!lw) return fail(-4, "null layer table");
  out->resize(n_layers);
  for (uint32_t l = 0; l < n_layers; ++l) {
    const gi_cuda_layer_weights_t& w = lw[l];
    gi::LayerRef& r = (*out)[l];
    int rc = 0;
    if ((rc = mat_ref(w.wq, w.wq_type, q_dim, dim, &r.wq, "layer wq"))) return rc;
    if ((rc = mat_ref(w.wk, w.wk_type, kv_dim, dim, &r.wk, "layer wk"))) return rc;
    if ((rc = mat_ref(w.wv, w.wv_type, kv_dim, dim, &r.wv, "layer wv"))) return rc;
    if ((rc = mat_ref(w.wo, w.wo_type, dim, q_dim, &r.wo, "layer wo"))) return rc;
    if ((rc = mat_ref(w.ffn_gate, w.ffn_gate_type, hidden, dim, &r.gate, "layer ffn_gate"))) return rc;
    if ((rc = mat_ref(w.ffn_up, w.ffn_up_type, hidden, dim, &r.up, "layer ffn_up"))) return rc;
    if ((rc = mat_ref(w.ffn_down, w.ffn_down_type, dim, hidden, &r.down, "layer ffn_down"))) return rc;
    if ((rc = vec_ref(w.attn_norm, dim, &r.attn_norm, false, "layer attn_norm"))) return rc;
    if ((rc = vec_ref(w.ffn_norm, dim, &r.ffn_norm, false, "layer ffn_norm"))) return rc;
    if ((rc = vec_ref(w.bq, q_dim, &r.bq, true, "layer bq"))) return rc;
    if ((rc = vec_ref(w.bk, kv_dim, &r.bk, true, "layer bk"))) return rc;
    if ((rc = vec_ref(w.bv, kv_dim, &r.bv, true, "layer bv"))) return rc;
  }
  return 0;
}

}  // namespace

// Fixed device scratch of gi_cuda_gemm_dev_noalloc: the prefill workspace
// (staged fp16 activation tiles, sub-block sums, per-token scales) lives in
// this module-scope array instead of memory allocated at call time.  Nothing
// in it needs to start at zero: the staging kernel writes every byte the
// GEMM reads, padding included.  One array per device context, shared by
// every call on that device: calls that overlap in time (other streams,
// other threads) race on it.
constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
void* g_noalloc_addr[kMaxDevices] = {};

// Address of g_noalloc_scratch on the bound device, looked up once per
// device with that device current (the first call does this set-up).
int noalloc_scratch(void** out) {
  if (g.device < 0 || g.device >= kMaxDevices) return fail(-1, "device ordinal out of range");
  if (!g_noalloc_addr[g.device]) {
    void* p = nullptr;
    GI_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_addr[g.device] = p;
  }
  *out = g_noalloc_addr[g.device];
  return 0;
}

}  // namespace

extern "C" {

int gi_cuda_init(void) {
  std::lock_guard<std::mutex> lk(g.mu);
  return init_locked(-1);
}

int gi_cuda_init_device(int device) {
  std::lock_guard<std::mutex> lk(g.mu);
  return init_locked(device);
}

bool gi_cuda_is_available(void) {
  std::lock_guard<std::mutex> lk(g.mu);
  return g.ready;
}

void gi_cuda_begin_batch(void) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (g.ready) g.batch = true;
}

void gi_cuda_end_batch(void) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (!g.ready || !g.batch) return;
  g.batch = false;
  cudaSetDevice(g.device);
  flush_pending_locked();  // on failure the reason is in gi_cuda_last_error
  release_batch_memory_locked();
  check_device_error();
}

gi_cuda_buffer_t gi_cuda_create_buffer(const void* ptr, size_t bytes) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (!ptr || bytes == 0 || ensure_ready()) return nullptr;
  Buffer* b = new Buffer;
  // 64 bytes of slack: kernels never read past `bytes`, the slack only keeps
  // the allocation a multiple of the 16-byte vector width.
  if (cudaMalloc(&b->dptr, bytes + 64) != cudaSuccess) {
    fail(-3, "cudaMalloc buffer");
    delete b;
    return nullptr;
  }
  cudaMemsetAsync(static_cast<uint8_t*>(b->dptr) + bytes, 0, 64, g.stream);
  if (cudaMemcpyAsync(b->dptr, ptr, bytes, cudaMemcpyHostToDevice, g.stream) != cudaSuccess ||
      cudaStreamSynchronize(g.stream) != cudaSuccess) {
    fail(-3, "copy buffer to device");
    cudaFree(b->dptr);
    delete b;
    return nullptr;
  }
  b->bytes = bytes;
  b->device = g.device;
  return b;
}

void gi_cuda_release_buffer(gi_cuda_buffer_t buf) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (!buf) return;
  Buffer* b = static_cast<Buffer*>(buf);
  if (g.ready) {
    cudaSetDevice(b->device);
    cudaStreamSynchronize(g.stream);
  }
  cudaFree(b->dptr);
  delete b;
}

const void* gi_cuda_buffer_device_ptr(gi_cuda_buffer_t buf) {
  return buf ? static_cast<Buffer*>(buf)->dptr : nullptr;
}

size_t gi_cuda_buffer_bytes(gi_cuda_buffer_t buf) { return buf ? static_cast<Buffer*>(buf)->bytes : 0; }

int gi_cuda_gemv_buf(int quant_type, float* y, const float* x, gi_cuda_buffer_t w_buf, uint32_t rows,
                     uint32_t cols) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!w_buf) return fail(-1, "null weight buffer");
  const Buffer* b = static_cast<const Buffer*>(w_buf);
  return run_host_io(quant_type, y, x, b->dptr, b->bytes, 1, rows, cols);
}

int gi_cuda_gemm_buf(int quant_type, float* y, const float* x, gi_cuda_buffer_t w_buf,
                     uint32_t batch_size, uint32_t rows, uint32_t cols) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!w_buf) return fail(-1, "null weight buffer");
  if (batch_size == 0) return fail(-4, "batch_size must be >= 1");
  const Buffer* b = static_cast<const Buffer*>(w_buf);
  return run_host_io(quant_type, y, x, b->dptr, b->bytes, batch_size, rows, cols);
}

// Gate and up of one FFN against the same host activations, SwiGLU'd:
// batch 1 is one fused GEMV launch (the decode step's gate/up kernel,
// silu(g) * u in its epilogue); larger batches run the two dequant-GEMMs of
// the prefill path and the SwiGLU kernel over the products.
int gi_cuda_gemm_fused_gate_up_buf(int quant_type, float* y, const float* x, gi_cuda_buffer_t gate_buf,
                                   gi_cuda_buffer_t up_buf, uint32_t batch_size, uint32_t rows,
                                   uint32_t cols) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  const Buffer* gb = as_buffer(gate_buf);
  const Buffer* ub = as_buffer(up_buf);
  if (!gb || !ub || !gb->dptr || !ub->dptr) return fail(-1, "null weight buffer");
  if (quant_type != GI_TYPE_Q4_K) return fail(-2, "fused gate/up: Q4_K only");
  if (!y || !x || batch_size == 0) return fail(-4, "null y or x, or batch_size 0");
  int rc = gi::gemv_check(GI_TYPE_Q4_K, rows, cols);
  if (rc) return fail(rc, "unsupported shape");
  const size_t wneed = (size_t)gi::row_bytes(GI_TYPE_Q4_K, cols) * rows;
  if (gb->bytes < wneed || ub->bytes < wneed) return fail(-4, "weight buffer smaller than rows x cols");
  const int64_t batch = batch_size;
  const size_t xbytes = ((sizeof(float) * batch * cols) + 255) & ~(size_t)255;
  const size_t ybytes = ((sizeof(float) * batch * rows) + 255) & ~(size_t)255;
  void* xd = nullptr;
  if ((rc = arena_alloc(xbytes + 2 * ybytes, &xd))) return rc;
  float* yd = reinterpret_cast<float*>(static_cast<uint8_t*>(xd) + xbytes);
  float* ud = reinterpret_cast<float*>(static_cast<uint8_t*>(xd) + xbytes + ybytes);
  const float* xin = static_cast<const float*>(xd);
  if (g.batch) {  // x may be an output of an earlier call of the batch
    if ((rc = stage_input(x, sizeof(float) * batch * cols, xd, &xin))) return rc;
  } else {
    GI_CUDA_TRY(cudaMemcpyAsync(xd, x, sizeof(float) * batch * cols, cudaMemcpyHostToDevice, g.stream),
                "copy x to device");
  }
  if (batch == 1) {
    float* ys[2] = {yd, ud};
    const void* ws[2] = {gb->dptr, ub->dptr};
    const size_t wb[2] = {gb->bytes, ub->bytes};
    const int64_t rr[2] = {rows, rows};
    gi::GemvFuse f;
    f.ymode = gi::kYSwiGLU;
    rc = gi::gemv_q4k_fused(2, ys, xin, ws, wb, rr, cols, f, launch_cfg(false), g.stream);
  } else {
    rc = run_dev(GI_TYPE_Q4_K, yd, xin, gb->dptr, gb->bytes, batch, rows, cols, g.stream, false);
    if (!rc) rc = run_dev(GI_TYPE_Q4_K, ud, xin, ub->dptr, ub->bytes, batch, rows, cols, g.stream, false);
    if (!rc && gi::swiglu_launch(yd, ud, batch * rows, g.stream) != cudaSuccess) rc = -5;
  }
  if (rc) return fail(rc, rc == -4 ? "unsupported shape" : "kernel launch failed",
                      rc == -5 ? cudaGetLastError() : cudaSuccess);
  const size_t yb = sizeof(float) * batch * rows;
  if (g.batch) {  // y reaches the host when the batch ends
    g.pending.add(y, yb, yd);
    return 0;
  }
  GI_CUDA_TRY(cudaMemcpyAsync(y, yd, yb, cudaMemcpyDeviceToHost, g.stream), "copy y to host");
  return complete_locked();
}

// a[i] = a[i] + b[i] (metal_add_residual) or silu(a[i]) * b[i] (metal_swiglu)
// over host arrays.  Inside a batch, operands that earlier calls of the
// batch produced are read from the device, and a reaches the host when the
// batch ends; a that is itself such an output is updated in place there.
static int host_elementwise(float* a, const float* b, uint32_t n, bool swiglu) {
  if (!a || !b || n == 0) return fail(-4, "null operand or zero length");
  const size_t bytes = sizeof(float) * n, slot = (bytes + 255) & ~(size_t)255;
  void* base = nullptr;
  int rc = arena_alloc(2 * slot, &base);
  if (rc) return rc;
  // b first: a lookup may flush the batch's outputs to the host, and a's
  // device copy must be taken after the last flush (an in-place update of a
  // flushed output would not reach the host).  A flush frees nothing, so a
  // device copy of b found before it stays valid.
  const void* fb = nullptr;
  if ((rc = batch_input(b, bytes, &fb))) return rc;
  const void* fa = nullptr;
  if ((rc = batch_input(a, bytes, &fa))) return rc;
  float* ad = fa ? const_cast<float*>(static_cast<const float*>(fa)) : static_cast<float*>(base);
  if (!fa)
    GI_CUDA_TRY(cudaMemcpyAsync(ad, a, bytes, cudaMemcpyHostToDevice, g.stream), "copy operand to device");
  if (!fb) {
    GI_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(base) + slot, b, bytes, cudaMemcpyHostToDevice, g.stream),
                "copy operand to device");
    fb = static_cast<uint8_t*>(base) + slot;
  }
  const cudaError_t e = swiglu ? gi::swiglu_launch(ad, static_cast<const float*>(fb), n, g.stream)
                               : gi::add_launch(ad, static_cast<const float*>(fb), n, g.stream);
  if (e != cudaSuccess) return fail(-5, swiglu ? "swiglu launch" : "residual add launch", e);
  if (g.batch) {
    if (!fa) g.pending.add(a, bytes, ad);
    return 0;
  }
  GI_CUDA_TRY(cudaMemcpyAsync(a, ad, bytes, cudaMemcpyDeviceToHost, g.stream), "copy result to host");
  return complete_locked();
}

int gi_cuda_add_residual(float* x, const float* proj, uint32_t dim) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  return host_elementwise(x, proj, dim, false);
}

int gi_cuda_swiglu(float* gate, const float* up, uint32_t hidden_dim) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  return host_elementwise(gate, up, hidden_dim, true);
}

#define GI_HOST_GEMV(name, qt)                                                            \
  int name(float* y, const float* x, const void* w, uint32_t rows, uint32_t cols) {        \
    std::lock_guard<std::mutex> lk(g.mu);                                                  \
    if (int rc = ensure_ready()) return rc;                                                \
    return run_host_weights(qt, y, x, w, 1, rows, cols);                                   \
  }
GI_HOST_GEMV(gi_cuda_gemv_q8_0, GI_TYPE_Q8_0)
GI_HOST_GEMV(gi_cuda_gemv_q4_k, GI_TYPE_Q4_K)
GI_HOST_GEMV(gi_cuda_gemv_q6_k, GI_TYPE_Q6_K)

#define GI_HOST_GEMM(name, qt)                                                                \
  int name(float* y, const float* x, const void* w, uint32_t batch, uint32_t rows, uint32_t cols) { \
    std::lock_guard<std::mutex> lk(g.mu);                                                      \
    if (int rc = ensure_ready()) return rc;                                                    \
    if (batch == 0) return fail(-4, "batch_size must be >= 1");                                \
    return run_host_weights(qt, y, x, w, batch, rows, cols);                                   \
  }
GI_HOST_GEMM(gi_cuda_gemm_q8_0, GI_TYPE_Q8_0)
GI_HOST_GEMM(gi_cuda_gemm_q4_k, GI_TYPE_Q4_K)
GI_HOST_GEMM(gi_cuda_gemm_q6_k, GI_TYPE_Q6_K)

int gi_cuda_gemv_dev(int quant_type, float* y, const float* x, const void* w, size_t w_bytes,
                     uint32_t rows, uint32_t cols, void* stream) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!y || !x || !w) return fail(-4, "null device pointer");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : g.stream;
  const int rc = run_dev(quant_type, y, x, w, w_bytes, 1, rows, cols, s, g.pdl);
  if (rc) return fail(rc, rc == -2 ? "unsupported quant type" : rc == -4 ? "unsupported shape" : "launch failed",
                      rc == -5 ? cudaGetLastError() : cudaSuccess);
  return 0;
}

int gi_cuda_gemm_dev(int quant_type, float* y, const float* x, const void* w, size_t w_bytes,
                     uint32_t batch_size, uint32_t rows, uint32_t cols, void* stream) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!y || !x || !w) return fail(-4, "null device pointer");
  if (batch_size == 0) return fail(-4, "batch_size must be >= 1");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : g.stream;
  const int rc = run_dev(quant_type, y, x, w, w_bytes, batch_size, rows, cols, s, g.pdl);
  if (rc) return fail(rc, rc == -2 ? "unsupported quant type" : rc == -4 ? "unsupported shape" : "launch failed",
                      rc == -5 ? cudaGetLastError() : cudaSuccess);
  return 0;
}

int gi_cuda_gemm_dev_noalloc(int quant_type, float* y, const float* x, const void* w, size_t w_bytes,
                             uint32_t batch_size, uint32_t rows, uint32_t cols, void* stream) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!y || !x || !w) return fail(-4, "null device pointer");
  if (batch_size == 0) return fail(-4, "batch_size must be >= 1");
  int rc = gi::gemm_check(quant_type, batch_size, rows, cols);
  if (rc) return fail(rc, rc == -2 ? "unsupported quant type" : "unsupported shape");
  const size_t need = gi::gemm_workspace_need(quant_type, batch_size, rows, cols);
  if (need > kNoAllocScratchBytes) {
    char buf[200];
    std::snprintf(buf, sizeof buf,
                  "gi_cuda_gemm_dev_noalloc: %u tokens x %u columns need %zu bytes of scratch, more than the "
                  "%zu-byte static buffer",
                  batch_size, cols, need, kNoAllocScratchBytes);
    return fail(-4, buf);
  }
  gi::GemmWorkspace ws;
  if ((rc = noalloc_scratch(&ws.ptr))) return rc;
  ws.bytes = kNoAllocScratchBytes;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : g.stream;
  rc = gi::gemm_launch(quant_type, y, x, w, w_bytes, batch_size, rows, cols, g.scratch, ws, launch_cfg(g.pdl), s);
  if (rc) return fail(rc, rc == -2 ? "unsupported quant type" : rc == -4 ? "unsupported shape" : "launch failed",
                      rc == -5 ? cudaGetLastError() : cudaSuccess);
  return 0;
}

int gi_cuda_alloc_buffers(uint32_t dim, uint32_t hidden_dim, uint32_t kv_dim, uint32_t vocab_size,
                          uint32_t num_layers, uint32_t max_seq) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!dim || !hidden_dim || !kv_dim || !vocab_size || !num_layers || !max_seq) return fail(-4, "zero size");
  delete g_mirror.m;
  g_mirror = Mirror();
  g_mirror.set = true;
  g_mirror.dim = dim;
  g_mirror.hidden = hidden_dim;
  g_mirror.kv_dim = kv_dim;
  g_mirror.vocab = vocab_size;
  g_mirror.layers = num_layers;
  g_mirror.max_seq = max_seq;
  return 0;
}

int gi_cuda_forward_transformer(const float* initial_x, float* out_logits, uint32_t* out_token,
                                const gi_cuda_layer_weights_t* layers, gi_cuda_buffer_t output_norm_buf,
                                gi_cuda_buffer_t output_weight_buf, int output_weight_type, uint32_t num_layers,
                                uint32_t dim, uint32_t hidden_dim, uint32_t kv_dim, uint32_t vocab_size,
                                uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim, uint32_t pos,
                                uint32_t slot, uint32_t max_seq, uint32_t active_context, float norm_eps,
                                float rope_theta, float attn_scale) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  Mirror& M = g_mirror;
  if (!M.set) return fail(-1, "gi_cuda_alloc_buffers has not been called");
  // a synchronous call: inside a batch, initial_x may be an earlier output
  if (int rc = flush_pending_locked()) return rc;
  if (dim != M.dim || hidden_dim != M.hidden || kv_dim != M.kv_dim || vocab_size != M.vocab ||
      num_layers != M.layers || max_seq != M.max_seq)
    return fail(-4, "sizes differ from gi_cuda_alloc_buffers");
  if (!initial_x) return fail(-4, "null initial_x");
  if (!num_heads || !num_kv_heads || num_kv_heads * head_dim != kv_dim || num_heads % num_kv_heads)
    return fail(-4, "inconsistent head layout");
  if (slot >= max_seq || active_context < 1 || active_context > max_seq) return fail(-4, "bad slot or context");
  constexpr uint32_t kMirrorMaxPos = 32768;
  if (pos >= kMirrorMaxPos) return fail(-4, "position beyond the RoPE table (32768)");
  std::vector<gi::LayerRef> refs;
  const int64_t q_dim = (int64_t)num_heads * head_dim;
  if (int rc = layer_refs(layers, num_layers, dim, q_dim, kv_dim, hidden_dim, &refs)) return rc;
  gi::MatRef out_ref, embd_ref;
  const float* onorm = nullptr;
  if (int rc = mat_ref(output_weight_buf, output_weight_type, vocab_size, dim, &out_ref, "output weight")) return rc;
  if (int rc = vec_ref(output_norm_buf, dim, &onorm, false, "output norm")) return rc;
  if (!M.m || M.n_heads != (int)num_heads || M.n_kv_heads != (int)num_kv_heads || M.head_dim != (int)head_dim ||
      M.eps != norm_eps || M.theta != rope_theta || M.scale != attn_scale) {
    delete M.m;
    M.m = new gi::DecodeModel();
    gi::ModelCfg c;
    c.n_layers = (int)num_layers;
    c.dim = (int)dim;
    c.hidden = (int)hidden_dim;
    c.n_heads = (int)num_heads;
    c.n_kv_heads = (int)num_kv_heads;
    c.head_dim = (int)head_dim;
    c.vocab = (int)vocab_size;
    c.max_seq = (int)max_seq;
    c.max_pos = (int)kMirrorMaxPos;
    c.eps = norm_eps;
    c.rope_theta = rope_theta;
    c.attn_scale = attn_scale;
    const int rc = M.m->init(c, refs.data(), embd_ref, onorm, out_ref, g.sm_count, g.scratch.error);
    if (rc) {
      delete M.m;
      M.m = nullptr;
      return fail(rc, "forward buffers");
    }
    M.n_heads = (int)num_heads;
    M.n_kv_heads = (int)num_kv_heads;
    M.head_dim = (int)head_dim;
    M.eps = norm_eps;
    M.theta = rope_theta;
    M.scale = attn_scale;
  } else {
    M.m->bind(refs.data(), embd_ref, onorm, out_ref);
  }
  gi::DecodeModel& m = *M.m;
  gi::StepState st = {};
  st.pos = pos;
  st.slot = slot;
  st.active = active_context;
  GI_CUDA_TRY(cudaMemcpyAsync(m.x(), initial_x, sizeof(float) * dim, cudaMemcpyHostToDevice, g.stream), "copy x");
  GI_CUDA_TRY(cudaMemcpyAsync(m.state(), &st, sizeof st, cudaMemcpyHostToDevice, g.stream), "copy state");
  int rc = m.enqueue_step(g.stream, false, g.pdl);
  if (rc) return fail(rc, "forward step launch", rc == -5 ? cudaGetLastError() : cudaSuccess);
  if (out_logits)
    GI_CUDA_TRY(cudaMemcpyAsync(out_logits, m.logits(), sizeof(float) * vocab_size, cudaMemcpyDeviceToHost, g.stream),
                "copy logits");
  if (out_token)
    GI_CUDA_TRY(cudaMemcpyAsync(out_token, m.tokens_out(), sizeof(uint32_t), cudaMemcpyDeviceToHost, g.stream),
                "copy token");
  GI_CUDA_TRY(cudaStreamSynchronize(g.stream), "forward step");
  return check_device_error();
}

gi_cuda_model_t gi_cuda_model_create(const gi_cuda_model_desc_t* d) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (ensure_ready()) return nullptr;
  if (!d || !d->num_layers || !d->dim || !d->num_heads || !d->num_kv_heads || !d->head_dim || !d->vocab_size ||
      !d->hidden_dim || !d->max_seq || d->num_heads % d->num_kv_heads) {
    fail(-4, "gi_cuda_model_create: bad description");
    return nullptr;
  }
  const int64_t q_dim = (int64_t)d->num_heads * d->head_dim, kv_dim = (int64_t)d->num_kv_heads * d->head_dim;
  std::vector<gi::LayerRef> refs;
  if (layer_refs(d->layers, d->num_layers, d->dim, q_dim, kv_dim, d->hidden_dim, &refs)) return nullptr;
  gi::MatRef out_ref, embd_ref;
  const float* onorm = nullptr;
  if (mat_ref(d->output_weight, d->output_weight_type, d->vocab_size, d->dim, &out_ref, "output weight") ||
      mat_ref(d->token_embd, d->token_embd_type, d->vocab_size, d->dim, &embd_ref, "token embedding") ||
      vec_ref(d->output_norm, d->dim, &onorm, false, "output norm"))
    return nullptr;
  gi::ModelCfg c;
  c.n_layers = (int)d->num_layers;
  c.dim = (int)d->dim;
  c.hidden = (int)d->hidden_dim;
  c.n_heads = (int)d->num_heads;
  c.n_kv_heads = (int)d->num_kv_heads;
  c.head_dim = (int)d->head_dim;
  c.vocab = (int)d->vocab_size;
  c.max_seq = (int)d->max_seq;
  c.max_pos = d->max_pos ? (int)d->max_pos : 32768;
  c.eps = d->norm_eps;
  c.rope_theta = d->rope_theta;
  c.attn_scale = gi::attn_scale_for((int)d->head_dim);
  c.tp_world = d->tp_world > 1 ? (int)d->tp_world : 1;
  c.tp_rank = c.tp_world > 1 ? (int)d->tp_rank : 0;
  c.vocab_offset = c.tp_world > 1 ? (int)d->vocab_offset : 0;
  if (c.tp_world > 1 && (!g_tp.connected || g_tp.world != c.tp_world || g_tp.rank != c.tp_rank ||
                         g_tp.max_dim < (int)d->dim)) {
    fail(-4, "gi_cuda_model_create: tensor parallelism not connected for this rank / world / dim");
    return nullptr;
  }
  ModelHandle* h = new ModelHandle();
  const int rc = h->m.init(c, refs.data(), embd_ref, onorm, out_ref, g.sm_count, g.scratch.error,
                           c.tp_world > 1 ? &g_tp.dev : nullptr);
  if (rc) {
    delete h;
    fail(rc, "gi_cuda_model_create: device buffers");
    return nullptr;
  }
  if (cudaHostAlloc(reinterpret_cast<void**>(&h->pinned_state), sizeof(gi::StepState), cudaHostAllocDefault) !=
      cudaSuccess) {
    delete h;
    fail(-5, "gi_cuda_model_create: pinned state");
    return nullptr;
  }
  return h;
}

void gi_cuda_model_destroy(gi_cuda_model_t model) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (!model || ensure_ready()) return;
  cudaStreamSynchronize(g.stream);
  delete static_cast<ModelHandle*>(model);
}

int gi_cuda_model_reset(gi_cuda_model_t model) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!model) return fail(-4, "null model");
  static_cast<ModelHandle*>(model)->m.reset_cache(g.stream);
  GI_CUDA_TRY(cudaStreamSynchronize(g.stream), "reset");
  return 0;
}

int gi_cuda_model_set_persistent(gi_cuda_model_t model, int enable) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!model) return fail(-4, "null model");
  ModelHandle* h = static_cast<ModelHandle*>(model);
  GI_CUDA_TRY(cudaStreamSynchronize(g.stream), "persistent layers");
  if (h->m.graph) {  // captured with the other kind of step
    cudaGraphExecDestroy(h->m.graph);
    h->m.graph = nullptr;
  }
  const int rc = h->m.set_persistent(enable != 0);
  if (rc == -2) return fail(rc, "persistent layers need Q4_K layer matrices and no biases");
  if (rc) return fail(rc, "persistent layer plan", rc == -5 ? cudaGetLastError() : cudaSuccess);
  return 0;
}

int gi_cuda_model_generate(gi_cuda_model_t model, const int32_t* tokens, uint32_t n_tokens, uint32_t start_pos,
                           uint32_t n_gen, uint32_t* out_tokens, float* out_logits, float* decode_ms) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!model || !tokens || !out_tokens || n_tokens < 1 || n_gen < 1) return fail(-4, "bad generate arguments");
  ModelHandle* h = static_cast<ModelHandle*>(model);
  gi::DecodeModel& m = h->m;
  const gi::ModelCfg& c = m.cfg();
  const uint64_t steps = (uint64_t)n_tokens + n_gen - 1;
  if ((uint64_t)start_pos + steps > (uint64_t)c.max_pos) return fail(-4, "positions beyond the RoPE table");
  if (steps > (uint64_t)m.max_out()) return fail(-4, "too many steps for one call");
  const int64_t full_vocab = (int64_t)c.vocab * c.tp_world;  // the token table is replicated
  for (uint32_t i = 0; i < n_tokens; ++i)
    if (tokens[i] < 0 || tokens[i] >= full_vocab) return fail(-4, "token id out of range");
  if (!m.graph) {
    cudaGraph_t graph = nullptr;
    GI_CUDA_TRY(cudaStreamBeginCapture(g.stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    const int rc = m.enqueue_step(g.stream, true, true);
    const cudaError_t ce = cudaStreamEndCapture(g.stream, &graph);
    if (rc || ce != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      return fail(rc ? rc : -5, "capturing the decode step", ce);
    }
    const cudaError_t ie = cudaGraphInstantiate(&m.graph, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) {
      m.graph = nullptr;
      return fail(-5, "instantiating the decode step", ie);
    }
  }
  if (h->pinned_cap < n_tokens) {
    if (h->pinned) cudaFreeHost(h->pinned);
    h->pinned = nullptr;
    h->pinned_cap = 0;
    GI_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&h->pinned), sizeof(uint32_t) * n_tokens, cudaHostAllocDefault),
                "pinned prompt");
    h->pinned_cap = n_tokens;
  }
  std::memcpy(h->pinned, tokens, sizeof(uint32_t) * n_tokens);
  gi::StepState* st = h->pinned_state;
  *st = gi::StepState();
  st->token = (uint32_t)tokens[0];
  st->pos = start_pos;
  st->slot = start_pos % (uint32_t)c.max_seq;
  st->active = start_pos + 1 < (uint32_t)c.max_seq ? start_pos + 1 : (uint32_t)c.max_seq;
  GI_CUDA_TRY(cudaMemcpyAsync(m.state(), st, sizeof *st, cudaMemcpyHostToDevice, g.stream), "copy state");
  for (uint32_t i = 0; i < n_tokens; ++i) {
    if (i > 0)  // the argmax just wrote st.token: the prompt overrides it
      GI_CUDA_TRY(cudaMemcpyAsync(&m.state()->token, h->pinned + i, sizeof(uint32_t), cudaMemcpyHostToDevice,
                                  g.stream),
                  "copy prompt token");
    GI_CUDA_TRY(cudaGraphLaunch(m.graph, g.stream), "decode step");
  }
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  GI_CUDA_TRY(cudaEventCreate(&e0), "event");
  GI_CUDA_TRY(cudaEventCreate(&e1), "event");
  cudaEventRecord(e0, g.stream);
  for (uint32_t i = 1; i < n_gen; ++i) GI_CUDA_TRY(cudaGraphLaunch(m.graph, g.stream), "decode step");
  cudaEventRecord(e1, g.stream);
  cudaError_t e = cudaMemcpyAsync(out_tokens, m.tokens_out() + (n_tokens - 1), sizeof(uint32_t) * n_gen,
                                  cudaMemcpyDeviceToHost, g.stream);
  if (e == cudaSuccess && out_logits)
    e = cudaMemcpyAsync(out_logits, m.logits(), sizeof(float) * c.vocab, cudaMemcpyDeviceToHost, g.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(g.stream);
  if (e == cudaSuccess && decode_ms) cudaEventElapsedTime(decode_ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (e != cudaSuccess) return fail(-5, "generate", e);
  return check_device_error();
}

int gi_cuda_tp_prepare(int world, uint32_t max_dim, void* handle_out) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (world < 1 || world > gi::kTpMaxWorld || max_dim < 1 || !handle_out) return fail(-4, "bad tensor-parallel size");
  tp_release();
  const gi::TpLayout L = gi::tp_layout(world, (int)max_dim);
  GI_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&g_tp.region), L.total), "cudaMalloc exchange region");
  GI_CUDA_TRY(cudaMemset(g_tp.region, 0, L.total), "clear exchange region");
  // flags start at 0xffffffff: no sequence number matches them
  GI_CUDA_TRY(cudaMemset(g_tp.region + L.flags, 0xFF, sizeof(uint32_t) * 2 * world), "init flags");
  GI_CUDA_TRY(cudaMemset(g_tp.region + L.aflag, 0xFF, sizeof(uint32_t) * 2 * world), "init flags");
  // tags start at 0xffffffff too
  GI_CUDA_TRY(cudaMemset(g_tp.region + L.ll, 0xFF, sizeof(unsigned long long) * 2 * world * max_dim), "init tags");
  GI_CUDA_TRY(cudaDeviceSynchronize(), "exchange region");
  cudaIpcMemHandle_t hnd;
  GI_CUDA_TRY(cudaIpcGetMemHandle(&hnd, g_tp.region), "cudaIpcGetMemHandle");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  std::memcpy(handle_out, &hnd, sizeof hnd);
  g_tp.world = world;
  g_tp.max_dim = (int)max_dim;
  return 0;
}

int gi_cuda_tp_connect(int rank, int world, const void* handles) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!g_tp.region || world != g_tp.world || rank < 0 || rank >= world || !handles)
    return fail(-4, "gi_cuda_tp_connect: call gi_cuda_tp_prepare with the same world first");
  const gi::TpLayout L = gi::tp_layout(world, g_tp.max_dim);
  gi::TpDev d;
  d.rank = rank;
  d.world = world;
  d.max_dim = g_tp.max_dim;
  for (int r = 0; r < world; ++r) {
    uint8_t* base = g_tp.region;
    if (r != rank) {
      cudaIpcMemHandle_t hnd;
      std::memcpy(&hnd, static_cast<const uint8_t*>(handles) + 64 * r, 64);
      void* p = nullptr;
      GI_CUDA_TRY(cudaIpcOpenMemHandle(&p, hnd, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
      g_tp.peer[r] = p;
      base = static_cast<uint8_t*>(p);
    }
    d.recv[r] = reinterpret_cast<float*>(base + L.recv);
    d.flags[r] = reinterpret_cast<uint32_t*>(base + L.flags);
    d.argv[r] = reinterpret_cast<float2*>(base + L.argv);
    d.aflag[r] = reinterpret_cast<uint32_t*>(base + L.aflag);
    d.ll[r] = reinterpret_cast<unsigned long long*>(base + L.ll);
  }
  d.seq = reinterpret_cast<uint32_t*>(g_tp.region + L.seq);
  d.done = reinterpret_cast<unsigned*>(g_tp.region + L.done);
  d.rdone = reinterpret_cast<unsigned*>(g_tp.region + L.rdone);
  g_tp.dev = d;
  g_tp.rank = rank;
  g_tp.connected = true;
  return 0;
}

int gi_cuda_tp_close(void) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  cudaDeviceSynchronize();
  tp_release();
  return 0;
}

int gi_cuda_gemv_multi_dev(int quant_type, int nmat, float* const* y, const float* x, const void* const* w,
                           const size_t* w_bytes, const uint32_t* rows, uint32_t cols, void* stream) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!y || !x || !w || !w_bytes || !rows || nmat < 1 || nmat > 3) return fail(-4, "bad multi-GEMV arguments");
  int64_t r64[3];
  for (int m = 0; m < nmat; ++m) {
    if (!y[m] || !w[m]) return fail(-4, "null device pointer");
    r64[m] = rows[m];
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : g.stream;
  const int rc = gi::gemv_multi_launch(quant_type, nmat, y, x, w, w_bytes, r64, cols, g.scratch, launch_cfg(g.pdl), s);
  if (rc) return fail(rc, rc == -2 ? "unsupported quant type" : rc == -4 ? "unsupported shape" : "launch failed",
                      rc == -5 ? cudaGetLastError() : cudaSuccess);
  return 0;
}

namespace {
// The feed-forward half of a layer on this rank's shard: gate and up with
// the RMSNorm prologue and SwiGLU epilogue into h, then down adding into x
// (under tensor parallelism the ranks' partials, summed in its epilogue).
int ffn_launch(float* x, const float* norm, const void* gate, const void* up, const void* down, size_t gate_bytes,
               size_t up_bytes, size_t down_bytes, float* h, uint32_t dim, uint32_t hidden, float eps,
               cudaStream_t s, bool pdl) {
  const gi::GemvLaunch L = launch_cfg(pdl);
  float* ys[2] = {h, h};  // the SwiGLU epilogue writes y[0]
  const void* wgu[2] = {gate, up};
  const size_t bgu[2] = {gate_bytes, up_bytes};
  const int64_t rgu[2] = {hidden, hidden};
  gi::GemvFuse f;
  f.xmode = gi::kXNorm;
  f.x2 = norm;
  f.eps = eps;
  f.ymode = gi::kYSwiGLU;
  int rc = gi::gemv_q4k_fused(2, ys, x, wgu, bgu, rgu, dim, f, L, s);
  if (rc) return rc;
  gi::TpDev tp;
  gi::GemvFuse fd;
  fd.ymode = gi::kYAdd;
  if (g_tp.connected && g_tp.world > 1) {
    if ((int)dim > g_tp.max_dim) return -4;
    tp = g_tp.dev;
    tp.error = g.scratch.error;
    fd.ymode = gi::kYPush;
    fd.tp = &tp;
  }
  float* yd[1] = {x};
  const void* wd[1] = {down};
  const size_t bd[1] = {down_bytes};
  const int64_t rd[1] = {dim};
  return gi::gemv_q4k_fused(1, yd, h, wd, bd, rd, hidden, fd, L, s);
}

int ffn_fail(int rc) {
  return fail(rc, rc == -4 ? "unsupported shape, alignment or buffer size" : "launch failed",
              rc == -5 ? cudaGetLastError() : cudaSuccess);
}
}  // namespace

int gi_cuda_ffn_dev(float* x, const float* norm, const void* gate, const void* up, const void* down,
                    size_t gate_bytes, size_t up_bytes, size_t down_bytes, float* h, uint32_t dim, uint32_t hidden,
                    float eps, void* stream) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!x || !norm || !gate || !up || !down || !h) return fail(-4, "null device pointer");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : g.stream;
  const int rc = ffn_launch(x, norm, gate, up, down, gate_bytes, up_bytes, down_bytes, h, dim, hidden, eps, s, g.pdl);
  return rc ? ffn_fail(rc) : 0;
}

int gi_cuda_ffn_buf(float* x, gi_cuda_buffer_t norm, gi_cuda_buffer_t gate, gi_cuda_buffer_t up,
                    gi_cuda_buffer_t down, uint32_t dim, uint32_t hidden, float eps) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  if (!x) return fail(-4, "null x");
  if (!norm || !gate || !up || !down) return fail(-1, "null buffer");
  if (g.batch) return fail(-4, "gi_cuda_ffn_buf: not inside gi_cuda_begin_batch / gi_cuda_end_batch");
  const Buffer* bn = static_cast<const Buffer*>(norm);
  if (bn->bytes < sizeof(float) * dim) return fail(-4, "norm buffer smaller than dim floats");
  void* xd;
  const size_t xbytes = (sizeof(float) * dim + 255) & ~(size_t)255;
  if (int rc = arena_alloc(xbytes + sizeof(float) * hidden, &xd)) return rc;
  float* hd = reinterpret_cast<float*>(static_cast<uint8_t*>(xd) + xbytes);
  GI_CUDA_TRY(cudaMemcpyAsync(xd, x, sizeof(float) * dim, cudaMemcpyHostToDevice, g.stream), "copy x to device");
  const Buffer *bg = static_cast<const Buffer*>(gate), *bu = static_cast<const Buffer*>(up),
               *bd = static_cast<const Buffer*>(down);
  const int rc = ffn_launch(static_cast<float*>(xd), static_cast<const float*>(bn->dptr), bg->dptr, bu->dptr, bd->dptr,
                            bg->bytes, bu->bytes, bd->bytes, hd, dim, hidden, eps, g.stream, false);
  if (rc) return ffn_fail(rc);
  GI_CUDA_TRY(cudaMemcpyAsync(x, xd, sizeof(float) * dim, cudaMemcpyDeviceToHost, g.stream), "copy x to host");
  return complete_locked();
}

int gi_cuda_set_pdl(int enable) {
  std::lock_guard<std::mutex> lk(g.mu);
  g.pdl = enable != 0;
  return 0;
}

int gi_cuda_set_q6k_mma(int enable) {
  std::lock_guard<std::mutex> lk(g.mu);
  g.q6k_mma = enable != 0;
  return 0;
}

int gi_cuda_set_prefill_pair(int enable) {
  std::lock_guard<std::mutex> lk(g.mu);
  gi::gemm_tc_set_pair(enable != 0);
  return 0;
}

const char* gi_cuda_last_error(void) { return t_err.c_str(); }

int64_t gi_quant_row_bytes(int quant_type, int64_t cols) { return gi::row_bytes(quant_type, cols); }

int gi_quantize_seeded(int quant_type, uint64_t seed, float stddev, int64_t row0, int64_t rows, int64_t col0,
                       int64_t cols, void* dst, int threads) {
  if (!dst) return fail(-4, "null pointer");
  if (threads <= 0) threads = (int)std::thread::hardware_concurrency();
  const int rc = gi::quantize_seeded(quant_type, seed, stddev, row0, rows, col0, cols, static_cast<uint8_t*>(dst),
                                     threads);
  if (rc) return fail(rc, rc == -2 ? "unsupported quant type" : "unsupported shape");
  return 0;
}

int gi_cuda_buffer_read(gi_cuda_buffer_t buf, void* dst, size_t bytes) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  const Buffer* b = static_cast<const Buffer*>(buf);
  if (!b || !b->dptr || !dst || bytes > b->bytes) return fail(-4, "bad buffer read");
  GI_CUDA_TRY(cudaMemcpy(dst, b->dptr, bytes, cudaMemcpyDeviceToHost), "read buffer");
  return 0;
}

gi_cuda_buffer_t gi_cuda_alloc_buffer(size_t bytes) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (ensure_ready() || bytes == 0) return nullptr;
  Buffer* b = new Buffer();
  if (cudaMalloc(&b->dptr, bytes + 64) != cudaSuccess) {
    delete b;
    fail(-3, "cudaMalloc buffer");
    return nullptr;
  }
  b->bytes = bytes;
  b->device = g.device;
  return b;
}

int gi_synth_weights(gi_cuda_buffer_t buf, int quant_type, uint64_t seed, float stddev, int64_t row0, int64_t rows,
                     int64_t col0, int64_t cols) {
  std::lock_guard<std::mutex> lk(g.mu);
  if (int rc = ensure_ready()) return rc;
  Buffer* b = static_cast<Buffer*>(buf);
  if (!b || !b->dptr) return fail(-3, "null buffer");
  const int rc = gi::synth_device(quant_type, seed, stddev, row0, rows, col0, cols, b->dptr, b->bytes, g.stream);
  if (rc) return fail(rc, rc == -2 ? "unsupported quant type" : rc == -4 ? "unsupported shape" : "launch failed",
                      rc == -5 ? cudaGetLastError() : cudaSuccess);
  GI_CUDA_TRY(cudaStreamSynchronize(g.stream), "synthetic weights");
  return 0;
}

int gi_quantize(int quant_type, const float* src, int64_t rows, int64_t cols, void* dst, int threads) {
  if (!src || !dst) return fail(-4, "null pointer");
  if (threads <= 0) threads = (int)std::thread::hardware_concurrency();
  const int rc = gi::quantize_host(quant_type, src, rows, cols, static_cast<uint8_t*>(dst), threads);
  if (rc) return fail(rc, rc == -2 ? "unsupported quant type" : "unsupported shape");
  return 0;
}

}  // extern "C"
