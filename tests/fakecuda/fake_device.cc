// Fake CUDA runtime and kernels for running the C ABI's host code
// (go-infer_b200/csrc/capi.cu) on the CPU.  Test infrastructure only.
//
// Device memory is host memory kept in a registry, so every copy and every
// fake kernel checks that its pointers are on the side they should be (a
// host pointer handed to a kernel, or a device pointer copied as host
// memory, aborts the test).  Streams are synchronous.  New device memory is
// filled with 0xFF bytes (NaN floats), so reading what nothing wrote shows.
// The kernels compute y = W x with a fixed stand-in for each weight format
// (fake_weight), in index order, so the test can predict every bit.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>

#include "cuda_runtime.h"
#include "gemm.cuh"
#include "gemv.cuh"
#include "model.cuh"

namespace {

std::mutex mu;
std::map<uintptr_t, size_t> dev_heap, pinned_heap;

bool in(const std::map<uintptr_t, size_t>& heap, const void* p, size_t n) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  auto it = heap.upper_bound(a);
  if (it == heap.begin()) return false;
  --it;
  return a >= it->first && a + n <= it->first + it->second;
}

[[noreturn]] void die(const char* what, const void* p, size_t n) {
  std::printf("FAKE CUDA: %s (%p, %zu bytes)\n", what, p, n);
  std::fflush(stdout);
  std::abort();
}

void need_dev(const void* p, size_t n, const char* what) {
  std::lock_guard<std::mutex> lk(mu);
  if (!in(dev_heap, p, n)) die(what, p, n);
}

void need_host(const void* p, size_t n, const char* what) {
  std::lock_guard<std::mutex> lk(mu);
  if (in(dev_heap, p, n)) die(what, p, n);
}

float silu_mul(float g, float u) {  // kernels.go:39-46
  const float s = g / (1.0f + (float)std::exp(-(double)g));
  return s * u;
}

}  // namespace

// The stand-in value of weight (row, c): F32 rows hold floats; for the
// block formats byte j of each 256-column block's bytes gives (j - 128) / 64.
float fake_weight(int qtype, const uint8_t* row, int64_t c) {
  if (qtype == gi::kTypeF32) return reinterpret_cast<const float*>(row)[c];
  const int64_t bb = gi::row_bytes(qtype, 256);
  return ((int)row[(c / 256) * bb + (c % 256) % bb] - 128) / 64.0f;
}

float fake_silu_mul(float g, float u) { return silu_mul(g, u); }

// ---- runtime ----------------------------------------------------------------

cudaError_t cudaGetDeviceCount(int* n) { *n = 1; return cudaSuccess; }
cudaError_t cudaGetDevice(int* d) { *d = 0; return cudaSuccess; }
cudaError_t cudaSetDevice(int) { return cudaSuccess; }
cudaError_t cudaGetDeviceProperties(cudaDeviceProp* p, int) {
  p->major = 10;
  p->minor = 0;
  p->multiProcessorCount = 148;
  return cudaSuccess;
}
cudaError_t cudaStreamCreate(cudaStream_t* s) { *s = reinterpret_cast<cudaStream_t>(0x5); return cudaSuccess; }
cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned) { return cudaStreamCreate(s); }
cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaDeviceSynchronize() { return cudaSuccess; }
cudaError_t cudaGetLastError() { return cudaSuccess; }
const char* cudaGetErrorString(cudaError_t) { return "fake error"; }

cudaError_t cudaMalloc(void** p, size_t n) {
  const size_t sz = (n + 255) & ~(size_t)255;
  void* q = std::aligned_alloc(256, sz ? sz : 256);
  if (!q) return cudaErrorMemoryAllocation;
  std::memset(q, 0xFF, sz ? sz : 256);
  std::lock_guard<std::mutex> lk(mu);
  dev_heap[reinterpret_cast<uintptr_t>(q)] = sz ? sz : 256;
  *p = q;
  return cudaSuccess;
}
cudaError_t cudaFree(void* p) {
  if (!p) return cudaSuccess;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = dev_heap.find(reinterpret_cast<uintptr_t>(p));
    if (it == dev_heap.end()) die("cudaFree of a pointer that is not a device allocation", p, 0);
    dev_heap.erase(it);
  }
  std::free(p);
  return cudaSuccess;
}
cudaError_t cudaHostAlloc(void** p, size_t n, unsigned) {
  const size_t sz = (n + 255) & ~(size_t)255;
  void* q = std::aligned_alloc(256, sz ? sz : 256);
  if (!q) return cudaErrorMemoryAllocation;
  std::lock_guard<std::mutex> lk(mu);
  pinned_heap[reinterpret_cast<uintptr_t>(q)] = sz ? sz : 256;
  *p = q;
  return cudaSuccess;
}
cudaError_t cudaFreeHost(void* p) {
  if (!p) return cudaSuccess;
  {
    std::lock_guard<std::mutex> lk(mu);
    pinned_heap.erase(reinterpret_cast<uintptr_t>(p));
  }
  std::free(p);
  return cudaSuccess;
}
cudaError_t cudaHostGetDevicePointer(void** d, void* h, unsigned) { *d = h; return cudaSuccess; }
cudaError_t cudaPointerGetAttributes(cudaPointerAttributes* a, const void* p) {
  std::lock_guard<std::mutex> lk(mu);
  if (in(pinned_heap, p, 1)) {
    a->type = cudaMemoryTypeHost;
    a->devicePointer = const_cast<void*>(p);
    a->hostPointer = const_cast<void*>(p);
    return cudaSuccess;
  }
  if (in(dev_heap, p, 1)) {
    a->type = cudaMemoryTypeDevice;
    a->devicePointer = const_cast<void*>(p);
    return cudaSuccess;
  }
  return cudaErrorInvalidValue;  // pageable memory, as the runtime answers for it
}
cudaError_t cudaMemcpy(void* dst, const void* src, size_t n, cudaMemcpyKind k) {
  if (k == cudaMemcpyHostToDevice || k == cudaMemcpyDeviceToDevice) need_dev(dst, n, "copy into non-device memory");
  if (k == cudaMemcpyDeviceToHost || k == cudaMemcpyDeviceToDevice) need_dev(src, n, "copy from non-device memory");
  if (k == cudaMemcpyHostToDevice) need_host(src, n, "host-to-device copy from device memory");
  if (k == cudaMemcpyDeviceToHost) need_host(dst, n, "device-to-host copy into device memory");
  std::memmove(dst, src, n);
  return cudaSuccess;
}
cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t n, cudaMemcpyKind k, cudaStream_t) {
  return cudaMemcpy(dst, src, n, k);
}
cudaError_t cudaMemset(void* p, int v, size_t n) {
  need_dev(p, n, "memset of non-device memory");
  std::memset(p, v, n);
  return cudaSuccess;
}
cudaError_t cudaMemsetAsync(void* p, int v, size_t n, cudaStream_t) { return cudaMemset(p, v, n); }
cudaError_t cudaEventCreate(cudaEvent_t*) { return cudaErrorNotSupported; }
cudaError_t cudaEventRecord(cudaEvent_t, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t cudaEventElapsedTime(float*, cudaEvent_t, cudaEvent_t) { return cudaErrorNotSupported; }
cudaError_t cudaEventDestroy(cudaEvent_t) { return cudaSuccess; }
cudaError_t cudaStreamBeginCapture(cudaStream_t, cudaStreamCaptureMode) { return cudaErrorNotSupported; }
cudaError_t cudaStreamEndCapture(cudaStream_t, cudaGraph_t*) { return cudaErrorNotSupported; }
cudaError_t cudaGraphInstantiate(cudaGraphExec_t*, cudaGraph_t, unsigned long long) { return cudaErrorNotSupported; }
cudaError_t cudaGraphDestroy(cudaGraph_t) { return cudaSuccess; }
cudaError_t cudaGraphExecDestroy(cudaGraphExec_t) { return cudaSuccess; }
cudaError_t cudaGraphLaunch(cudaGraphExec_t, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t cudaIpcGetMemHandle(cudaIpcMemHandle_t*, void*) { return cudaErrorNotSupported; }
cudaError_t cudaIpcOpenMemHandle(void**, cudaIpcMemHandle_t, unsigned) { return cudaErrorNotSupported; }
cudaError_t cudaIpcCloseMemHandle(void*) { return cudaSuccess; }

void fake_register_device_symbol(const void* p, size_t n) {
  std::lock_guard<std::mutex> lk(mu);
  dev_heap[reinterpret_cast<uintptr_t>(p)] = n;
}

// ---- the library's kernels, faked -------------------------------------------

namespace gi {

int gemv_prepare_device() { return 0; }
int gemm_prepare_device() { return 0; }
void gemm_tc_set_pair(bool) {}

int64_t row_bytes(int qtype, int64_t cols) {
  switch (qtype) {
    case kTypeQ8_0: return (cols / 32) * 34;
    case kTypeQ4_K: return (cols / 256) * 144;
    case kTypeQ6_K: return (cols / 256) * 210;
    case kTypeF32: return cols * 4;
    default: return -1;
  }
}

int gemv_check(int qtype, int64_t rows, int64_t cols) {
  if (row_bytes(qtype, 256) < 0) return -2;
  if (rows < 1 || cols < 1) return -4;
  if (qtype == kTypeF32 ? cols % 4 != 0 : cols % 256 != 0) return -4;
  return 0;
}

static void dot_rows(int qtype, float* y, const float* x, const void* w, int64_t rows, int64_t cols) {
  const int64_t rb = row_bytes(qtype, cols);
  need_dev(w, (size_t)(rb * rows), "kernel weights not in device memory");
  need_dev(x, sizeof(float) * cols, "kernel input not in device memory");
  need_dev(y, sizeof(float) * rows, "kernel output not in device memory");
  for (int64_t r = 0; r < rows; ++r) {
    const uint8_t* row = static_cast<const uint8_t*>(w) + r * rb;
    float s = 0.f;
    for (int64_t c = 0; c < cols; ++c) s += fake_weight(qtype, row, c) * x[c];
    y[r] = s;
  }
}

int gemv_launch(int qtype, float* y, const float* x, const void* w, size_t w_bytes, int64_t rows, int64_t cols,
                const GemvScratch&, const GemvLaunch&, cudaStream_t) {
  if (int rc = gemv_check(qtype, rows, cols)) return rc;
  if (w_bytes < (size_t)(row_bytes(qtype, cols) * rows)) return -4;
  dot_rows(qtype, y, x, w, rows, cols);
  return 0;
}

int gemm_check(int qtype, int64_t batch, int64_t rows, int64_t cols) {
  return batch < 1 ? -4 : gemv_check(qtype, rows, cols);
}
size_t gemm_workspace_need(int, int64_t, int64_t, int64_t) { return 0; }
int gemm_launch(int qtype, float* y, const float* x, const void* w, size_t w_bytes, int64_t batch, int64_t rows,
                int64_t cols, const GemvScratch& s, const GemmWorkspace&, const GemvLaunch& L, cudaStream_t st) {
  for (int64_t b = 0; b < batch; ++b)
    if (int rc = gemv_launch(qtype, y + b * rows, x + b * cols, w, w_bytes, rows, cols, s, L, st)) return rc;
  return 0;
}

int gemv_multi_launch(int qtype, int nmat, float* const* y, const float* x, const void* const* w, const size_t* wb,
                      const int64_t* rows, int64_t cols, const GemvScratch& s, const GemvLaunch& L,
                      cudaStream_t st) {
  for (int m = 0; m < nmat; ++m)
    if (int rc = gemv_launch(qtype, y[m], x, w[m], wb[m], rows[m], cols, s, L, st)) return rc;
  return 0;
}

int gemv_q4k_fused(int nmat, float* const* y, const float* x, const void* const* w, const size_t* wb,
                   const int64_t* rows, int64_t cols, const GemvFuse& f, const GemvLaunch&, cudaStream_t) {
  if (nmat != 2 || f.ymode != kYSwiGLU || rows[0] != rows[1]) return -4;
  for (int m = 0; m < 2; ++m)
    if (wb[m] < (size_t)(row_bytes(kTypeQ4_K, cols) * rows[m])) return -4;
  float* g = new float[rows[0]];
  float* u = new float[rows[0]];
  // the products land in device scratch first, as the kernel keeps them on chip
  float* gd = nullptr;
  cudaMalloc(&gd, sizeof(float) * 2 * rows[0]);
  dot_rows(kTypeQ4_K, gd, x, w[0], rows[0], cols);
  dot_rows(kTypeQ4_K, gd + rows[0], x, w[1], rows[0], cols);
  std::memcpy(g, gd, sizeof(float) * rows[0]);
  std::memcpy(u, gd + rows[0], sizeof(float) * rows[0]);
  cudaFree(gd);
  need_dev(y[0], sizeof(float) * rows[0], "fused output not in device memory");
  for (int64_t r = 0; r < rows[0]; ++r) y[0][r] = silu_mul(g[r], u[r]);
  delete[] g;
  delete[] u;
  return 0;
}

cudaError_t swiglu_launch(float* gate, const float* up, int64_t n, cudaStream_t) {
  need_dev(gate, sizeof(float) * n, "swiglu operand not in device memory");
  need_dev(up, sizeof(float) * n, "swiglu operand not in device memory");
  for (int64_t i = 0; i < n; ++i) gate[i] = silu_mul(gate[i], up[i]);
  return cudaSuccess;
}

cudaError_t add_launch(float* x, const float* p, int64_t n, cudaStream_t) {
  need_dev(x, sizeof(float) * n, "residual operand not in device memory");
  need_dev(p, sizeof(float) * n, "residual operand not in device memory");
  for (int64_t i = 0; i < n; ++i) x[i] = x[i] + p[i];
  return cudaSuccess;
}

float attn_scale_for(int) { return 1.f; }
int quantize_host(int, const float*, int64_t, int64_t, uint8_t*, int) { return -2; }
int quantize_seeded(int, uint64_t, float, int64_t, int64_t, int64_t, int64_t, uint8_t*, int) { return -2; }
int synth_device(int, uint64_t, float, int64_t, int64_t, int64_t, int64_t, void*, size_t, cudaStream_t) { return -2; }

DecodeModel::~DecodeModel() {}
int DecodeModel::init(const ModelCfg&, const LayerRef*, const MatRef&, const float*, const MatRef&, int, int*,
                      const TpDev*) {
  return -1;
}
int DecodeModel::enqueue_step(cudaStream_t, bool, bool) { return -1; }
void DecodeModel::reset_cache(cudaStream_t) {}
void DecodeModel::bind(const LayerRef*, const MatRef&, const float*, const MatRef&) {}
int DecodeModel::project_partial(const MatRef&, const float*, int, cudaStream_t, bool) { return -1; }
int DecodeModel::set_persistent(bool) { return -2; }

}  // namespace gi
