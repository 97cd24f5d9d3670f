// A stand-in for the CUDA runtime header, for compiling the C ABI's host
// code (go-infer_b200/csrc/capi.cu) with g++ on a machine without a GPU:
// the types, constants and entry points that file uses, implemented in
// fake_device.cc over host memory with synchronous streams.  Test
// infrastructure only.
#pragma once

#include <cstddef>
#include <cstdint>

#define __device__
#define __align__(n) __attribute__((aligned(n)))

enum cudaError_t { cudaSuccess = 0, cudaErrorInvalidValue = 1, cudaErrorMemoryAllocation = 2,
                   cudaErrorNotSupported = 801 };
enum cudaMemcpyKind { cudaMemcpyHostToHost = 0, cudaMemcpyHostToDevice = 1, cudaMemcpyDeviceToHost = 2,
                      cudaMemcpyDeviceToDevice = 3, cudaMemcpyDefault = 4 };
enum cudaMemoryType { cudaMemoryTypeUnregistered = 0, cudaMemoryTypeHost = 1, cudaMemoryTypeDevice = 2,
                      cudaMemoryTypeManaged = 3 };
enum cudaStreamCaptureMode { cudaStreamCaptureModeGlobal = 0, cudaStreamCaptureModeThreadLocal = 1,
                             cudaStreamCaptureModeRelaxed = 2 };

constexpr unsigned cudaHostAllocDefault = 0, cudaHostAllocMapped = 2, cudaStreamNonBlocking = 1,
                   cudaIpcMemLazyEnablePeerAccess = 1;

struct CUstream_st;
struct CUevent_st;
struct CUgraph_st;
struct CUgraphExec_st;
typedef CUstream_st* cudaStream_t;
typedef CUevent_st* cudaEvent_t;
typedef CUgraph_st* cudaGraph_t;
typedef CUgraphExec_st* cudaGraphExec_t;

struct float2 {
  float x, y;
};
struct cudaDeviceProp {
  int major, minor, multiProcessorCount;
};
struct cudaPointerAttributes {
  cudaMemoryType type;
  int device;
  void* devicePointer;
  void* hostPointer;
};
struct cudaIpcMemHandle_t {
  char reserved[64];
};

cudaError_t cudaGetDeviceCount(int* n);
cudaError_t cudaGetDevice(int* d);
cudaError_t cudaSetDevice(int d);
cudaError_t cudaGetDeviceProperties(cudaDeviceProp* p, int d);
cudaError_t cudaStreamCreate(cudaStream_t* s);
cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned flags);
cudaError_t cudaStreamSynchronize(cudaStream_t s);
cudaError_t cudaDeviceSynchronize();
cudaError_t cudaGetLastError();
const char* cudaGetErrorString(cudaError_t e);
cudaError_t cudaMalloc(void** p, size_t n);
template <typename T>
cudaError_t cudaMalloc(T** p, size_t n) {
  return cudaMalloc(reinterpret_cast<void**>(p), n);
}
cudaError_t cudaFree(void* p);
cudaError_t cudaHostAlloc(void** p, size_t n, unsigned flags);
cudaError_t cudaFreeHost(void* p);
cudaError_t cudaHostGetDevicePointer(void** d, void* h, unsigned flags);
cudaError_t cudaPointerGetAttributes(cudaPointerAttributes* a, const void* p);
cudaError_t cudaMemcpy(void* dst, const void* src, size_t n, cudaMemcpyKind k);
cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t n, cudaMemcpyKind k, cudaStream_t s = nullptr);
cudaError_t cudaMemset(void* p, int v, size_t n);
cudaError_t cudaMemsetAsync(void* p, int v, size_t n, cudaStream_t s = nullptr);
cudaError_t cudaEventCreate(cudaEvent_t* e);
cudaError_t cudaEventRecord(cudaEvent_t e, cudaStream_t s = nullptr);
cudaError_t cudaEventElapsedTime(float* ms, cudaEvent_t a, cudaEvent_t b);
cudaError_t cudaEventDestroy(cudaEvent_t e);
cudaError_t cudaStreamBeginCapture(cudaStream_t s, cudaStreamCaptureMode m);
cudaError_t cudaStreamEndCapture(cudaStream_t s, cudaGraph_t* g);
cudaError_t cudaGraphInstantiate(cudaGraphExec_t* e, cudaGraph_t g, unsigned long long flags = 0);
cudaError_t cudaGraphDestroy(cudaGraph_t g);
cudaError_t cudaGraphExecDestroy(cudaGraphExec_t e);
cudaError_t cudaGraphLaunch(cudaGraphExec_t e, cudaStream_t s);
cudaError_t cudaIpcGetMemHandle(cudaIpcMemHandle_t* h, void* p);
cudaError_t cudaIpcOpenMemHandle(void** p, cudaIpcMemHandle_t h, unsigned flags);
cudaError_t cudaIpcCloseMemHandle(void* p);
// A __device__ array is host memory here; registering it lets the fake
// kernels accept its address as device memory.
void fake_register_device_symbol(const void* p, size_t n);
template <typename T>
cudaError_t cudaGetSymbolAddress(void** p, const T& symbol) {
  *p = const_cast<void*>(static_cast<const void*>(&symbol));
  fake_register_device_symbol(*p, sizeof(T));
  return cudaSuccess;
}
