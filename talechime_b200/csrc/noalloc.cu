// q8lin_forward_noalloc: the batched Q8_0 linear with its activation scratch in a
// fixed device array that is part of this library, so a call allocates nothing.
//
// Who needs it: callers that must not allocate device memory while they run.  A
// real-time audio producer (talechime's inference thread feeds a playback
// buffer) cannot afford cudaMalloc/cudaFree, which synchronize the device and
// can stall the stream for milliseconds; an embedder whose own allocator owns
// all device memory, or a process under a hard memory quota, may not be allowed
// to take memory behind its allocator's back.  q8lin_forward allocates its
// workspace lazily and q8lin_forward_ws needs the caller to own one; this entry
// point needs neither.
//
// The scratch is one file-scope __device__ array per GPU that loads the library:
// kNoAllocScratchBytes (9 MiB) held from module load until the process exits.
// It carries the Q8_0-quantized activations: int8 values (at most
// kNoAllocMaxValues = M*K) followed by one f32 scale per 32 values.  Every call
// on a device shares it and it keeps the last call's contents.  Nothing in it
// needs to start at zero: each call's quantize pass writes every byte that the
// call's matmul then reads.  Calls that overlap on the GPU (two streams, or two
// threads launching on different streams) race on it; calls issued on one stream
// are ordered.
//
// Host code cannot use the array's name as a device address (on the host it is
// only a stand-in symbol), so the first call on each device, with that device
// current, asks the runtime for the address with cudaGetSymbolAddress and keeps
// it.  That first call should therefore come before any stream capture.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include <cuda.h>

#include "common.cuh"
#include "internal.h"
#include "q8lin.h"

namespace q8lin {
namespace {

constexpr size_t kNoAllocMaxValues = size_t(8) << 20;                         // M*K limit
constexpr size_t kNoAllocQsBytes = kNoAllocMaxValues;                          // int8 values
constexpr size_t kNoAllocScaleBytes = (kNoAllocMaxValues / kQK) * sizeof(float);  // f32 scales
constexpr size_t kNoAllocScratchBytes = kNoAllocQsBytes + kNoAllocScaleBytes;  // 9 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 128;
std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {};
CUcontext g_ctx[kMaxDevices] = {};  // the context g_addr belongs to

// The calling thread's current CUDA context (the driver entry point is resolved once).
CUcontext current_context() {
  using CtxGetCurrentFn = CUresult (*)(CUcontext*);
  static const CtxGetCurrentFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (CtxGetCurrentFn) nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(ptr);
  }();
  CUcontext c = nullptr;
  if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}

// Device address of g_noalloc_scratch on `device` (which must be current).  Cached per
// device together with the context it was looked up in: after a device reset (a new
// primary context, the module loaded again at possibly another address) it is looked up
// again.
int scratch_address(int device, void** out) {
  if (device < 0 || device >= kMaxDevices)
    return fail(Q8LIN_ERR_DEVICE, "device ordinal " + std::to_string(device) + " beyond the supported range");
  std::lock_guard<std::mutex> lock(g_addr_mu);
  const CUcontext ctx = current_context();
  if (!g_addr[device] || !ctx || g_ctx[device] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
    g_addr[device] = p;
    g_ctx[device] = current_context();  // the lookup may have created the context
  }
  *out = g_addr[device];
  return Q8LIN_OK;
}

}  // namespace
}  // namespace q8lin

using namespace q8lin;

extern "C" int q8lin_forward_noalloc(const q8lin_weight* w, const float* x, float* y, int64_t m,
                                     q8lin_stream_t stream) {
  if (!w) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "weight handle is null");
  if (!w->packed || w->n <= 0 || w->k <= 0) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "weight handle is not initialised");
  if (m < 0) return fail(Q8LIN_ERR_SHAPE, "row count must be non-negative, got " + std::to_string(m));
  if (m == 0) return Q8LIN_OK;
  if ((size_t)m * (size_t)w->k > kNoAllocMaxValues)
    return fail(Q8LIN_ERR_SHAPE, "M*K = " + std::to_string((size_t)m * (size_t)w->k) +
                                     " exceeds the no-allocation scratch limit of " +
                                     std::to_string(kNoAllocMaxValues) +
                                     " activation values; use q8lin_forward or q8lin_forward_ws");
  if (!x || !y) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "x and y must be non-null device pointers");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(y) & 15u))
    return fail(Q8LIN_ERR_ALIGNMENT, "x and y must be 16-byte aligned");

  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (prev != w->device) {
    e = cudaSetDevice(w->device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  }
  int status = Q8LIN_OK;
  void* scratch = nullptr;
  status = scratch_address(w->device, &scratch);
  if (status == Q8LIN_OK) {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int8_t* qx = static_cast<int8_t*>(scratch);
    float* dx = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + kNoAllocQsBytes);
    e = launch_quantize_rows(x, m, w->k, qx, nullptr, dx, s);
    if (e != cudaSuccess) {
      status = cuda_fail(e, "quantize launch");
    } else {
      e = launch_gemm(*w, qx, dx, y, m, s);
      if (e != cudaSuccess) status = cuda_fail(e, "gemm launch");
    }
  }
  if (prev != w->device) cudaSetDevice(prev);
  return status;
}
