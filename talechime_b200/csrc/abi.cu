// C ABI of libq8lin.so (declared in include/q8lin.h): argument checks, weight
// upload/repack, workspace management and dispatch to the kernels.
#include <climits>
#include <cstring>
#include <cuda_runtime.h>
#include <stdlib.h>

#include <atomic>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "q8lin.h"

namespace q8lin {

static thread_local std::string g_last_error;

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  const int status = (e == cudaErrorMemoryAllocation) ? Q8LIN_ERR_OUT_OF_MEMORY : Q8LIN_ERR_CUDA;
  return fail(status, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

int sm_count(int device) {
  static int cache[128] = {0};
  if (device < 0 || device >= 128) return 148;
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
    cache[device] = v;
  }
  return cache[device];
}

std::atomic<uint64_t> g_wait_limit_ns{1000000000ull};

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("Q8LIN_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

namespace {

constexpr size_t kGemvSmemLimit = 200 * 1024;
constexpr size_t kAlign = 256;


// Dispatch by activation rows (crossovers measured on B200 in CUDA graphs): M <= 4
// streams the weights through the GEMV kernels, or the small-batch dp4a kernel below;
// 5 <= M <= 32 takes the small-batch kernel where it wins, else the int8 tensor-core
// path with the weights on the MMA's 128-row side; larger batches the f16 tensor-core
// GEMM.
constexpr int kGemvPathMaxM = 4;
// The small-batch streaming kernel (dp4a, gemv_mrow.cu) takes, measured on B200 in CUDA
// graphs over weight copies spanning twice the L2 (us per call, this kernel vs the
// alternative):
//   K <= 2048, 5 <= M <= 16  vs int8 tensor cores: qkv M=8 10.2 vs 17.1, o M=8 7.5 vs 14.4;
//   K <= 2048, M = 3, 4 and N*K >= 8M weights  vs the register-streaming GEMV: qkv M=4
//     7.1 vs 8.4, gate_up M=4 10.4 vs 12.7 (but o 2048x2048 M=4: 5.0 vs 4.9, and at M = 2
//     the GEMV keeps o and gate_up: 3.4 vs 4.0, 8.5 vs 8.9);
//   K > 2048, 2 <= M <= 6  vs the GEMV / int8 tensor cores: down 6144->2048 M=2 7.3 vs 8.1,
//     M=4 10.0 vs 12.6, M=6 12.8 vs 14.1 (M=8: 15.4 vs 14.3 -- there the per-CTA
//     quantization of every activation row outgrows the tensor-core path's).
// Q8LIN_MROW=0 turns it off (comparisons).
constexpr int kMrowMinM = 5;                     // K <= 2048: from here on
constexpr int kMrowSmallK = 2048;
constexpr int kMrowMaxMLongK = 6;                // K > 2048: up to here
constexpr int64_t kMrowMinWeights = 8 << 20;     // M = 3, 4 at K <= 2048: N*K at least this
bool use_mrow(int64_t m, int64_t k, int64_t n) {
  static const bool on = [] {
    const char* v = getenv("Q8LIN_MROW");
    return !(v && v[0] == '0');
  }();
  if (!on || m < 2 || m > kMrowMaxM) return false;
  bool pick;
  if (k > kMrowSmallK) pick = m <= kMrowMaxMLongK;
  else if (m >= kMrowMinM) pick = true;
  else pick = m >= 3 && n * k >= kMrowMinWeights;
  return pick && mrow_applies(m, k);
}
bool use_gemv(int64_t m, int64_t k) {
  return m >= 1 && m <= kGemvPathMaxM && gemv_smem_bytes((int)m, k) <= kGemvSmemLimit;
}
bool use_skinny(int64_t m) { return m > kGemvPathMaxM && m <= kSkinnyMaxM; }
// Small batches on mma.sync int8 (gemm_mma.cu), activations quantized once per call: from
// M = 12 where the activations fit in shared memory beside the rings (K <= 2048 at
// M = 16).  Measured on B200 in CUDA graphs (us per call, this path vs the dp4a kernel):
// qkv 2048->6144 M=12 12.3 vs 13.6, M=16 13.4 vs 16.4; o 2048->2048 M=12 7.7 vs 8.6,
// M=16 8.6 vs 10.4; gate_up 2048->12288 M=16 21.2 vs 23.1 (M=12 20.0 vs 19.1).  Below
// M = 12 the quantization launch (two dependency releases, ~2.3 us) outweighs it
// (qkv M=4 9.4 vs 6.8).  Q8LIN_SMALL_MMA=0 turns it off, =1 takes it from M = 2
// (comparisons).
constexpr int kMmaMinM = 12;
bool use_mma(int64_t m, int64_t k) {
  static const int mode = [] {
    const char* v = getenv("Q8LIN_SMALL_MMA");
    return v ? (v[0] == '0' ? 0 : (v[0] == '1' ? 2 : 1)) : 1;
  }();
  if (mode == 0) return false;
  return (mode == 2 || m >= kMmaMinM) && mma_applies(m, k);
}

// (Where the kernel choice depends on N -- M = 3, 4 at K <= 2048 -- both candidates need
// no workspace, so the size needs only M and K.)
size_t workspace_bytes(int64_t m, int64_t k) {
  if (m <= 0) return 0;
  if (use_mma(m, k)) return gemm_mma_workspace_bytes(m, k);
  if (use_mrow(m, k, INT64_MAX / k) || use_gemv(m, k)) return 0;
  if (use_skinny(m)) return gemm_skinny_workspace_bytes(m, k);
  return gemm_tc_workspace_bytes(m, k);
}

int validate_weight(const q8lin_weight* w) {
  if (!w) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "weight handle is null");
  if (!w->packed || w->n <= 0 || w->k <= 0) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "weight handle is not initialised");
  return Q8LIN_OK;
}

}  // namespace

DeviceGuard::DeviceGuard(int device) {
  ok_ = cudaGetDevice(&prev_) == cudaSuccess;
  if (ok_ && prev_ != device) ok_ = cudaSetDevice(device) == cudaSuccess;
  switched_ = ok_ && prev_ != device;
}
DeviceGuard::~DeviceGuard() {
  if (switched_) cudaSetDevice(prev_);
}

int check_device(int device) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= count)
    return fail(Q8LIN_ERR_DEVICE, "device " + std::to_string(device) + " out of range (" +
                                      std::to_string(count) + " visible)");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0)
    return fail(Q8LIN_ERR_DEVICE, "libq8lin is built for sm_100a only; device " + std::to_string(device) +
                                      " is sm_" + std::to_string(major) + std::to_string(minor));
  return Q8LIN_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

namespace {
std::mutex g_attr_mu;
}  // namespace

// configured[dev]: the largest dynamic shared memory already set for fn on that device.
// Read with an acquire load on every launch (no lock once configured); the first call per
// device and size sets the attribute under a lock and publishes it with a release store.
cudaError_t ensure_smem(const void* fn, int* configured, int device, size_t smem, bool max_carveout) {
  const int dev = (device >= 0 && device < 128) ? device : 0;
  if ((int)smem <= __atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) return cudaSuccess;
  std::lock_guard<std::mutex> lock(g_attr_mu);
  if ((int)smem <= __atomic_load_n(&configured[dev], __ATOMIC_RELAXED)) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess && max_carveout)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) __atomic_store_n(&configured[dev], (int)smem, __ATOMIC_RELEASE);
  return e;
}

}  // namespace q8lin

using namespace q8lin;

extern "C" {

int q8lin_version(void) { return Q8LIN_VERSION; }

const char* q8lin_last_error(void) { return g_last_error.c_str(); }

const char* q8lin_status_string(int status) {
  switch (status) {
    case Q8LIN_OK: return "Q8LIN_OK";
    case Q8LIN_ERR_INVALID_ARGUMENT: return "Q8LIN_ERR_INVALID_ARGUMENT";
    case Q8LIN_ERR_SHAPE: return "Q8LIN_ERR_SHAPE";
    case Q8LIN_ERR_ALIGNMENT: return "Q8LIN_ERR_ALIGNMENT";
    case Q8LIN_ERR_CUDA: return "Q8LIN_ERR_CUDA";
    case Q8LIN_ERR_NCCL: return "Q8LIN_ERR_NCCL";
    case Q8LIN_ERR_OUT_OF_MEMORY: return "Q8LIN_ERR_OUT_OF_MEMORY";
    case Q8LIN_ERR_DEVICE: return "Q8LIN_ERR_DEVICE";
    case Q8LIN_ERR_WORKSPACE: return "Q8LIN_ERR_WORKSPACE";
    case Q8LIN_ERR_FORMAT: return "Q8LIN_ERR_FORMAT";
    case Q8LIN_ERR_IO: return "Q8LIN_ERR_IO";
    case Q8LIN_ERR_NOT_FOUND: return "Q8LIN_ERR_NOT_FOUND";
    default: return "Q8LIN_ERR_UNKNOWN";
  }
}

int q8lin_weight_create(const void* gguf_blocks, int64_t n, int64_t k, int device,
                        q8lin_stream_t stream, q8lin_weight** out) {
  if (!out) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "out is null");
  *out = nullptr;
  if (!gguf_blocks) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "gguf_blocks is null");
  if (n <= 0 || k <= 0) return fail(Q8LIN_ERR_SHAPE, "weight shape must be positive, got (" + std::to_string(n) + ", " + std::to_string(k) + ")");
  if (k % kQK) return fail(Q8LIN_ERR_SHAPE, "in-features " + std::to_string(k) + " is not a multiple of the Q8_0 block size 32");
  if (n > (int64_t)1 << 30 || k > (int64_t)1 << 24)
    return fail(Q8LIN_ERR_SHAPE, "weight shape beyond supported limits (n <= 2^30, k <= 2^24)");
  int st = check_device(device);
  if (st != Q8LIN_OK) return st;
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  const int64_t nb = k / kQK;
  const size_t src_bytes = (size_t)(n * nb * kBlockBytes);
  cudaPointerAttributes attr = {};
  cudaError_t e = cudaPointerGetAttributes(&attr, gguf_blocks);
  if (e != cudaSuccess) {
    cudaGetLastError();
    attr.type = cudaMemoryTypeUnregistered;
  }
  const bool on_device = (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged);
  if (on_device && attr.type == cudaMemoryTypeDevice && attr.device != device)
    return fail(Q8LIN_ERR_DEVICE, "gguf_blocks live on device " + std::to_string(attr.device) + ", not " + std::to_string(device));
  if (on_device && (reinterpret_cast<uintptr_t>(gguf_blocks) & 1u))
    return fail(Q8LIN_ERR_ALIGNMENT, "device gguf_blocks must be 2-byte aligned");

  q8lin_weight* w = new q8lin_weight();
  w->device = device;
  w->n = n;
  w->k = k;
  w->row_stride = packed_row_stride(k);
  w->bytes = (size_t)(n * w->row_stride);
  e = cudaMalloc(&w->packed, w->bytes);
  if (e != cudaSuccess) {
    delete w;
    return cuda_fail(e, "cudaMalloc(weight)");
  }
  const uint8_t* src = static_cast<const uint8_t*>(gguf_blocks);
  uint8_t* staging = nullptr;
  if (!on_device) {
    e = cudaMalloc(&staging, src_bytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(staging, gguf_blocks, src_bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
      cudaFree(staging);
      cudaFree(w->packed);
      delete w;
      return cuda_fail(e, "upload of gguf_blocks");
    }
    src = staging;
  }
  e = launch_repack(src, w->packed, n, k, w->row_stride, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (staging) cudaFree(staging);
  if (e != cudaSuccess) {
    cudaFree(w->packed);
    delete w;
    return cuda_fail(e, "repack");
  }
  *out = w;
  return Q8LIN_OK;
}

int q8lin_weight_destroy(q8lin_weight* w) {
  if (!w) return Q8LIN_OK;
  DeviceGuard guard(w->device);
  cudaError_t e = w->packed ? cudaFree(w->packed) : cudaSuccess;
  delete w;
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree(weight)");
  return Q8LIN_OK;
}

int q8lin_weight_shape(const q8lin_weight* w, int64_t* n, int64_t* k, int* device) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (n) *n = w->n;
  if (k) *k = w->k;
  if (device) *device = w->device;
  return Q8LIN_OK;
}

int q8lin_weight_device_bytes(const q8lin_weight* w, size_t* bytes) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (!bytes) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "bytes is null");
  *bytes = w->bytes;
  return Q8LIN_OK;
}

int q8lin_weight_dequantize(const q8lin_weight* w, float* out, q8lin_stream_t stream) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (!out) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "out is null");
  if (!aligned16(out)) return fail(Q8LIN_ERR_ALIGNMENT, "out must be 16-byte aligned");
  DeviceGuard guard(w->device);
  cudaError_t e = launch_dequantize(w->packed, out, w->n, w->k, w->row_stride, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dequantize launch");
  return Q8LIN_OK;
}

int q8lin_weight_export_gguf(const q8lin_weight* w, void* out_blocks, q8lin_stream_t stream) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (!out_blocks) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "out_blocks is null");
  if (reinterpret_cast<uintptr_t>(out_blocks) & 1u) return fail(Q8LIN_ERR_ALIGNMENT, "out_blocks must be 2-byte aligned");
  DeviceGuard guard(w->device);
  cudaError_t e = launch_unpack(w->packed, static_cast<uint8_t*>(out_blocks), w->n, w->k, w->row_stride,
                                reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "export launch");
  return Q8LIN_OK;
}

size_t q8lin_workspace_size(const q8lin_weight* w, int64_t m) {
  if (!w || m <= 0) return 0;
  return workspace_bytes(m, w->k);
}

int q8lin_forward_ws(const q8lin_weight* w, const float* x, float* y, int64_t m, void* workspace,
                     size_t workspace_bytes_avail, q8lin_stream_t stream) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (m < 0) return fail(Q8LIN_ERR_SHAPE, "row count must be non-negative, got " + std::to_string(m));
  if (m == 0) return Q8LIN_OK;
  if (m > (int64_t)1 << 24) return fail(Q8LIN_ERR_SHAPE, "row count beyond supported limit 2^24");
  if (!x || !y) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "x and y must be non-null device pointers");
  if (!aligned16(x) || !aligned16(y)) return fail(Q8LIN_ERR_ALIGNMENT, "x and y must be 16-byte aligned");
  DeviceGuard guard(w->device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (use_mma(m, w->k)) {
    const size_t need = workspace_bytes(m, w->k);
    if (need > 0) {
      if (!workspace || workspace_bytes_avail < need)
        return fail(Q8LIN_ERR_WORKSPACE, "workspace of " + std::to_string(workspace_bytes_avail) +
                                             " bytes is smaller than the " + std::to_string(need) +
                                             " bytes needed for M=" + std::to_string(m));
      if (reinterpret_cast<uintptr_t>(workspace) % kAlign)
        return fail(Q8LIN_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
    }
    e = launch_gemm_mma(*w, x, workspace, y, m, s);
    if (e != cudaSuccess) return cuda_fail(e, "small-batch tensor-core launch");
    return Q8LIN_OK;
  }
  if (use_mrow(m, w->k, w->n)) {
    e = launch_gemv_mrow(*w, x, y, (int)m, s);
    if (e != cudaSuccess) return cuda_fail(e, "small-batch gemv launch");
    return Q8LIN_OK;
  }
  if (use_gemv(m, w->k)) {
    e = launch_gemv(*w, x, y, (int)m, s);
    if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
    return Q8LIN_OK;
  }
  const size_t need = workspace_bytes(m, w->k);
  if (!workspace || workspace_bytes_avail < need)
    return fail(Q8LIN_ERR_WORKSPACE, "workspace of " + std::to_string(workspace_bytes_avail) + " bytes is smaller than the " +
                                         std::to_string(need) + " bytes needed for M=" + std::to_string(m));
  if (reinterpret_cast<uintptr_t>(workspace) % kAlign)
    return fail(Q8LIN_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  if (use_skinny(m)) {
    e = launch_gemm_skinny(*w, x, workspace, y, m, s);
    if (e != cudaSuccess) return cuda_fail(e, "int8 tensor-core matmul launch");
    return Q8LIN_OK;
  }
  e = launch_gemm_tc(*w, x, workspace, y, m, s);
  if (e != cudaSuccess) return cuda_fail(e, "tensor-core gemm launch");
  return Q8LIN_OK;
}

int q8lin_forward(const q8lin_weight* w, const float* x, float* y, int64_t m, q8lin_stream_t stream) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (m <= 0 || m > (int64_t)1 << 24) return q8lin_forward_ws(w, x, y, m, nullptr, 0, stream);
  const size_t need = workspace_bytes(m, w->k);
  if (need == 0) return q8lin_forward_ws(w, x, y, m, nullptr, 0, stream);
  const q8lin_workspace* ws = w->ws;
  if (!ws || ws->bytes < need)
    return fail(Q8LIN_ERR_WORKSPACE, "M=" + std::to_string(m) + " needs a workspace of " + std::to_string(need) +
                                         " bytes; bind one with q8lin_weight_bind_workspace (q8lin_workspace_create "
                                         "sized for the largest M) or call q8lin_forward_ws");
  if (ws->device != w->device) return fail(Q8LIN_ERR_DEVICE, "the bound workspace lives on another device");
  return q8lin_forward_ws(w, x, y, m, ws->ptr, ws->bytes, stream);
}

size_t q8lin_workspace_bytes(int64_t max_m, int64_t max_k) {
  if (max_m <= 0 || max_k <= 0 || max_k % kQK || max_m > (int64_t)1 << 24 || max_k > (int64_t)1 << 24) return 0;
  // the int8 tensor-core path up to M = 32, the f16 path above it: each grows with M and K
  const size_t b = workspace_bytes(max_m < kSkinnyMaxM ? max_m : kSkinnyMaxM, max_k);
  const size_t t = workspace_bytes(max_m, max_k);
  return t > b ? t : b;
}

int q8lin_workspace_create(int device, int64_t max_m, int64_t max_k, q8lin_workspace** out) {
  if (!out) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "out is null");
  *out = nullptr;
  if (max_m <= 0 || max_k <= 0 || max_k % kQK || max_m > (int64_t)1 << 24 || max_k > (int64_t)1 << 24)
    return fail(Q8LIN_ERR_SHAPE, "a workspace needs 0 < max_m <= 2^24 and max_k a positive multiple of 32 <= 2^24");
  int st = check_device(device);
  if (st != Q8LIN_OK) return st;
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  q8lin_workspace* ws = new q8lin_workspace();
  ws->device = device;
  ws->bytes = q8lin_workspace_bytes(max_m, max_k);
  if (ws->bytes > 0) {
    cudaError_t e = cudaMalloc(&ws->ptr, ws->bytes);
    if (e != cudaSuccess) {
      delete ws;
      return cuda_fail(e, "cudaMalloc(workspace)");
    }
  }
  *out = ws;
  return Q8LIN_OK;
}

int q8lin_workspace_destroy(q8lin_workspace* ws) {
  if (!ws) return Q8LIN_OK;
  DeviceGuard guard(ws->device);
  cudaError_t e = ws->ptr ? cudaFree(ws->ptr) : cudaSuccess;
  delete ws;
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree(workspace)");
  return Q8LIN_OK;
}

int q8lin_workspace_capacity(const q8lin_workspace* ws, size_t* bytes) {
  if (!ws || !bytes) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "workspace and bytes must be non-null");
  *bytes = ws->bytes;
  return Q8LIN_OK;
}

int q8lin_weight_bind_workspace(q8lin_weight* w, q8lin_workspace* ws) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (ws && ws->device != w->device)
    return fail(Q8LIN_ERR_DEVICE, "workspace on device " + std::to_string(ws->device) + ", weight on device " +
                                      std::to_string(w->device));
  w->ws = ws;
  return Q8LIN_OK;
}

int q8lin_set_wait_limit_ns(uint64_t ns) {
  g_wait_limit_ns.store(ns, std::memory_order_relaxed);
  return Q8LIN_OK;
}

uint64_t q8lin_wait_limit_ns(void) { return wait_limit_ns(); }

int q8lin_dispatch_path(int64_t m, int64_t k, int64_t n) {
  if (m <= 0 || k <= 0 || n <= 0 || k % kQK) return -1;
  // the order of q8lin_forward_ws
  if (use_mma(m, k)) return Q8LIN_PATH_SMALL_BATCH_TC;
  if (use_mrow(m, k, n)) return Q8LIN_PATH_SMALL_BATCH;
  if (use_gemv(m, k)) return (m == 1 && stream_applies(k)) ? Q8LIN_PATH_STREAM_GEMV : Q8LIN_PATH_GEMV;
  if (use_skinny(m)) return Q8LIN_PATH_INT8_TC;
  return Q8LIN_PATH_F16_TC;
}

int q8lin_fault_status(int device, uint32_t* flags, int clear) {
  if (!flags) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "flags is null");
  int st = check_device(device);
  if (st != Q8LIN_OK) return st;
  DeviceGuard guard(device);
  unsigned int f = 0, g = 0, h = 0, a = 0, p = 0;
  cudaError_t e = read_tc_fault(&f, clear != 0);
  if (e == cudaSuccess) e = read_gemv_fault(&g, clear != 0);
  if (e == cudaSuccess) e = read_skinny_fault(&h, clear != 0);
  if (e == cudaSuccess) e = read_attention_fault(&a, clear != 0);
  unsigned int r = 0;
  if (e == cudaSuccess) e = read_step_fault(&p, clear != 0);
  if (e == cudaSuccess) e = read_mrow_fault(&r, clear != 0);
  if (e != cudaSuccess) return cuda_fail(e, "read fault word");
  *flags = f | g | h | a | p | r;
  return Q8LIN_OK;
}

int q8lin_quantize_rows(const float* x, int64_t m, int64_t k, int8_t* qs, uint16_t* d_f16,
                        q8lin_stream_t stream) {
  if (m < 0 || k <= 0 || k % kQK) return fail(Q8LIN_ERR_SHAPE, "quantize needs m >= 0 and k a positive multiple of 32");
  if (m == 0) return Q8LIN_OK;
  if (!x || !qs || !d_f16) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "x, qs and d_f16 must be non-null device pointers");
  if (!aligned16(x) || !aligned16(qs) || (reinterpret_cast<uintptr_t>(d_f16) & 1u))
    return fail(Q8LIN_ERR_ALIGNMENT, "x and qs must be 16-byte aligned, d_f16 2-byte aligned");
  cudaError_t e = launch_quantize_rows(x, m, k, qs, d_f16, nullptr, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
  return Q8LIN_OK;
}

int q8lin_swiglu(const float* gu, int64_t m, int64_t inter, float* h, q8lin_stream_t stream) {
  if (m < 0 || inter <= 0) return fail(Q8LIN_ERR_SHAPE, "swiglu needs m >= 0 and inter > 0");
  if (m == 0) return Q8LIN_OK;
  if (!gu || !h) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "gu and h must be non-null device pointers");
  if ((reinterpret_cast<uintptr_t>(gu) & 3u) || (reinterpret_cast<uintptr_t>(h) & 3u))
    return fail(Q8LIN_ERR_ALIGNMENT, "gu and h must be 4-byte aligned");
  cudaError_t e = launch_swiglu(gu, m, inter, h, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "swiglu launch");
  return Q8LIN_OK;
}

int q8lin_forward_fused(const q8lin_weight* w, const float* x, float* y, int64_t m, int32_t prologue,
                        const float* norm_weight, float eps, const float* residual, q8lin_stream_t stream) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (m != 1) return fail(Q8LIN_ERR_SHAPE, "the fused forms take one activation row (decode), got M=" + std::to_string(m));
  if (w->k > kFusedMaxK) return fail(Q8LIN_ERR_SHAPE, "the fused forms need K <= 8192");
  if (prologue < kPrologueNone || prologue > kPrologueSwiGLU) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "unknown prologue");
  if (!x || !y) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "x and y must be non-null device pointers");
  if (!aligned16(x) || !aligned16(y)) return fail(Q8LIN_ERR_ALIGNMENT, "x and y must be 16-byte aligned");
  if (prologue == kPrologueRmsNorm && (!norm_weight || !aligned16(norm_weight)))
    return fail(Q8LIN_ERR_INVALID_ARGUMENT, "the rms_norm prologue needs a 16-byte aligned norm weight");
  if (residual && (reinterpret_cast<uintptr_t>(residual) & 3u))
    return fail(Q8LIN_ERR_ALIGNMENT, "residual must be 4-byte aligned");
  DeviceGuard guard(w->device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  GemvFusion f;
  f.prologue = prologue;
  f.norm_w = norm_weight;
  f.eps = eps;
  f.residual = residual;
  cudaError_t e = launch_gemv_fused(*w, x, y, f, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fused gemv launch");
  return Q8LIN_OK;
}

int q8lin_peer_alloc(int device, size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "peer_alloc needs bytes > 0, ptr and handle");
  *ptr = nullptr;
  int st = check_device(device);
  if (st != Q8LIN_OK) return st;
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "peer buffer");
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return Q8LIN_OK;
}

int q8lin_peer_open(int device, const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "peer_open needs a handle and ptr");
  *ptr = nullptr;
  int st = check_device(device);
  if (st != Q8LIN_OK) return st;
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return Q8LIN_OK;
}

int q8lin_peer_close(int device, void* ptr) {
  if (!ptr) return Q8LIN_OK;
  DeviceGuard guard(device);
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return Q8LIN_OK;
}

int q8lin_peer_free(int device, void* ptr) {
  if (!ptr) return Q8LIN_OK;
  DeviceGuard guard(device);
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree(peer buffer)");
  return Q8LIN_OK;
}

size_t q8lin_allreduce_stage_bytes(int64_t n, int32_t world) {
  // [2 halves][world][n] tagged words: the epoch of the call next to the f32 value
  return (n > 0 && world > 0) ? (size_t)2 * (size_t)world * (size_t)n * sizeof(unsigned long long) : 0;
}

size_t q8lin_allreduce_flag_bytes(int32_t world) {
  return world > 0 ? (size_t)kAllreduceMaxCtas * (size_t)world * sizeof(uint32_t) : 0;
}

int q8lin_forward_allreduce(const q8lin_weight* w, const float* x, float* y, int64_t m, void* const* stage_ptrs,
                            void* const* flag_ptrs, int64_t stage_n, int32_t rank, int32_t world, uint32_t epoch,
                            const float* residual, q8lin_stream_t stream) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (world > 1 && w->n > stage_n)
    return fail(Q8LIN_ERR_SHAPE, "the staging buffers hold " + std::to_string(stage_n) + " rows, the weight has " +
                                     std::to_string(w->n));
  if (m != 1) return fail(Q8LIN_ERR_SHAPE, "the fused all-reduce takes one activation row (decode), got M=" + std::to_string(m));
  if (w->k > kFusedMaxK) return fail(Q8LIN_ERR_SHAPE, "the fused all-reduce needs K <= 8192");
  if (world < 1 || rank < 0 || rank >= world) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "rank must lie in [0, world)");
  if (epoch == 0) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "epoch counts calls from 1");
  if (!x || !y || (world > 1 && !stage_ptrs))
    return fail(Q8LIN_ERR_INVALID_ARGUMENT, "x, y and (world > 1) the peer pointer arrays must be non-null");
  if (!aligned16(x) || !aligned16(y)) return fail(Q8LIN_ERR_ALIGNMENT, "x and y must be 16-byte aligned");
  if (residual && (reinterpret_cast<uintptr_t>(residual) & 3u))
    return fail(Q8LIN_ERR_ALIGNMENT, "residual must be 4-byte aligned");
  if (sm_count(w->device) > kAllreduceMaxCtas) return fail(Q8LIN_ERR_DEVICE, "more SMs than the flag array covers");
  DeviceGuard guard(w->device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  GemvFusion f;
  f.residual = residual;
  f.ar_stage = reinterpret_cast<unsigned long long* const*>(stage_ptrs);
  f.ar_flags = reinterpret_cast<unsigned* const*>(flag_ptrs);
  f.ar_rank = rank;
  f.ar_world = world;
  f.ar_epoch = epoch;
  cudaError_t e = launch_gemv_fused(*w, x, y, f, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fused gemv + all-reduce launch");
  return Q8LIN_OK;
}

int q8lin_embed_rows(const q8lin_weight* w, const int32_t* tokens, int64_t n, float* out, q8lin_stream_t stream) {
  int st = validate_weight(w);
  if (st != Q8LIN_OK) return st;
  if (n < 0 || n > (1 << 20)) return fail(Q8LIN_ERR_SHAPE, "token count must be in [0, 2^20]");
  if (n == 0) return Q8LIN_OK;
  if (!tokens || !out) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "tokens and out must be non-null device pointers");
  DeviceGuard guard(w->device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  cudaError_t e = launch_embed_rows(*w, tokens, (int)n, out, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "embed launch");
  return Q8LIN_OK;
}

int q8lin_rmsnorm(const float* x, const float* weight, int64_t m, int64_t n, float eps, float* y,
                  q8lin_stream_t stream) {
  if (m < 0 || n <= 0 || m > (1 << 24)) return fail(Q8LIN_ERR_SHAPE, "rmsnorm needs 0 <= m and n > 0");
  if (m == 0) return Q8LIN_OK;
  if (!x || !weight || !y) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "x, weight and y must be non-null device pointers");
  cudaError_t e = launch_rmsnorm(x, weight, eps, m, n, y, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
  return Q8LIN_OK;
}

int q8lin_rope_kv(const float* qkv, const int32_t* pos, const float* cos_t, const float* sin_t, float* k_cache,
                  float* v_cache, int32_t hq, int32_t hkv, int32_t d, int32_t max_t, float* q_out,
                  q8lin_stream_t stream) {
  if (hq <= 0 || hkv <= 0 || hq % hkv || d <= 0 || d % 2 || d > 1024 || max_t <= 0)
    return fail(Q8LIN_ERR_SHAPE, "rope needs hq a positive multiple of hkv, an even d <= 1024 and max_t > 0");
  if (!qkv || !pos || !cos_t || !sin_t || !k_cache || !v_cache || !q_out)
    return fail(Q8LIN_ERR_INVALID_ARGUMENT, "rope pointers must be non-null device pointers");
  cudaError_t e = launch_rope_kv(qkv, pos, cos_t, sin_t, k_cache, v_cache, hq, hkv, d, max_t, q_out,
                                 reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope launch");
  return Q8LIN_OK;
}

size_t q8lin_attention_workspace_size(int32_t hq, int32_t max_t) {
  if (hq <= 0 || max_t <= 0) return 0;
  return attention_workspace_bytes(hq, max_t);
}

int q8lin_attention_decode(const float* q, const float* k_cache, const float* v_cache, const int32_t* pos,
                           int32_t hq, int32_t hkv, int32_t d, int32_t max_t, void* workspace, size_t workspace_bytes,
                           float* out, q8lin_stream_t stream) {
  if (d != 128) return fail(Q8LIN_ERR_SHAPE, "attention_decode supports head width 128");
  if (hq <= 0 || hkv <= 0 || hq % hkv || max_t <= 0)
    return fail(Q8LIN_ERR_SHAPE, "attention needs hq a positive multiple of hkv and max_t > 0");
  if (!q || !k_cache || !v_cache || !pos || !workspace || !out)
    return fail(Q8LIN_ERR_INVALID_ARGUMENT, "attention pointers must be non-null device pointers");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(Q8LIN_ERR_ALIGNMENT, "q and the caches must be 16-byte aligned");
  if (workspace_bytes < attention_workspace_bytes(hq, max_t))
    return fail(Q8LIN_ERR_WORKSPACE, "attention workspace too small (see q8lin_attention_workspace_size)");
  cudaError_t e = launch_attention_decode(q, k_cache, v_cache, pos, hq, hkv, max_t, workspace, out,
                                          reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return Q8LIN_OK;
}

int q8lin_rope_attention_decode(const float* qkv, const int32_t* pos, const float* cos_t, const float* sin_t,
                                float* k_cache, float* v_cache, int32_t hq, int32_t hkv, int32_t d, int32_t max_t,
                                float* out, q8lin_stream_t stream) {
  return q8lin_rope_attention_decode_ex(qkv, pos, cos_t, sin_t, k_cache, v_cache, hq, hkv, d, max_t, out, 0u, stream);
}

int q8lin_rope_attention_decode_ex(const float* qkv, const int32_t* pos, const float* cos_t, const float* sin_t,
                                   float* k_cache, float* v_cache, int32_t hq, int32_t hkv, int32_t d, int32_t max_t,
                                   float* out, uint32_t flags, q8lin_stream_t stream) {
  if (d != 128) return fail(Q8LIN_ERR_SHAPE, "rope_attention_decode supports head width 128");
  if (hq <= 0 || hkv <= 0 || hq % hkv || max_t <= 0 || hq > 65535)
    return fail(Q8LIN_ERR_SHAPE, "attention needs hq a positive multiple of hkv and max_t > 0");
  if (!qkv || !pos || !cos_t || !sin_t || !k_cache || !v_cache || !out)
    return fail(Q8LIN_ERR_INVALID_ARGUMENT, "rope_attention pointers must be non-null device pointers");
  if (!aligned16(k_cache) || !aligned16(v_cache)) return fail(Q8LIN_ERR_ALIGNMENT, "the caches must be 16-byte aligned");
  int device = 0;
  cudaGetDevice(&device);
  cudaError_t e = launch_rope_attention(qkv, pos, cos_t, sin_t, k_cache, v_cache, hq, hkv, max_t, out, device,
                                        reinterpret_cast<cudaStream_t>(stream), (flags & Q8LIN_ATTN_POS_READY) != 0);
  if (e != cudaSuccess) return cuda_fail(e, "rope_attention launch");
  return Q8LIN_OK;
}

// pos0 / t / batch / head counts of a prefill call (the context-limit check of
// transformer.rs:110-113 included); 0 when they are valid.
static int prefill_shape_fail(int32_t batch, int64_t t, int32_t pos0, int32_t hq, int32_t hkv, int32_t d,
                              int32_t max_t, int max_d) {
  if (hq <= 0 || hkv <= 0 || hq % hkv || d <= 0 || d % 2 || d > max_d || max_t <= 0 || hq + 2 * hkv > 65535)
    return fail(Q8LIN_ERR_SHAPE, "prefill needs hq a positive multiple of hkv, a supported head width and max_t > 0");
  if (batch <= 0 || batch > 65535 || t < 0) return fail(Q8LIN_ERR_SHAPE, "prefill needs 0 < batch <= 65535 and t >= 0");
  if ((int64_t)batch * t > INT32_MAX) return fail(Q8LIN_ERR_SHAPE, "prefill needs batch * t < 2^31");
  if (pos0 < 0 || (int64_t)pos0 + t > max_t) return fail(Q8LIN_ERR_SHAPE, "Transformer context limit exceeded");
  return Q8LIN_OK;
}

int q8lin_rope_kv_rows(const float* qkv, int32_t batch, int64_t t, int32_t pos0, const float* cos_t,
                       const float* sin_t, float* k_cache, float* v_cache, int32_t hq, int32_t hkv, int32_t d,
                       int32_t max_t, float* q_out, q8lin_stream_t stream) {
  if (int st = prefill_shape_fail(batch, t, pos0, hq, hkv, d, max_t, 1024)) return st;
  if (!qkv || !cos_t || !sin_t || !k_cache || !v_cache || !q_out)
    return fail(Q8LIN_ERR_INVALID_ARGUMENT, "rope pointers must be non-null device pointers");
  if (t == 0) return Q8LIN_OK;
  cudaError_t e = launch_rope_kv_rows(qkv, batch, (int)t, pos0, cos_t, sin_t, k_cache, v_cache, hq, hkv, d, max_t,
                                      q_out, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope_kv_rows launch");
  return Q8LIN_OK;
}

int q8lin_attention_prefill(const float* q, const float* k_cache, const float* v_cache, int32_t batch, int64_t t,
                            int32_t pos0, int32_t hq, int32_t hkv, int32_t d, int32_t max_t, float* out,
                            q8lin_stream_t stream) {
  if (d != 128) return fail(Q8LIN_ERR_SHAPE, "attention_prefill supports head width 128");
  if (int st = prefill_shape_fail(batch, t, pos0, hq, hkv, d, max_t, 128)) return st;
  if (!q || !k_cache || !v_cache || !out)
    return fail(Q8LIN_ERR_INVALID_ARGUMENT, "attention pointers must be non-null device pointers");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return fail(Q8LIN_ERR_ALIGNMENT, "q, the caches and out must be 16-byte aligned");
  if (t == 0) return Q8LIN_OK;
  int device = 0;
  cudaGetDevice(&device);
  cudaError_t e = launch_attention_prefill(q, k_cache, v_cache, batch, (int)t, pos0, hq, hkv, max_t, out, device,
                                           reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attention_prefill launch");
  return Q8LIN_OK;
}

int q8lin_add_rmsnorm(float* x, const float* y, const float* weight, int64_t m, int64_t n, float eps, float* h,
                      q8lin_stream_t stream) {
  if (m < 0 || n <= 0 || m > INT32_MAX) return fail(Q8LIN_ERR_SHAPE, "add_rmsnorm needs 0 <= m < 2^31 and n > 0");
  if (m == 0) return Q8LIN_OK;
  if (!x || !y || !weight || !h) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "add_rmsnorm pointers must be non-null");
  cudaError_t e = launch_add_rmsnorm(x, y, weight, eps, m, n, h, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "add_rmsnorm launch");
  return Q8LIN_OK;
}

int q8lin_add(float* x, const float* y, int64_t n, q8lin_stream_t stream) {
  if (n < 0) return fail(Q8LIN_ERR_SHAPE, "n must be non-negative");
  if (n == 0) return Q8LIN_OK;
  if (!x || !y) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "x and y must be non-null device pointers");
  cudaError_t e = launch_add(x, y, n, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "add launch");
  return Q8LIN_OK;
}

size_t q8lin_argmax_workspace_size(void) { return argmax_workspace_bytes(); }

int q8lin_argmax(const float* logits, int64_t n, void* workspace, size_t workspace_bytes, int32_t* token, int32_t* pos,
                 q8lin_stream_t stream) {
  if (n <= 0 || n > INT32_MAX) return fail(Q8LIN_ERR_SHAPE, "argmax needs 0 < n < 2^31");
  if (!logits || !workspace || !token) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "logits, workspace and token must be non-null");
  if (workspace_bytes < argmax_workspace_bytes())
    return fail(Q8LIN_ERR_WORKSPACE, "argmax workspace too small (see q8lin_argmax_workspace_size)");
  cudaError_t e = launch_argmax(logits, (int)n, workspace, token, pos, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
  return Q8LIN_OK;
}

}  // extern "C"

struct q8lin_step {
  int device = -1;
  int nops = 0;
  int grid = 0;
  q8lin::StepOp* ops = nullptr;  // device copy of the program
  unsigned* done = nullptr;      // [nops + 1] arrival counters
  float* attn_part = nullptr;    // [hq][splits][132]
  unsigned* head_cnt = nullptr;  // [hq]
  float* am_gv = nullptr;        // [grid]
  int* am_gi = nullptr;          // [grid]
  int32_t* pos = nullptr;
  int32_t* token = nullptr;
};

namespace q8lin {
namespace {

void step_free(q8lin_step* st) {
  if (!st) return;
  cudaFree(st->ops);
  cudaFree(st->done);
  cudaFree(st->attn_part);
  cudaFree(st->head_cnt);
  cudaFree(st->am_gv);
  cudaFree(st->am_gi);
  delete st;
}

int op_fail(int i, const std::string& msg) { return fail(Q8LIN_ERR_INVALID_ARGUMENT, "op " + std::to_string(i) + ": " + msg); }

}  // namespace
}  // namespace q8lin

extern "C" {

int q8lin_step_create(const q8lin_op* ops, int32_t nops, int32_t* pos, int32_t* token, int device, q8lin_step** out) {
  if (!out) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "out is null");
  *out = nullptr;
  if (!ops || nops <= 0 || nops > 65536) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "ops must hold 1..65536 operations");
  if (!pos || !token) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "pos and token must be device pointers");
  int st = check_device(device);
  if (st != Q8LIN_OK) return st;
  std::vector<StepOp> dev_ops((size_t)nops);
  int max_hq = 0;
  for (int i = 0; i < nops; ++i) {
    const q8lin_op& o = ops[i];
    StepOp& d = dev_ops[(size_t)i];
    d = StepOp();
    d.kind = o.kind;
    d.prologue = o.prologue;
    if (o.kind == Q8LIN_OP_GEMV || o.kind == Q8LIN_OP_EMBED) {
      const q8lin_weight* w = o.weight;
      if (!w || !w->packed) return op_fail(i, "needs a weight");
      if (w->device != device) return fail(Q8LIN_ERR_DEVICE, "op " + std::to_string(i) + ": weight on another device");
      d.n = (int)w->n;
      d.k = (int)w->k;
      d.S = w->row_stride;
      d.W = w->packed;
      d.y = o.y;
      if (!o.y || !aligned16(o.y)) return op_fail(i, "y must be a 16-byte aligned device pointer");
    }
    switch (o.kind) {
      case Q8LIN_OP_GEMV: {
        if (d.k > kStepMaxK) return fail(Q8LIN_ERR_SHAPE, "op " + std::to_string(i) + ": K beyond 8192");
        d.rpc = step_rows_per_chunk(d.k);
        if (d.rpc < 1) return fail(Q8LIN_ERR_SHAPE, "op " + std::to_string(i) + ": row too wide for the ring");
        if (o.prologue < Q8LIN_PROLOGUE_NONE || o.prologue > Q8LIN_PROLOGUE_SWIGLU) return op_fail(i, "unknown prologue");
        if (o.epilogue != Q8LIN_EPILOGUE_NONE && o.epilogue != Q8LIN_EPILOGUE_SWIGLU) return op_fail(i, "unknown epilogue");
        if (!o.x || !aligned16(o.x)) return op_fail(i, "x must be a 16-byte aligned device pointer");
        if (o.prologue == Q8LIN_PROLOGUE_RMSNORM && (!o.norm_weight || !aligned16(o.norm_weight)))
          return op_fail(i, "rms_norm needs a 16-byte aligned norm weight");
        if (o.residual && !aligned16(o.residual)) return op_fail(i, "residual must be 16-byte aligned");
        if (o.epilogue == Q8LIN_EPILOGUE_SWIGLU) {
          if (d.n % 2 || d.rpc < 2 || d.k > 2048 || o.residual || o.argmax)
            return fail(Q8LIN_ERR_SHAPE, "op " + std::to_string(i) +
                                             ": the SwiGLU epilogue takes [gate | up] rows, K <= 2048, no residual "
                                             "or argmax");
        }
        d.x = o.x;
        d.residual = o.residual;
        d.norm_w = o.norm_weight;
        d.eps = o.eps;
        d.argmax = o.argmax ? 1 : 0;
        d.epilogue = o.epilogue;
        break;
      }
      case Q8LIN_OP_ATTENTION: {
        if (o.head_dim != 128) return fail(Q8LIN_ERR_SHAPE, "op " + std::to_string(i) + ": head width must be 128");
        if (o.hq <= 0 || o.hkv <= 0 || o.hq % o.hkv || o.max_t <= 0 || o.hq > 4096)
          return fail(Q8LIN_ERR_SHAPE, "op " + std::to_string(i) + ": needs hq a multiple of hkv");
        if (!o.x || !o.y || !o.k_cache || !o.v_cache || !o.cos_t || !o.sin_t) return op_fail(i, "attention pointers are null");
        if (!aligned16(o.x) || !aligned16(o.y) || !aligned16(o.k_cache) || !aligned16(o.v_cache))
          return fail(Q8LIN_ERR_ALIGNMENT, "op " + std::to_string(i) + ": qkv, output and caches must be 16-byte aligned");
        d.x = o.x;
        d.y = o.y;
        d.hq = o.hq;
        d.hkv = o.hkv;
        d.max_t = o.max_t;
        d.scale = (float)(1.0 / std::sqrt(128.0));
        d.kc = o.k_cache;
        d.vc = o.v_cache;
        d.cos_t = o.cos_t;
        d.sin_t = o.sin_t;
        if (o.hq > max_hq) max_hq = o.hq;
        break;
      }
      case Q8LIN_OP_EMBED:
        break;
      case Q8LIN_OP_ARGMAX:
        if (i == 0 || ops[i - 1].kind != Q8LIN_OP_GEMV || !ops[i - 1].argmax)
          return op_fail(i, "an argmax op follows a GEMV with argmax set");
        d.n = (int)ops[i - 1].weight->n;
        break;
      default:
        return op_fail(i, "unknown kind");
    }
  }
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  q8lin_step* s = new q8lin_step();
  s->device = device;
  s->nops = nops;
  s->pos = pos;
  s->token = token;
  cudaError_t e = step_max_grid(device, &s->grid);
  if (e == cudaSuccess && s->grid <= 0) {
    delete s;
    return fail(Q8LIN_ERR_DEVICE, "the decode-step kernel does not fit on an SM");
  }
  if (e == cudaSuccess) e = cudaMalloc(&s->ops, sizeof(StepOp) * (size_t)nops);
  if (e == cudaSuccess) e = cudaMalloc(&s->done, sizeof(unsigned) * (size_t)(nops + 1));
  const size_t hq_alloc = (size_t)(max_hq > 0 ? max_hq : 1);
  if (e == cudaSuccess) e = cudaMalloc(&s->attn_part, sizeof(float) * hq_alloc * step_splits() * 132);
  if (e == cudaSuccess) e = cudaMalloc(&s->head_cnt, sizeof(unsigned) * hq_alloc);
  if (e == cudaSuccess) e = cudaMemset(s->head_cnt, 0, sizeof(unsigned) * hq_alloc);
  if (e == cudaSuccess)
    for (StepOp& d : dev_ops)
      if (d.kind == kStepOpAttention) {
        d.attn_part = s->attn_part;
        d.head_cnt = s->head_cnt;
      }
  if (e == cudaSuccess) e = cudaMalloc(&s->am_gv, sizeof(float) * (size_t)s->grid);
  if (e == cudaSuccess) e = cudaMalloc(&s->am_gi, sizeof(int) * (size_t)s->grid);
  if (e == cudaSuccess)
    e = cudaMemcpy(s->ops, dev_ops.data(), sizeof(StepOp) * (size_t)nops, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(s->done, 0, sizeof(unsigned) * (size_t)(nops + 1));
  if (e != cudaSuccess) {
    step_free(s);
    return cuda_fail(e, "decode-step setup");
  }
  *out = s;
  return Q8LIN_OK;
}

int q8lin_step_run(q8lin_step* s, q8lin_stream_t stream) {
  if (!s) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "step is null");
  DeviceGuard guard(s->device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  cudaError_t e = launch_decode_step(s->ops, s->nops, s->pos, s->token, s->done, s->am_gv, s->am_gi, s->grid,
                                     s->device, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode-step launch");
  return Q8LIN_OK;
}

int q8lin_step_destroy(q8lin_step* s) {
  if (!s) return Q8LIN_OK;
  DeviceGuard guard(s->device);
  step_free(s);
  return Q8LIN_OK;
}

}  // extern "C"
