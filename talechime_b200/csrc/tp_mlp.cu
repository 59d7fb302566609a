// Tensor-parallel Q8_0 SwiGLU MLP behind the C ABI (q8lin_mlp_tp_*, include/q8lin.h).
//
// The VoxCPM MLP is down(silu(gate(h)) * up(h)) with three Q8_0 QMatMuls
// (crates/voxcpm/src/transformer.rs:147-150).  Over P ranks of one node (one exchange):
//   * gate and up split by output rows: rank r keeps rows [I*r/P, I*(r+1)/P) of each as one
//     fused weight [gate rows; up rows], so one linear gives both halves;
//   * SwiGLU is local;
//   * down splits by Q8_0 block columns [nb*r/P, nb*(r+1)/P) of every row; I/P must be a
//     multiple of 32, so the rank's slice of h quantizes to exactly the blocks of the
//     unsplit row;
//   * the partial outputs are summed over the ranks: ncclAllReduce on the caller's
//     communicator, or -- for one activation row with Q8LIN_TP_FUSED_DECODE once the peers
//     are connected -- inside the down projection's kernel over NVLink peer memory (the
//     kernel of q8lin_forward_allreduce, with the SwiGLU folded into its activation
//     quantization).
// All scratch (gate|up output, SwiGLU output, partial sum, the batched workspace, the
// staging and flag buffers) is allocated at create for up to max_m rows: forward
// allocates nothing.  The only collective the library runs is forward's all-reduce; the
// staging buffers' IPC handles travel over the caller's own transport.
//
// NCCL is resolved at run time from the libnccl.so.2 the process has already loaded --
// the one that made the caller's communicator -- or loaded here if none is; only the C
// entry points and enum values of NCCL's public header are used.
#include <dlfcn.h>
#include <string.h>

#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "q8lin.h"

struct q8lin_mlp_tp {
  int device = -1, rank = 0, world = 1;
  int64_t hidden = 0, inter = 0, il = 0, max_m = 0;
  void* comm = nullptr;
  q8lin_weight* gate_up = nullptr;
  q8lin_weight* down = nullptr;
  q8lin_workspace* ws = nullptr;
  float* gu = nullptr;    // [max_m][2 il]
  float* h = nullptr;     // [max_m][il]
  float* part = nullptr;  // [max_m][hidden] (world > 1)
  // fused decode: staging and flag buffers (own at index rank), device pointer arrays
  bool fused = false;
  float* stage = nullptr;
  unsigned* flags = nullptr;
  cudaIpcMemHandle_t handles[2];  // of stage and flags, for the peers
  std::vector<void*> opened;
  void** peer_ptrs = nullptr;  // device: [world] stage pointers, then [world] flag pointers
  uint32_t epoch = 0;
};
static_assert(sizeof(cudaIpcMemHandle_t) == Q8LIN_IPC_HANDLE_BYTES, "IPC handle size");

namespace q8lin {
namespace {

constexpr int kNcclFloat32 = 7, kNcclSum = 0;

struct Nccl {
  int (*all_reduce)(const void*, void*, size_t, int, int, void*, cudaStream_t) = nullptr;
  int (*comm_count)(void*, int*) = nullptr;
  int (*comm_user_rank)(void*, int*) = nullptr;
  const char* (*error_string)(int) = nullptr;
  bool ok = false;
};

const Nccl& nccl() {
  static const Nccl lib = [] {
    Nccl n;
    void* h = dlopen("libnccl.so.2", RTLD_NOLOAD | RTLD_LAZY);
    if (!h) h = dlopen("libnccl.so.2", RTLD_LAZY | RTLD_LOCAL);
    if (!h) return n;
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
    n.comm_count = reinterpret_cast<decltype(n.comm_count)>(dlsym(h, "ncclCommCount"));
    n.comm_user_rank = reinterpret_cast<decltype(n.comm_user_rank)>(dlsym(h, "ncclCommUserRank"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.all_reduce && n.comm_count && n.comm_user_rank && n.error_string;
    return n;
  }();
  return lib;
}

int nccl_fail(int r, const char* what) {
  const Nccl& n = nccl();
  return fail(Q8LIN_ERR_NCCL, std::string(what) + ": " + (n.error_string ? n.error_string(r) : "NCCL error") +
                                  " (" + std::to_string(r) + ")");
}

// Shard plan of the partition above.
int shard_plan(int64_t hidden, int64_t inter, int32_t rank, int32_t world, int64_t* row0, int64_t* rows,
               int64_t* blk0, int64_t* blks) {
  if (hidden <= 0 || inter <= 0 || hidden % kQK || inter % kQK)
    return fail(Q8LIN_ERR_SHAPE, "hidden and intermediate sizes must be positive multiples of 32");
  if (world < 1 || rank < 0 || rank >= world) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "rank must lie in [0, world)");
  if (inter % ((int64_t)kQK * world))
    return fail(Q8LIN_ERR_SHAPE, "intermediate " + std::to_string(inter) + " does not split into " +
                                     std::to_string(world) + " shards of whole Q8_0 blocks");
  const int64_t il = inter / world;
  *row0 = il * rank;
  *rows = il;
  *blk0 = (il / kQK) * rank;
  *blks = il / kQK;
  return Q8LIN_OK;
}

void release(q8lin_mlp_tp* t) {
  if (!t) return;
  DeviceGuard guard(t->device);
  for (void* p : t->opened) cudaIpcCloseMemHandle(p);
  t->opened.clear();
  cudaFree(t->peer_ptrs);
  cudaFree(t->stage);
  cudaFree(t->flags);
  cudaFree(t->gu);
  cudaFree(t->h);
  cudaFree(t->part);
  q8lin_weight_destroy(t->gate_up);
  q8lin_weight_destroy(t->down);
  q8lin_workspace_destroy(t->ws);
  delete t;
}

// The staging and flag buffers of the fused decode path (zeroed) and their IPC handles.
int alloc_fused(q8lin_mlp_tp* t, cudaStream_t s) {
  const size_t stage_bytes = q8lin_allreduce_stage_bytes(t->hidden, t->world);
  const size_t flag_bytes = q8lin_allreduce_flag_bytes(t->world);
  cudaError_t e = cudaMalloc(&t->stage, stage_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&t->flags, flag_bytes);
  if (e == cudaSuccess) e = cudaMemsetAsync(t->stage, 0, stage_bytes, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(t->flags, 0, flag_bytes, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&t->handles[0], t->stage);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&t->handles[1], t->flags);
  if (e != cudaSuccess) return cuda_fail(e, "fused all-reduce buffers");
  return Q8LIN_OK;
}

}  // namespace
}  // namespace q8lin

using namespace q8lin;

extern "C" {

int q8lin_mlp_tp_shard(int64_t hidden, int64_t inter, int32_t rank, int32_t world, int64_t* row0, int64_t* rows,
                       int64_t* blk0, int64_t* blks) {
  if (!row0 || !rows || !blk0 || !blks) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "output pointers must be non-null");
  return shard_plan(hidden, inter, rank, world, row0, rows, blk0, blks);
}

int q8lin_nccl_available(void) { return nccl().ok ? 1 : 0; }

int q8lin_mlp_tp_create(const void* gate_blocks, const void* up_blocks, const void* down_blocks, int64_t hidden,
                        int64_t inter, int32_t rank, int32_t world, void* nccl_comm, int device, int64_t max_m,
                        uint32_t flags, q8lin_stream_t stream, q8lin_mlp_tp** out) {
  if (!out) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "out is null");
  *out = nullptr;
  if (!gate_blocks || !up_blocks || !down_blocks) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "weight blocks must be non-null");
  int64_t row0, rows, blk0, blks;
  int st = shard_plan(hidden, inter, rank, world, &row0, &rows, &blk0, &blks);
  if (st != Q8LIN_OK) return st;
  if (max_m <= 0 || max_m > (int64_t)1 << 20) return fail(Q8LIN_ERR_SHAPE, "max_m must lie in [1, 2^20]");
  if (flags & ~Q8LIN_TP_FUSED_DECODE) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "unknown flags");
  if (world > 1) {
    if (!nccl_comm) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "world > 1 needs an NCCL communicator");
    const Nccl& n = nccl();
    if (!n.ok) return fail(Q8LIN_ERR_NCCL, "libnccl.so.2 could not be loaded");
    int count = 0, me = -1, r = n.comm_count(nccl_comm, &count);
    if (r == 0) r = n.comm_user_rank(nccl_comm, &me);
    if (r != 0) return nccl_fail(r, "communicator query");
    if (count != world || me != rank)
      return fail(Q8LIN_ERR_INVALID_ARGUMENT, "communicator has " + std::to_string(count) + " ranks, this one is " +
                                                  std::to_string(me) + "; the call says rank " + std::to_string(rank) +
                                                  " of " + std::to_string(world));
  }
  st = check_device(device);
  if (st != Q8LIN_OK) return st;
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  q8lin_mlp_tp* t = new q8lin_mlp_tp();
  t->device = device;
  t->rank = rank;
  t->world = world;
  t->hidden = hidden;
  t->inter = inter;
  t->il = rows;
  t->max_m = max_m;
  t->comm = nccl_comm;
  auto bail = [&](int status) {
    release(t);
    return status;
  };
  // this rank's shards, gathered on the device: [gate rows; up rows] and down's block columns
  const size_t row_bytes = (size_t)(hidden / kQK) * kBlockBytes;
  const size_t dn_src_pitch = (size_t)(inter / kQK) * kBlockBytes;
  const size_t dn_pitch = (size_t)blks * kBlockBytes;
  const size_t gu_bytes = 2 * (size_t)rows * row_bytes, dn_bytes = (size_t)hidden * dn_pitch;
  uint8_t* stg = nullptr;
  cudaError_t e = cudaMalloc(&stg, gu_bytes > dn_bytes ? gu_bytes : dn_bytes);
  if (e != cudaSuccess) return bail(cuda_fail(e, "shard staging buffer"));
  const uint8_t* gate = static_cast<const uint8_t*>(gate_blocks);
  const uint8_t* up = static_cast<const uint8_t*>(up_blocks);
  const uint8_t* dn = static_cast<const uint8_t*>(down_blocks);
  e = cudaMemcpyAsync(stg, gate + (size_t)row0 * row_bytes, (size_t)rows * row_bytes, cudaMemcpyDefault, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(stg + (size_t)rows * row_bytes, up + (size_t)row0 * row_bytes, (size_t)rows * row_bytes,
                        cudaMemcpyDefault, s);
  if (e != cudaSuccess) {
    cudaFree(stg);
    return bail(cuda_fail(e, "gate/up shard copy"));
  }
  st = q8lin_weight_create(stg, 2 * rows, hidden, device, stream, &t->gate_up);  // synchronizes s
  if (st == Q8LIN_OK) {
    e = cudaMemcpy2DAsync(stg, dn_pitch, dn + (size_t)blk0 * kBlockBytes, dn_src_pitch, dn_pitch, (size_t)hidden,
                          cudaMemcpyDefault, s);
    if (e != cudaSuccess) st = cuda_fail(e, "down shard copy");
  }
  if (st == Q8LIN_OK) st = q8lin_weight_create(stg, hidden, rows, device, stream, &t->down);
  cudaFree(stg);
  if (st != Q8LIN_OK) return bail(st);
  // scratch for max_m rows
  const int64_t wk = hidden > rows ? hidden : rows;
  if (q8lin_workspace_bytes(max_m, wk) > 0) {
    st = q8lin_workspace_create(device, max_m, wk, &t->ws);
    if (st == Q8LIN_OK) st = q8lin_weight_bind_workspace(t->gate_up, t->ws);
    if (st == Q8LIN_OK) st = q8lin_weight_bind_workspace(t->down, t->ws);
    if (st != Q8LIN_OK) return bail(st);
  }
  e = cudaMalloc(&t->gu, (size_t)max_m * 2 * rows * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&t->h, (size_t)max_m * rows * sizeof(float));
  if (e == cudaSuccess && world > 1) e = cudaMalloc(&t->part, (size_t)max_m * hidden * sizeof(float));
  if (e != cudaSuccess) return bail(cuda_fail(e, "MLP scratch"));
  if ((flags & Q8LIN_TP_FUSED_DECODE) && world > 1) {
    if (hidden > kFusedMaxK || rows > kFusedMaxK || !stream_applies(rows) || !stream_applies(hidden))
      return bail(fail(Q8LIN_ERR_SHAPE, "the fused decode path needs hidden and intermediate / world <= 8192"));
    if (sm_count(device) > kAllreduceMaxCtas) return bail(fail(Q8LIN_ERR_DEVICE, "more SMs than the flag array covers"));
    st = alloc_fused(t, s);
    if (st != Q8LIN_OK) return bail(st);
  }
  *out = t;
  return Q8LIN_OK;
}

int q8lin_mlp_tp_peer_handle(const q8lin_mlp_tp* t, void* out) {
  if (!t || !out) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "MLP handle and out must be non-null");
  if (!t->stage) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "the MLP was created without Q8LIN_TP_FUSED_DECODE");
  memcpy(out, t->handles, sizeof(t->handles));
  return Q8LIN_OK;
}

int q8lin_mlp_tp_connect_peers(q8lin_mlp_tp* t, const void* all) {
  if (!t || !all) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "MLP handle and handles must be non-null");
  if (!t->stage) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "the MLP was created without Q8LIN_TP_FUSED_DECODE");
  if (t->fused || !t->opened.empty()) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "the peers are connected already");
  DeviceGuard guard(t->device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  const unsigned char* h = static_cast<const unsigned char*>(all);
  constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
  if (memcmp(h + (size_t)t->rank * 2 * kH, t->handles, 2 * kH) != 0)
    return fail(Q8LIN_ERR_INVALID_ARGUMENT, "entry `rank` of the handles is not this rank's (q8lin_mlp_tp_peer_handle)");
  std::vector<void*> ptrs(2 * (size_t)t->world);
  for (int p = 0; p < t->world; ++p) {
    if (p == t->rank) {
      ptrs[p] = t->stage;
      ptrs[t->world + p] = t->flags;
      continue;
    }
    for (int which = 0; which < 2; ++which) {
      cudaIpcMemHandle_t ph;
      memcpy(&ph, h + ((size_t)p * 2 + which) * kH, kH);
      void* q = nullptr;
      cudaError_t e = cudaIpcOpenMemHandle(&q, ph, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        for (void* o : t->opened) cudaIpcCloseMemHandle(o);
        t->opened.clear();
        return cuda_fail(e, "cudaIpcOpenMemHandle (the ranks must share one node)");
      }
      t->opened.push_back(q);
      ptrs[which * t->world + p] = q;
    }
  }
  cudaError_t e = t->peer_ptrs ? cudaSuccess : cudaMalloc(&t->peer_ptrs, ptrs.size() * sizeof(void*));
  if (e == cudaSuccess) e = cudaMemcpy(t->peer_ptrs, ptrs.data(), ptrs.size() * sizeof(void*), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "peer pointer arrays");
  t->fused = true;
  return Q8LIN_OK;
}

int q8lin_mlp_tp_forward(q8lin_mlp_tp* t, const float* x, float* y, int64_t m, q8lin_stream_t stream) {
  if (!t) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "MLP handle is null");
  if (m < 0 || m > t->max_m)
    return fail(Q8LIN_ERR_SHAPE, "M=" + std::to_string(m) + " outside [0, max_m=" + std::to_string(t->max_m) + "]");
  if (m == 0) return Q8LIN_OK;
  if (!x || !y) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "x and y must be non-null device pointers");
  if (!aligned16(x) || !aligned16(y)) return fail(Q8LIN_ERR_ALIGNMENT, "x and y must be 16-byte aligned");
  DeviceGuard guard(t->device);
  if (!guard.ok()) return fail(Q8LIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* dst = t->world > 1 ? t->part : y;
  const bool decode = m == 1 && t->il <= kFusedMaxK && stream_applies(t->il);
  if (decode) {
    // gate|up GEMV, then the down GEMV with silu(gate) * up folded into its activation
    // quantization (and, fused, the cross-GPU sum in its tail)
    int st = q8lin_forward_ws(t->gate_up, x, t->gu, 1, nullptr, 0, stream);
    if (st != Q8LIN_OK) return st;
    GemvFusion f;
    f.prologue = kPrologueSwiGLU;
    if (t->fused) {
      const uint32_t epoch = t->epoch + 1;
      f.ar_stage = reinterpret_cast<unsigned long long* const*>(t->peer_ptrs);
      f.ar_flags = reinterpret_cast<unsigned* const*>(t->peer_ptrs + t->world);
      f.ar_rank = t->rank;
      f.ar_world = t->world;
      f.ar_epoch = epoch;
      cudaError_t e = launch_gemv_fused(*t->down, t->gu, y, f, s);
      if (e != cudaSuccess) return cuda_fail(e, "fused down projection + all-reduce launch");
      t->epoch = epoch;  // counted only once the launch is in the stream
      return Q8LIN_OK;
    }
    cudaError_t e = launch_gemv_fused(*t->down, t->gu, dst, f, s);
    if (e != cudaSuccess) return cuda_fail(e, "down projection launch");
  } else {
    int st = q8lin_forward(t->gate_up, x, t->gu, m, stream);
    if (st != Q8LIN_OK) return st;
    cudaError_t e = launch_swiglu(t->gu, m, t->il, t->h, s);
    if (e != cudaSuccess) return cuda_fail(e, "swiglu launch");
    st = q8lin_forward(t->down, t->h, dst, m, stream);
    if (st != Q8LIN_OK) return st;
  }
  if (t->world > 1) {
    const int r = nccl().all_reduce(t->part, y, (size_t)m * t->hidden, kNcclFloat32, kNcclSum, t->comm, s);
    if (r != 0) return nccl_fail(r, "ncclAllReduce");
  }
  return Q8LIN_OK;
}

int q8lin_mlp_tp_close_peers(q8lin_mlp_tp* t) {
  if (!t) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "MLP handle is null");
  if (t->opened.empty() && !t->fused) return Q8LIN_OK;
  DeviceGuard guard(t->device);
  cudaError_t e = cudaDeviceSynchronize();  // no kernel of this rank still writes to a peer
  for (void* p : t->opened) cudaIpcCloseMemHandle(p);
  t->opened.clear();
  t->fused = false;
  if (e != cudaSuccess) return cuda_fail(e, "synchronize before unmapping the peers");
  return Q8LIN_OK;
}

int q8lin_mlp_tp_destroy(q8lin_mlp_tp* t) {
  if (!t) return Q8LIN_OK;
  {
    DeviceGuard guard(t->device);
    cudaDeviceSynchronize();
  }
  release(t);
  return Q8LIN_OK;
}

int q8lin_mlp_tp_info(const q8lin_mlp_tp* t, int64_t* inter_local, int32_t* fused) {
  if (!t) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "MLP handle is null");
  if (inter_local) *inter_local = t->il;
  if (fused) *fused = t->fused ? 1 : 0;
  return Q8LIN_OK;
}

}  // extern "C"
