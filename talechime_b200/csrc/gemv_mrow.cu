// Small-batch streaming GEMV: y[M][N] = Q8_0(x)[M][K] . W^T for 2 <= M <= 16, on the CUDA
// cores (dp4a), with the M = 1 kernel's weight stream.
//
// At these M the per-block scale of Q8_0 makes tensor-core tiles spend their time in
// the per-block rescale handshakes; here the integer block dots run as dp4a, which at
// M <= 16 keep pace with HBM (~2.7 us of dp4a work for the qkv weight at M = 16).
//   * one CTA per SM: 15 consumer warps + 1 producer warp; the producer streams the CTA's
//     contiguous rows through a shared-memory ring of 1-D bulk copies (as in the M = 1
//     kernel), issuing the first ring before the dependency wait;
//   * consumers quantize the M activation rows into shared memory (candle's rules, one
//     thread per block), then each warp takes two weight rows at a time against every activation
//     row: lane l owns blocks l and l + 32 of a 2048-value segment, loads the two rows'
//     blocks once (per-lane half order: conflict-free) and, per activation row m, the
//     activation blocks, accumulating ((f32(isum) * dw) * dx) per block (each product
//     rounded, as candle's scalar vec_dot);
//   * the MR sums of a row are reduced across the warp by a transposing reduction
//     (each level halves the values a lane holds), MR - 1 + 5 - log2(MR) shuffles per row
//     instead of 5 MR;
//   * a row of K > 2048 takes ceil(K / 2048) warps whose partials meet in shared memory and
//     are added in segment order.
// MR is M rounded up to a power of two; rows m >= M are skipped.  Every wait is bounded
// (fault word bit 1).
#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

constexpr int kMrConsumerWarps = 15;  // 16 consumer + 1 producer warps would cap registers at 96
constexpr int kMrThreads = (kMrConsumerWarps + 1) * 32;
constexpr int kMrRingBytes = 96 * 1024;
constexpr int kMrMaxSlots = 16;
constexpr int kMrMaxRpc = 4;
constexpr int kMrMaxSegs = 4;
constexpr int kMrSegBlocks = 64;  // blocks of a 2048-value segment
constexpr uint32_t kMrWaitLimit = 1u << 24;
constexpr size_t kMrSmemLimit = 227 * 1024;

__device__ unsigned int g_mrow_fault;

__host__ __device__ constexpr int64_t rnd16(int64_t v) { return (v + 15) / 16 * 16; }

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool mr_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMrWaitLimit; ++i) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok) : "r"(su32(bar)), "r"(parity) : "memory");
    if (ok) return true;
  }
  atomicOr(&g_mrow_fault, 2u);
  return false;
}

// Sum over the warp of v[m], m < MR, leaving in every lane the total of row mr_index(lane).
template <int MR>
__device__ __forceinline__ float transpose_reduce(float (&v)[MR], int lane) {
#pragma unroll
  for (int L = 0; L < 5; ++L) {
    const int o = 16 >> L;
    const int c = MR >> L;  // values held before this level
    if (c > 1) {
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < MR / 2; ++i) {
        if (i < c / 2) {
          const float send = up ? v[i] : v[i + c / 2];
          const float keep = up ? v[i + c / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(kFull, send, o);
        }
      }
    } else {
      v[0] += __shfl_xor_sync(kFull, v[0], o);
    }
  }
  return v[0];
}

template <int MR>
__device__ __forceinline__ int mr_index(int lane) {
  int m = 0;
#pragma unroll
  for (int L = 0; L < 5; ++L) {
    const int c = MR >> L;
    if (c > 1 && (lane & (16 >> L))) m += c / 2;
  }
  return m;
}

// Block `blk` of a weight row (two 16-byte halves in the lane's half order) and its scale.
struct WBlock {
  int4 h0, h1;
  float d;
};

__device__ __forceinline__ WBlock load_wblock(const uint8_t* row, int K, int blk, int hoff) {
  WBlock w;
  w.h0 = *reinterpret_cast<const int4*>(row + (size_t)blk * 32 + hoff);
  w.h1 = *reinterpret_cast<const int4*>(row + (size_t)blk * 32 + (16 - hoff));
  w.d = __half2float(reinterpret_cast<const __half*>(row + K)[blk]);
  return w;
}

__device__ __forceinline__ float wterm(const WBlock& w, const int4& x0, const int4& x1, float dxs) {
  const int isum = dot16(w.h1, x1, dot16(w.h0, x0, 0));
  return __fmul_rn(__fmul_rn(__int2float_rn(isum), w.d), dxs);
}

template <int MR>
__global__ void __launch_bounds__(kMrThreads, 1)
gemv_q8_0_mrow_kernel(const uint8_t* __restrict__ W, int64_t S, int N, int K, int M, const float* __restrict__ x,
                      float* __restrict__ y, int rpc, int slots) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = K >> 5;
  const int nseg = (nb + kMrSegBlocks - 1) / kMrSegBlocks;
  const int ngroups = kMrConsumerWarps / nseg;
  const int r0 = (int)(((int64_t)N * blockIdx.x) / gridDim.x);
  const int r1 = (int)(((int64_t)N * (blockIdx.x + 1)) / gridDim.x);
  const int nrows = r1 - r0;
  const int nchunks = (nrows + rpc - 1) / rpc;
  const size_t chunk_bytes = (size_t)rpc * S;
  // [ring | qx: MR x K int8 | dx: MR x nb f32 | part: [slot][row][seg][MR] f32 |
  //  cnt: [slot][row] int | full, empty mbarriers]
  uint8_t* ring = smem;
  int8_t* qx = reinterpret_cast<int8_t*>(smem + kMrRingBytes);
  float* dx = reinterpret_cast<float*>(smem + kMrRingBytes + rnd16((int64_t)MR * K));
  float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(dx) + rnd16((int64_t)MR * nb * 4));
  int* cnt = reinterpret_cast<int*>(part + kMrMaxSlots * kMrMaxRpc * kMrMaxSegs * MR);
  uint64_t* full = reinterpret_cast<uint64_t*>(cnt + kMrMaxSlots * kMrMaxRpc);
  uint64_t* empty = full + kMrMaxSlots;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < slots; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&full[i])), "r"(1) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&empty[i])), "r"(rpc * nseg) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = threadIdx.x; i < kMrMaxSlots * kMrMaxRpc; i += kMrThreads) cnt[i] = 0;
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kMrConsumerWarps) {
    // ---------------- producer (weights are constant: no dependency wait) ----------------
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < nchunks; ++j) {
        const int slot = j % slots;
        if (j >= slots && !mr_wait(&empty[slot], (uint32_t)((j / slots - 1) & 1))) break;
        const int row = r0 + j * rpc;
        const uint32_t bytes = (uint32_t)(min(rpc, r1 - row) * S);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[slot])), "r"(bytes)
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(su32(ring + (size_t)slot * chunk_bytes)), "l"(W + (size_t)row * S), "r"(bytes),
                     "r"(su32(&full[slot]))
                     : "memory");
        issued = j + 1;
      }
      for (int j = (issued > slots ? issued - slots : 0); j < issued; ++j)
        mr_wait(&full[j % slots], (uint32_t)((j / slots) & 1));
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();
  {
    // quantize the M activation rows, one thread per 32-value block (rows >= M stay
    // unread: the row loop skips them)
    const int blocks = M * nb;
    for (int i = threadIdx.x; i < blocks; i += kMrConsumerWarps * 32) {
      const int m = i / nb, b = i - m * nb;
      const float4* src = reinterpret_cast<const float4*>(x + (size_t)m * K + (size_t)b * kQK);
      float4 v[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t);
      int q[8];
      __half dh;
      quantize_block_regs(v, q, dh);
      int4* dst = reinterpret_cast<int4*>(qx + (size_t)m * K + (size_t)b * kQK);
      dst[0] = make_int4(q[0], q[1], q[2], q[3]);
      dst[1] = make_int4(q[4], q[5], q[6], q[7]);
      dx[m * nb + b] = __half2float(dh);
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kMrConsumerWarps * 32) : "memory");

  const int seg = warp % nseg, grp = warp / nseg;
  const int hoff = half_order(lane) * 16;
  const int b0 = seg * kMrSegBlocks + lane, b1 = b0 + 32;
  const bool v0 = b0 < nb, v1 = b1 < nb;
  const int my_m = mr_index<MR>(lane);
  struct Pos {
    int ri, slot;
    uint32_t parity;
  };
  auto advance = [&](Pos p, int rows) {
    p.ri += rows;
    while (p.ri >= rpc) {
      p.ri -= rpc;
      if (++p.slot == slots) {
        p.slot = 0;
        p.parity ^= 1u;
      }
    }
    return p;
  };
  // finish row `rr` (ring slot / row in chunk) with this lane's total `v` of row my_m
  auto finish = [&](int rr, int slot, int ri, float v) {
    const bool writer = !(lane & 1) && my_m < M;  // lanes 2j and 2j + 1 hold the same row
    if (nseg == 1) {
      if (writer) y[(size_t)my_m * N + r0 + rr] = v;
    } else {
      float* pr = part + ((slot * kMrMaxRpc + ri) * kMrMaxSegs + seg) * MR;
      if (!(lane & 1)) pr[my_m] = v;
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(&cnt[slot * kMrMaxRpc + ri], 1) == nseg - 1;
        if (last) cnt[slot * kMrMaxRpc + ri] = 0;
        __threadfence_block();
      }
      last = __shfl_sync(kFull, last, 0);
      if (last && writer) {
        const float* base = part + (slot * kMrMaxRpc + ri) * kMrMaxSegs * MR;
        float sum = base[my_m];
        for (int q = 1; q < nseg; ++q) sum += base[q * MR + my_m];
        y[(size_t)my_m * N + r0 + rr] = sum;
      }
    }
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&empty[slot])) : "memory");
  };
  Pos pa = advance(Pos{0, 0, 0u}, grp);
  for (int rr = grp < ngroups ? grp : nrows; rr < nrows; rr += 2 * ngroups, pa = advance(pa, 2 * ngroups)) {
    const int rb = rr + ngroups;
    const bool has_b = rb < nrows;
    if (!mr_wait(&full[pa.slot], pa.parity)) break;
    const Pos pb = has_b ? advance(pa, ngroups) : pa;
    if (has_b && !mr_wait(&full[pb.slot], pb.parity)) break;
    const uint8_t* wa = ring + (size_t)pa.slot * chunk_bytes + (size_t)pa.ri * S;
    const uint8_t* wb = ring + (size_t)pb.slot * chunk_bytes + (size_t)pb.ri * S;
    WBlock a0, a1, c0, c1;
    if (v0) {
      a0 = load_wblock(wa, K, b0, hoff);
      c0 = load_wblock(wb, K, b0, hoff);
    }
    if (v1) {
      a1 = load_wblock(wa, K, b1, hoff);
      c1 = load_wblock(wb, K, b1, hoff);
    }
    float sa[MR], sb[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      sa[m] = 0.0f;
      sb[m] = 0.0f;
      if (m < M) {
        const int8_t* xr = qx + (size_t)m * K;
        const float* dr = dx + m * nb;
        if (v0) {
          const int4 x0 = *reinterpret_cast<const int4*>(xr + (size_t)b0 * 32 + hoff);
          const int4 x1 = *reinterpret_cast<const int4*>(xr + (size_t)b0 * 32 + (16 - hoff));
          const float d = dr[b0];
          sa[m] = wterm(a0, x0, x1, d);
          sb[m] = wterm(c0, x0, x1, d);
        }
        if (v1) {
          const int4 x0 = *reinterpret_cast<const int4*>(xr + (size_t)b1 * 32 + hoff);
          const int4 x1 = *reinterpret_cast<const int4*>(xr + (size_t)b1 * 32 + (16 - hoff));
          const float d = dr[b1];
          sa[m] = __fadd_rn(sa[m], wterm(a1, x0, x1, d));
          sb[m] = __fadd_rn(sb[m], wterm(c1, x0, x1, d));
        }
      }
    }
    const float ta = transpose_reduce<MR>(sa, lane);
    const float tb = transpose_reduce<MR>(sb, lane);
    finish(rr, pa.slot, pa.ri, ta);
    if (has_b) finish(rb, pb.slot, pb.ri, tb);
  }
}

// Rows per chunk and ring slots for this K (as the M = 1 kernel: at least 8 chunks).
void mrow_plan(int64_t S, int* rpc, int* slots) {
  *rpc = kMrMaxRpc;
  while (*rpc > 1 && kMrRingBytes / (*rpc * S) < 8) *rpc /= 2;
  const int64_t s = kMrRingBytes / (*rpc * S);
  *slots = s < 2 ? 0 : (int)(s > kMrMaxSlots ? kMrMaxSlots : s);
}

template <int MR>
size_t mrow_smem(int64_t k) {
  return (size_t)(kMrRingBytes + rnd16((int64_t)MR * k) + rnd16((int64_t)MR * (k / kQK) * 4) +
                  (int64_t)kMrMaxSlots * kMrMaxRpc * kMrMaxSegs * MR * 4 + kMrMaxSlots * kMrMaxRpc * 4 +
                  2 * kMrMaxSlots * 8);
}

template <int MR>
cudaError_t launch_mrow_t(const q8lin_weight& w, const float* x, float* y, int m, cudaStream_t s) {
  const int K = (int)w.k, N = (int)w.n;
  int rpc, slots;
  mrow_plan(w.row_stride, &rpc, &slots);
  const size_t smem = mrow_smem<MR>(K);
  static int configured_smem[128] = {0};
  const int dev = (w.device >= 0 && w.device < 128) ? w.device : 0;
  if ((int)smem > configured_smem[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_q8_0_mrow_kernel<MR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    configured_smem[dev] = (int)smem;
  }
  int grid = sm_count(w.device);
  if (grid > N) grid = N;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMrThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_q8_0_mrow_kernel<MR>, (const uint8_t*)w.packed, w.row_stride, N, K, m, x, y,
                            rpc, slots);
}

int mrow_width(int m) { return m <= 2 ? 2 : m <= 4 ? 4 : m <= 8 ? 8 : 16; }

}  // namespace

bool mrow_applies(int64_t m, int64_t k) {
  if (m < 2 || m > kMrowMaxM || k > (int64_t)kMrMaxSegs * kMrSegBlocks * kQK) return false;
  int rpc, slots;
  mrow_plan(packed_row_stride(k), &rpc, &slots);
  if (slots == 0) return false;
  size_t smem = 0;
  switch (mrow_width((int)m)) {
    case 2: smem = mrow_smem<2>(k); break;
    case 4: smem = mrow_smem<4>(k); break;
    case 8: smem = mrow_smem<8>(k); break;
    default: smem = mrow_smem<16>(k); break;
  }
  return smem <= kMrSmemLimit;
}

cudaError_t launch_gemv_mrow(const q8lin_weight& w, const float* x, float* y, int m, cudaStream_t s) {
  switch (mrow_width(m)) {
    case 2: return launch_mrow_t<2>(w, x, y, m, s);
    case 4: return launch_mrow_t<4>(w, x, y, m, s);
    case 8: return launch_mrow_t<8>(w, x, y, m, s);
    default: return launch_mrow_t<16>(w, x, y, m, s);
  }
}

cudaError_t read_mrow_fault(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_mrow_fault, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_mrow_fault, &z, sizeof(z));
  }
  return e;
}

}  // namespace q8lin
