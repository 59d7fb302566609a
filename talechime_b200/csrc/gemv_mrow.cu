// Small-batch streaming GEMV: y[M][N] = Q8_0(x)[M][K] . W^T for 2 <= M <= 16, on the CUDA
// cores (dp4a), with the M = 1 kernel's weight stream.
//
// At these M the per-block scale of Q8_0 makes tensor-core tiles spend their time in
// the per-block rescale handshakes; here the integer block dots run as dp4a, which at
// M <= 16 keep pace with HBM (~2.7 us of dp4a work for the qkv weight at M = 16).
//   * one CTA per SM owning a contiguous row range; its 16 warps each stream their own
//     rows through a private shared-memory ring with 16-byte cp.async copies (slot j of
//     the CTA belongs to warp j % nw), issuing the first slots before the dependency
//     wait -- as the M = 1 kernel, and for the same reasons: a thread's TMA / bulk copies
//     complete one after another on B200, and a warp that consumes its own slots in
//     order needs no mbarrier parity;
//   * the CTA quantizes the M activation rows into shared memory (candle's rules, 8
//     lanes per block), then each warp takes two weight rows at a time against every
//     activation row: lane l owns blocks l and l + 32 of each 2048-value segment, loads the
//     two rows' blocks once (per-lane half order: conflict-free) and, per activation row
//     m, the activation blocks, accumulating ((f32(isum) * dw) * dx) per block (each
//     product rounded, as candle's scalar vec_dot) over all segments of the row;
//   * the MR sums of a row are reduced across the warp by a transposing reduction (each
//     level halves the values a lane holds), MR - 1 + 5 - log2(MR) shuffles per row
//     instead of 5 MR.
// MR is M rounded up to a power of two; rows m >= M are skipped.  The kernel has no spin
// wait (a warp waits for its own copies with cp.async.wait_group).
#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

constexpr int kMrWarps = 16;
constexpr int kMrThreads = kMrWarps * 32;
constexpr int kMrSlotTarget = 4352;  // two rows of K = 2048
constexpr int kMrMaxRps = 16;
constexpr int kMrDepth = 2;
constexpr int kMrSegBlocks = 64;  // blocks of a 2048-value segment
constexpr int kMrMaxK = 8192;
constexpr size_t kMrSmemLimit = 227 * 1024;

__device__ unsigned int g_mrow_fault;  // (no spin waits left: kept for the fault word's bit 1)

__host__ __device__ constexpr int64_t rnd16(int64_t v) { return (v + 15) / 16 * 16; }

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

struct MrowGeo {
  int rps = 0, nw = 0, slot_bytes = 0;
};

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
                      float* __restrict__ y, const MrowGeo geo) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = K >> 5;
  const int nseg = (nb + kMrSegBlocks - 1) / kMrSegBlocks;
  const int r0 = (int)(((int64_t)N * blockIdx.x) / gridDim.x);
  const int r1 = (int)(((int64_t)N * (blockIdx.x + 1)) / gridDim.x);
  const int nrows = r1 - r0;
  const int rps = geo.rps, nw = geo.nw;
  const int nslots = (nrows + rps - 1) / rps;
  // [rings: nw x kMrDepth slots | qx: MR x K int8 | dx: MR x nb f32]
  int8_t* qx = reinterpret_cast<int8_t*>(smem + (size_t)nw * kMrDepth * geo.slot_bytes);
  float* dx = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(qx) + rnd16((int64_t)MR * K));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + (size_t)warp * kMrDepth * geo.slot_bytes;

  pdl_launch_dependents();
  const uint64_t l2pol = l2_evict_first_policy();
  auto issue = [&](int t) {
    const int j = warp + t * nw;
    if (j < nslots) {
      const int row = j * rps;
      const int units = (min(rps, nrows - row) * (int)S) >> 4;
      const uint8_t* src = W + (size_t)(r0 + row) * S;
      const uint32_t dst = su32(ring + (size_t)(t % kMrDepth) * geo.slot_bytes);
      for (int u = lane; u < units; u += 32) cp_async16_stream(dst + 16u * u, src + 16 * (size_t)u, l2pol);
    }
    cp_async_commit();
  };
  if (warp < nw)  // weights are constant: their first slots before the dependency wait
    for (int t = 0; t < kMrDepth; ++t) issue(t);

  pdl_wait();
  {
    // quantize the M activation rows (rows >= M stay unread: the row loop skips them):
    // 8 lanes per 32-value block, 4 values each (x is [M][K] row-major, so quad i of the
    // flattened rows is values 4i .. 4i + 3 and 8 consecutive quads form one block); the
    // loads of up to four passes of the CTA are issued before any is quantized
    constexpr int kPass = 4;
    const int nquads = M * (K >> 2);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int base = 0; base < nquads; base += kPass * kMrThreads) {  // uniform over the CTA
      float4 v[kPass];
#pragma unroll
      for (int g = 0; g < kPass; ++g) {
        const int i = base + g * kMrThreads + threadIdx.x;
        v[g] = i < nquads ? __ldg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int g = 0; g < kPass; ++g) {
        if (base + g * kMrThreads < nquads) {  // uniform: every lane takes part in the shuffles
          const int i = base + g * kMrThreads + threadIdx.x;
          __half dh;
          const int q = quantize_octet(v[g], dh);
          if (i < nquads) {
            reinterpret_cast<int*>(qx)[i] = q;  // qx rows are K apart: quad i lands at 4i
            if ((i & 7) == 0) dx[i >> 3] = __half2float(dh);  // block i / 8 = m * nb + b
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp >= nw) return;

  const int hoff = half_order(lane) * 16;
  const int my_m = mr_index<MR>(lane);
  const bool writer = !(lane & 1) && my_m < M;  // lanes 2j and 2j + 1 hold the same row
  for (int t = 0, j = warp; j < nslots; ++t, j += nw) {
    cp_async_wait(kMrDepth - 1);  // this thread's copies of slot t have landed
    __syncwarp();                 // ... and every lane's
    const uint8_t* sl = ring + (size_t)(t % kMrDepth) * geo.slot_bytes;
    const int row0 = j * rps;
    const int rows = min(rps, nrows - row0);
    for (int i = 0; i < rows; i += 2) {
      const bool has_b = i + 1 < rows;
      const uint8_t* wa = sl + (size_t)i * S;
      const uint8_t* wb = has_b ? wa + S : wa;
      float sa[MR], sb[MR];
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        sa[m] = 0.0f;
        sb[m] = 0.0f;
      }
      for (int sg = 0; sg < nseg; ++sg) {
        const int b0 = sg * kMrSegBlocks + lane, b1 = b0 + 32;
        const bool v0 = b0 < nb, v1 = b1 < nb;
        WBlock a0, a1, c0, c1;
        if (v0) {
          a0 = load_wblock(wa, K, b0, hoff);
          c0 = load_wblock(wb, K, b0, hoff);
        }
        if (v1) {
          a1 = load_wblock(wa, K, b1, hoff);
          c1 = load_wblock(wb, K, b1, hoff);
        }
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          if (m < M) {
            const int8_t* xr = qx + (size_t)m * K;
            const float* dr = dx + m * nb;
            if (v0) {
              const int4 x0 = *reinterpret_cast<const int4*>(xr + (size_t)b0 * 32 + hoff);
              const int4 x1 = *reinterpret_cast<const int4*>(xr + (size_t)b0 * 32 + (16 - hoff));
              const float d = dr[b0];
              sa[m] = __fadd_rn(sa[m], wterm(a0, x0, x1, d));
              sb[m] = __fadd_rn(sb[m], wterm(c0, x0, x1, d));
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
      }
      const float ta = transpose_reduce<MR>(sa, lane);
      const float tb = transpose_reduce<MR>(sb, lane);
      if (writer) {
        y[(size_t)my_m * N + r0 + row0 + i] = ta;
        if (has_b) y[(size_t)my_m * N + r0 + row0 + i + 1] = tb;
      }
    }
    __syncwarp();  // every lane is done with the slot before it is refilled
    issue(t + kMrDepth);
  }
  cp_async_wait(0);
}

// Slot geometry for this K and MR: slots of about two K = 2048 rows, depth 2, as many of
// the 16 warps as the shared memory beside the quantized activations allows.
MrowGeo mrow_geometry(int64_t S, int64_t k, int mr) {
  MrowGeo g;
  if (k > kMrMaxK) return g;
  int64_t rps = kMrSlotTarget / S;
  rps = rps < 1 ? 1 : (rps > kMrMaxRps ? kMrMaxRps : rps);
  const int64_t fixed = rnd16((int64_t)mr * k) + rnd16((int64_t)mr * (k / kQK) * 4) + 1024;
  if ((int64_t)kMrSmemLimit <= fixed) return g;
  int64_t nw = ((int64_t)kMrSmemLimit - fixed) / (kMrDepth * rps * S);
  if (nw > kMrWarps) nw = kMrWarps;
  if (nw < 1) return g;
  g.rps = (int)rps;
  g.nw = (int)nw;
  g.slot_bytes = (int)(rps * S);
  return g;
}

size_t mrow_smem(const MrowGeo& g, int64_t k, int mr) {
  return (size_t)g.nw * kMrDepth * g.slot_bytes + rnd16((int64_t)mr * k) + rnd16((int64_t)mr * (k / kQK) * 4);
}

template <int MR>
cudaError_t launch_mrow_t(const q8lin_weight& w, const float* x, float* y, int m, cudaStream_t s) {
  const int K = (int)w.k, N = (int)w.n;
  const MrowGeo g = mrow_geometry(w.row_stride, K, MR);
  if (g.nw == 0) return cudaErrorInvalidValue;
  const size_t smem = mrow_smem(g, K, MR);
  static int configured_smem[128] = {0};
  cudaError_t e = ensure_smem((const void*)gemv_q8_0_mrow_kernel<MR>, configured_smem, w.device, smem, false);
  if (e != cudaSuccess) return e;
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
  return cudaLaunchKernelEx(&cfg, gemv_q8_0_mrow_kernel<MR>, (const uint8_t*)w.packed, w.row_stride, N, K, m, x, y, g);
}

int mrow_width(int m) { return m <= 2 ? 2 : m <= 4 ? 4 : m <= 8 ? 8 : 16; }

}  // namespace

bool mrow_applies(int64_t m, int64_t k) {
  if (m < 2 || m > kMrowMaxM || k > kMrMaxK) return false;
  return mrow_geometry(packed_row_stride(k), k, mrow_width((int)m)).nw > 0;
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
