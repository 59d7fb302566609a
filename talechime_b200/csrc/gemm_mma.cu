// Small batches of the Q8_0 linear (2 <= M <= 16) on mma.sync int8 tensor cores.
//
// y[M][N] = x[M][K] . W[N][K]^T with candle's Q8_0 arithmetic (the CPU QMatMul::forward
// of candle-core 0.11.0 as used by Linear::forward, crates/voxcpm/src/weights.rs:209-229):
// every activation row is quantized to Q8_0 (quantize_rows_i8t, once per call, into the
// workspace), and each output is the sum over blocks of ((f32(I_b) * dw_b) * dx_b), I_b
// the exact int32 dot product of block b.
//
// Why mma.sync here: one m16n8k32 int8 MMA is exactly one Q8_0 block of 16 weight rows
// against 8 activation rows, and its int32 result lands in registers, where the per-block
// rescale costs four CUDA-core operations per output.  The batch is small, so the work is
// bounded by streaming the weights and by per-launch latency, not by MMA throughput; the
// rescale is what costs, and every warp shares it (the tcgen05 int8 kernel reads every
// block's result back from tensor memory in 4 epilogue warps).
//
// Layout: units of 16 weight rows x 8 blocks (256 values): per row 256 bytes of int8 and
// the 8 f16 scales, 272 bytes, so the 16 rows of a unit (4352 bytes) sit 272 bytes apart
// and ldmatrix reads them without bank conflicts.  Each of the 8 warps streams its
// own units through a private ring of 2 or 3 slots with 16-byte cp.async (L2
// evict-first); the first slots are issued before the dependency wait, so they overlap the
// quantization launch.  A CTA owns a contiguous range of 16-row tiles:
//   - more tiles than ring warps: warp w takes tiles w, w + nw, ..., all K each, and
//     writes y itself;
//   - otherwise the CTA's units (tile-major) are cut into nw contiguous ranges of at most
//     one tile's worth; a range touches at most two tiles, whose partial sums stay in
//     registers and are added across warps in chunk order through shared memory (the ring,
//     free by then).  Sums are deterministic; their association differs from candle's
//     sequential loop only in where the chunks meet (f32 summation tolerance).
#include <cstdint>
#include <cstdlib>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace q8lin {
namespace {

constexpr int kMmWarps = 8;
constexpr int kMmThreads = kMmWarps * 32;
constexpr int kUnitBlocks = 8;                          // Q8_0 blocks per unit
constexpr int kUnitRowBytes = kUnitBlocks * 32 + 16;    // 272: int8 of 8 blocks + their f16 scales
constexpr int kUnitBytes = 16 * kUnitRowBytes;          // 4352
constexpr int kMmRingWarps = kMmWarps;
// Ring slots per warp: 2 (8 x 2 x 4352 = 69632 bytes, two CTAs per SM where the activations
// fit beside them) or 3 (104448 bytes, one CTA per SM; the deeper ring keeps a unit's
// refill off the critical path).
__host__ __device__ constexpr int ring_bytes(int depth) { return kMmRingWarps * depth * kUnitBytes; }

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__host__ __device__ constexpr int64_t round_up16(int64_t v) { return (v + 15) / 16 * 16; }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// d = A (16 x 32 int8, row) . B (32 x 8 int8, col), int32 (exact)
__device__ __forceinline__ void mma_s8(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int (&d)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

struct MmaArgs {
  const uint8_t* W;  // packed rows, stride S
  int64_t S;
  int N, K, M, Mp;
  const int8_t* qx;  // [M][K] int8 activations (null: the kernel quantizes x itself)
  const float* dxT;  // [K/32][Mp] their scales
  const float* x;    // [M][K] f32 activations (when qx is null)
  float* y;          // [M][N]
};

// Adds unit (16 rows x blocks b0 .. b0 + nblk - 1) from its ring slot to acc:
// acc[nt][0], [1] = weight row g x activation rows nt*8 + 2q, + 1; acc[nt][2], [3] = row
// g + 8 (g = lane / 4, q = lane % 4), per block ((f32(I) * dw) * dx) in block order.
// xs: the int8 activations in shared memory, rows xstride bytes apart; dxs: their scales
// [K/32][Mp].
template <int NT>
__device__ __forceinline__ void unit_mma(const MmaArgs& a, uint32_t slot, uint32_t xs, uint32_t xstride, uint32_t dxs,
                                         int b0, int nblk, float (&acc)[NT][4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  // ldmatrix row of this lane: matrices (rows 0-7 | 8-15) x (bytes 0-15 | 16-31 of a block)
  const uint32_t arow =
      slot + (uint32_t)(((lane & 7) + ((lane >> 3) & 1) * 8) * kUnitRowBytes + ((lane >> 4) & 1) * 16);
  uint32_t sg[4], sg8[4];  // the 8 f16 scales of rows g and g + 8
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(sg[0]), "=r"(sg[1]), "=r"(sg[2]), "=r"(sg[3])
               : "r"(slot + (uint32_t)(g * kUnitRowBytes + 256)));
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(sg8[0]), "=r"(sg8[1]), "=r"(sg8[2]), "=r"(sg8[3])
               : "r"(slot + (uint32_t)((g + 8) * kUnitRowBytes + 256)));
  uint32_t xr[NT];  // B-fragment rows (activation rows >= M read row M - 1; discarded)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) xr[nt] = xs + (uint32_t)min(nt * 8 + g, a.M - 1) * xstride + 4u * q;
  // a group of blocks: every fragment load first (they issue back to back), then the MMAs
  // and rescales; blocks past nblk repeat the unit's last block and are not accumulated
  constexpr int kGroup = NT == 1 ? kUnitBlocks : kUnitBlocks / 2;
#pragma unroll
  for (int h = 0; h < kUnitBlocks; h += kGroup) {
    uint32_t af[kGroup][4], bx[kGroup][NT][2];
    float dxv[kGroup][NT][2];
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
      const int jj = min(h + j, nblk - 1);
      const uint32_t b = (uint32_t)(b0 + jj);
      ldsm_x4(arow + 32u * (uint32_t)jj, af[j][0], af[j][1], af[j][2], af[j][3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(bx[j][nt][0]) : "r"(xr[nt] + b * 32u));
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(bx[j][nt][1]) : "r"(xr[nt] + b * 32u + 16u));
        asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];"
                     : "=f"(dxv[j][nt][0]), "=f"(dxv[j][nt][1])
                     : "r"(dxs + 4u * (b * (uint32_t)a.Mp + (uint32_t)(nt * 8 + 2 * q))));
      }
    }
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
      const int jj = h + j;
      if (jj < nblk) {
        const uint32_t hw = sg[jj >> 1], hw8 = sg8[jj >> 1];
        const float dw = __half2float(__ushort_as_half((unsigned short)((jj & 1) ? (hw >> 16) : (hw & 0xffffu))));
        const float dw8 = __half2float(__ushort_as_half((unsigned short)((jj & 1) ? (hw8 >> 16) : (hw8 & 0xffffu))));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          int d[4];
          mma_s8(af[j], bx[j][nt][0], bx[j][nt][1], d);
          acc[nt][0] = __fadd_rn(acc[nt][0], __fmul_rn(__fmul_rn(__int2float_rn(d[0]), dw), dxv[j][nt][0]));
          acc[nt][1] = __fadd_rn(acc[nt][1], __fmul_rn(__fmul_rn(__int2float_rn(d[1]), dw), dxv[j][nt][1]));
          acc[nt][2] = __fadd_rn(acc[nt][2], __fmul_rn(__fmul_rn(__int2float_rn(d[2]), dw8), dxv[j][nt][0]));
          acc[nt][3] = __fadd_rn(acc[nt][3], __fmul_rn(__fmul_rn(__int2float_rn(d[3]), dw8), dxv[j][nt][1]));
        }
      }
    }
  }
}

template <int NT, int DEPTH>
__global__ void __launch_bounds__(kMmThreads, 2) gemm_q8_0_mma_kernel(const MmaArgs a) {
  constexpr int kMmDepth = DEPTH;
  constexpr int kMmRingBytes = ring_bytes(DEPTH);
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = a.K >> 5;
  const int nkc = (nb + kUnitBlocks - 1) / kUnitBlocks;  // units per tile
  const int T = (a.N + 15) >> 4;
  const int t0 = (int)((int64_t)T * blockIdx.x / gridDim.x);
  const int ntc = (int)((int64_t)T * (blockIdx.x + 1) / gridDim.x) - t0;  // this CTA's tiles
  const int nw = kMmRingWarps;
  const bool whole = ntc > nw;
  const int U = ntc * nkc;
  const int L = whole ? 1 : (U + nw - 1) / nw;  // units per warp range (<= nkc when !whole)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int u_begin = 0, my_units = 0;
  if (warp < nw) {
    if (whole) {
      my_units = ((ntc - warp + nw - 1) / nw) * nkc;  // tiles warp, warp + nw, ...
    } else {
      u_begin = warp * L;
      my_units = max(0, min(U, u_begin + L) - u_begin);
    }
  }
  auto unit_of = [&](int t, int& lt, int& ch) {  // this warp's unit t -> CTA tile, chunk
    if (whole) {
      const int i = t / nkc;
      lt = warp + i * nw;
      ch = t - i * nkc;
    } else {
      const int u = u_begin + t;
      lt = u / nkc;
      ch = u - lt * nkc;
    }
  };
  const uint32_t ring_s = su32(smem) + (uint32_t)(warp * kMmDepth * kUnitBytes);

  pdl_launch_dependents();
  const uint64_t pol = l2_evict_first_policy();
  auto issue = [&](int t) {  // unit t into ring position t % kMmDepth; one copy group
    if (t < my_units) {
      int lt, ch;
      unit_of(t, lt, ch);
      const int b0 = ch * kUnitBlocks, nblk = min(kUnitBlocks, nb - b0);
      const uint32_t dst = ring_s + (uint32_t)((t % kMmDepth) * kUnitBytes);
      const int row0 = (t0 + lt) * 16;
      // 16-byte pieces per row: the int8 of the blocks, then the 8 scales from 2 * b0
      // (b0 % 8 == 0: inside the row's 16-byte-padded scale area)
      auto piece = [&](int r, int pc, int np) {
        if (row0 + r < a.N) {
          const uint8_t* rp = a.W + (size_t)(row0 + r) * a.S;
          if (pc < np - 1)
            cp_async16_stream(dst + (uint32_t)(r * kUnitRowBytes + pc * 16), rp + (size_t)b0 * 32 + pc * 16, pol);
          else
            cp_async16_stream(dst + (uint32_t)(r * kUnitRowBytes + 256), rp + a.K + 2 * b0, pol);
        }
      };
      if (nblk == kUnitBlocks) {
        constexpr int kPieces = 2 * kUnitBlocks + 1;
#pragma unroll
        for (int i = lane; i < 16 * kPieces; i += 32) piece(i / kPieces, i % kPieces, kPieces);
      } else {
        const int pieces = 2 * nblk + 1;
        for (int i = lane; i < 16 * pieces; i += 32) piece(i / pieces, i % pieces, pieces);
      }
    }
    cp_async_commit();
  };
  for (int t = 0; t < kMmDepth; ++t) issue(t);  // weights are constant: before the dependency wait
  pdl_wait();                                   // the quantized activations come from upstream

  // the int8 activations (rows 16 bytes longer than K: conflict-free fragment reads) and
  // their scales into shared memory behind the rings, once per CTA
  const uint32_t xstride = (uint32_t)a.K + 16u;
  const uint32_t xs = su32(smem) + (uint32_t)kMmRingBytes;
  const uint32_t dxs = xs + (uint32_t)round_up16((int64_t)a.M * xstride);
  if (a.qx) {  // quantized once per call by the quantization launch
    const int per_row = a.K >> 4;
    for (int i = threadIdx.x; i < a.M * per_row; i += kMmThreads) {
      const int m = i / per_row, c = i - m * per_row;
      cp_async16(xs + (uint32_t)m * xstride + 16u * c, a.qx + (size_t)m * a.K + 16 * c);
    }
    const int dpieces = (nb * a.Mp) >> 2;  // Mp % 16 == 0
    for (int i = threadIdx.x; i < dpieces; i += kMmThreads) cp_async16(dxs + 16u * i, a.dxT + 4 * i);
    cp_async_commit();
    cp_async_wait(0);  // (the ring's first units too: they were issued long before)
    __syncthreads();
  } else {  // small M*K: every CTA quantizes x itself, one 32-value block per thread
    for (int i = threadIdx.x; i < a.M * nb; i += kMmThreads) {
      const int m = i / nb, b = i - m * nb;
      const float4* src = reinterpret_cast<const float4*>(a.x + (size_t)m * a.K + (size_t)b * 32);
      float4 v[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t);
      int q[8];
      __half dh;
      quantize_block_regs(v, q, dh);
      const uint32_t d = xs + (uint32_t)m * xstride + 32u * (uint32_t)b;
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(d), "r"(q[0]), "r"(q[1]), "r"(q[2]), "r"(q[3])
                   : "memory");
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(d + 16u), "r"(q[4]), "r"(q[5]), "r"(q[6]),
                   "r"(q[7]) : "memory");
      asm volatile("st.shared.f32 [%0], %1;" ::"r"(dxs + 4u * (uint32_t)(b * a.Mp + m)), "f"(__half2float(dh))
                   : "memory");
    }
    __syncthreads();
  }

  const int g = lane >> 2, q = lane & 3;
  float accA[NT][4], accB[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      accA[nt][i] = 0.0f;
      accB[nt][i] = 0.0f;
    }
  auto write_tile = [&](int tile, const float (&acc)[NT][4]) {  // whole mode: straight to y
    const int r0 = tile * 16 + g, r1 = r0 + 8;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int m0 = nt * 8 + 2 * q, m1 = m0 + 1;
      if (m0 < a.M) {
        if (r0 < a.N) a.y[(size_t)m0 * a.N + r0] = acc[nt][0];
        if (r1 < a.N) a.y[(size_t)m0 * a.N + r1] = acc[nt][2];
      }
      if (m1 < a.M) {
        if (r0 < a.N) a.y[(size_t)m1 * a.N + r0] = acc[nt][1];
        if (r1 < a.N) a.y[(size_t)m1 * a.N + r1] = acc[nt][3];
      }
    }
  };
  int tileA = -1;
  bool touchedB = false;
  for (int t = 0; t < my_units; ++t) {
    cp_async_wait(kMmDepth - 1);  // this thread's copies of unit t have landed
    __syncwarp();                 // ... and every lane's
    int lt, ch;
    unit_of(t, lt, ch);
    const uint32_t slot = ring_s + (uint32_t)((t % kMmDepth) * kUnitBytes);
    const int b0 = ch * kUnitBlocks, nblk = min(kUnitBlocks, nb - b0);
    if (whole) {
      unit_mma<NT>(a, slot, xs, xstride, dxs, b0, nblk, accA);
      if (ch == nkc - 1) {
        write_tile(t0 + lt, accA);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) accA[nt][i] = 0.0f;
      }
    } else {
      if (tileA < 0) tileA = lt;
      if (lt == tileA) {
        unit_mma<NT>(a, slot, xs, xstride, dxs, b0, nblk, accA);
      } else {
        unit_mma<NT>(a, slot, xs, xstride, dxs, b0, nblk, accB);
        touchedB = true;
      }
    }
    __syncwarp();  // every lane is done with the slot before it is refilled
    issue(t + kMmDepth);
  }
  cp_async_wait(0);  // no copy of this warp outlives the loop (the trailing groups are empty)
  if (whole) return;

  // partial tiles -> shared memory (the ring is free once every warp is past its loop):
  // stage[warp][k][16 rows][16 activation rows], k = 0 the warp's first tile, 1 the next
  __syncthreads();
  float* stage = reinterpret_cast<float*>(smem);
  if (warp < nw && my_units > 0) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (k == 1 && !touchedB) break;
      float* st = stage + (size_t)(warp * 2 + k) * 256;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m0 = nt * 8 + 2 * q;
        const float* acc = k ? accB[nt] : accA[nt];
        st[g * 16 + m0] = acc[0];
        st[g * 16 + m0 + 1] = acc[1];
        st[(g + 8) * 16 + m0] = acc[2];
        st[(g + 8) * 16 + m0 + 1] = acc[3];
      }
    }
  }
  __syncthreads();
  // y[m][n] = the partials of the warps whose ranges meet the tile, in chunk order
  for (int i = threadIdx.x; i < ntc * 16 * a.M; i += kMmThreads) {
    const int lt = i / (16 * a.M), rem = i - lt * 16 * a.M, m = rem >> 4, r = rem & 15;
    const int n = (t0 + lt) * 16 + r;
    if (n >= a.N) continue;
    const int wf = (lt * nkc) / L, wl = min(nw - 1, ((lt + 1) * nkc - 1) / L);
    float v = 0.0f;
    for (int w = wf; w <= wl; ++w) {
      const int k = lt - (w * L) / nkc;  // 0 or 1: which of warp w's tiles this is
      const float p = stage[(size_t)(w * 2 + k) * 256 + r * 16 + m];
      v = w == wf ? p : __fadd_rn(v, p);
    }
    a.y[(size_t)m * a.N + n] = v;
  }
}

size_t up256_mm(size_t v) { return (v + 255) / 256 * 256; }
int mp_of(int64_t m) { return (int)((m + 15) / 16 * 16); }
// rings, then the int8 activations (rows K + 16 bytes apart) and their scales [K/32][Mp]
size_t mma_smem_bytes(int64_t m, int64_t k, int depth = 2) {
  return (size_t)ring_bytes(depth) + (size_t)round_up16(m * (k + 16)) + (size_t)mp_of(m) * (k / kQK) * sizeof(float);
}

template <int NT, int DEPTH>
cudaError_t launch_mma_t(const MmaArgs& a, int device, cudaStream_t s) {
  static int configured[128] = {0};
  auto fn = gemm_q8_0_mma_kernel<NT, DEPTH>;
  const size_t smem = mma_smem_bytes(a.M, a.K, DEPTH);
  cudaError_t e = ensure_smem((const void*)fn, configured, device, smem, true);
  if (e != cudaSuccess) return e;
  const int tiles = (a.N + 15) / 16;
  int grid = sm_count(device);
  if (grid > tiles) grid = tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace

// Where the activations fit beside two-slot rings in one CTA's shared memory.
bool mma_applies(int64_t m, int64_t k) {
  return m >= 2 && m <= kMmaMaxM && k <= (1 << 20) && mma_smem_bytes(m, k) <= kMmaMaxSmem;
}

// Whether every CTA quantizes the activations itself instead of a quantization launch
// before the kernel: where M*K is small (a few blocks per thread) and the CTAs hold
// several 16-row tiles each, so the quantization overlaps the weight stream.  Measured
// on B200 (graph-timed, us per call, in-kernel vs launch): gate_up 2048->12288 M=12
// 17.1 vs 20.1, M=16 18.6 vs 21.3; qkv 2048->6144 M=16 13.4 vs 13.6; but o 2048->2048
// (one tile per CTA) M=16 14.6 vs 8.7.  Q8LIN_MMA_QUANT=launch / =kernel force one way
// (comparisons).
bool mma_quant_in_kernel(int64_t m, int64_t k, int64_t n) {
  static const int mode = [] {
    const char* v = getenv("Q8LIN_MMA_QUANT");
    return v ? (v[0] == 'l' ? 0 : (v[0] == 'k' ? 2 : 1)) : 1;
  }();
  if (mode != 1) return mode == 2;
  return m * k <= kMmaInKernelMaxValues && n >= kMmaInKernelMinN;
}

// int8 activations [M][K], then their scales [K/32][Mp] (Mp = M rounded up to 16): what
// the quantization launch writes (the kernel that quantizes x itself leaves it unused)
size_t gemm_mma_workspace_bytes(int64_t m, int64_t k) {
  return up256_mm((size_t)(m * k)) + up256_mm((size_t)mp_of(m) * (k / kQK) * sizeof(float));
}

cudaError_t launch_gemm_mma(const q8lin_weight& w, const float* x, void* workspace, float* y, int64_t m,
                            cudaStream_t s) {
  if (!mma_applies(m, w.k)) return cudaErrorInvalidValue;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  MmaArgs a;
  a.W = static_cast<const uint8_t*>(w.packed);
  a.S = w.row_stride;
  a.N = (int)w.n;
  a.K = (int)w.k;
  a.M = (int)m;
  a.Mp = mp_of(m);
  a.y = y;
  a.x = x;
  if (mma_quant_in_kernel(m, w.k, w.n)) {
    a.qx = nullptr;
    a.dxT = nullptr;
  } else {
    a.qx = reinterpret_cast<const int8_t*>(ws);
    a.dxT = reinterpret_cast<const float*>(ws + up256_mm((size_t)(m * w.k)));
    cudaError_t e = launch_quantize_rows_i8t(x, a.M, a.Mp, a.K, reinterpret_cast<int8_t*>(ws),
                                             const_cast<float*>(a.dxT), s);
    if (e != cudaSuccess) return e;
  }
  // Three ring slots where they fit, except where every CTA quantizes x itself (there two
  // CTAs per SM let the next CTA start streaming during the quantization).  Measured on
  // B200 (graph-timed, us, 2 -> 3 slots): qkv 2048->6144 M=12 12.5 -> 10.5, M=16 13.6 ->
  // 12.1; o 2048->2048 M=16 8.7 -> 7.5; gate_up 2048->12288 (x quantized in the kernel)
  // M=16 18.6 -> 19.4.
  const bool deep = a.qx != nullptr && mma_smem_bytes(m, w.k, 3) <= kMmaMaxSmem;
  if (m <= 8) return deep ? launch_mma_t<1, 3>(a, w.device, s) : launch_mma_t<1, 2>(a, w.device, s);
  return deep ? launch_mma_t<2, 3>(a, w.device, s) : launch_mma_t<2, 2>(a, w.device, s);
}

}  // namespace q8lin
