// Decode GEMV for 1 <= M <= 16: y[M][N] = Q8_0(x)[M][K] . W^T.
//
// HBM-bound: every launch streams the whole repacked weight (N*K*34/32 bytes) once.
// Geometry: two 512-thread CTAs per SM; CTA c owns the contiguous weight rows
// [N*c/G, N*(c+1)/G), its warps take those rows round-robin, and the 32 lanes of a
// warp stride a row in 16-byte chunks (chunk c = half of block c/2) with 128-bit
// streaming loads, four chunks in flight per lane and the next batch issued before
// the current one is reduced.
//
// Dependent-launch structure (the kernel is launched with programmatic stream
// serialization):
//   1. prologue -- weights are constant, so before griddepcontrol.wait every warp
//      issues its first weight batch into registers.  This overlaps the upstream
//      kernel's tail and the dependency-release latency.
//   2. griddepcontrol.wait, then launch_dependents so the next kernel's prologue
//      can start.
//   3. the CTA quantizes the M activation rows into shared memory with candle's
//      from_float rules, 8 lanes per 32-value block.
//   4. dp4a against the quantized activations, the two half-blocks joined with
//      one shuffle, each block term scaled as candle's scalar vec_dot does
//      ((f32(isum) * dw) * dx, each product rounded) and the row reduced across
//      the warp.  The sum over blocks is a tree, so outputs agree with the
//      sequential CPU order within f32 summation tolerance.
// Nothing upstream (x) is read and nothing (y) is written before step 2.
#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

constexpr int kThreads = 512;
constexpr int kUnroll = 4;  // 16-byte chunks in flight per lane per batch

template <int M>
__global__ void __launch_bounds__(kThreads, (M <= 4 ? 2 : 1))
gemv_q8_0_kernel(const uint8_t* __restrict__ W, int64_t S, int N, int K,
                 const float* __restrict__ x, float* __restrict__ y) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = K >> 5;
  const int nchunk = K >> 4;
  int8_t* qx = reinterpret_cast<int8_t*>(smem);
  float* dx = reinterpret_cast<float*>(smem + (((size_t)M * K + 15) / 16) * 16);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int r0 = (int)(((int64_t)N * blockIdx.x) / gridDim.x);
  const int r1 = (int)(((int64_t)N * (blockIdx.x + 1)) / gridDim.x);

  // ---- 1. prologue: weights only ------------------------------------------------
  const int nbat = (nchunk + 32 * kUnroll - 1) / (32 * kUnroll);
  const int my_rows = (r0 + warp < r1) ? (r1 - r0 - warp + nwarps - 1) / nwarps : 0;
  const int total = my_rows * nbat;

  auto load_batch = [&](int it, int4 (&wv)[kUnroll], float (&dw)[kUnroll]) {
    const int row = r0 + warp + (it / nbat) * nwarps;
    const int c0 = (it % nbat) * 32 * kUnroll;
    const uint8_t* wr = W + (size_t)row * S;
    const __half* sr = reinterpret_cast<const __half*>(wr + K);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < nchunk) {
        wv[u] = ld_stream_v4(wr + (size_t)c * 16);
        dw[u] = __half2float(sr[c >> 1]);
      } else {
        wv[u] = make_int4(0, 0, 0, 0);
        dw[u] = 0.0f;
      }
    }
  };

  int4 cur[kUnroll];
  float dcur[kUnroll];
  if (total > 0) load_batch(0, cur, dcur);

  // ---- 2. dependency on the producer of x ---------------------------------------
  pdl_wait();
  pdl_launch_dependents();

  // ---- 3. activations -> Q8_0 in shared memory (8 lanes per block) --------------
  // The loads of four passes are issued together: one L2 round trip per group.
  const int nquads = M * nb * 8;  // float4 pieces of x
  constexpr int kQG = 4;
  for (int base = 0; base < nquads; base += kQG * kThreads) {
    float4 v[kQG];
#pragma unroll
    for (int g = 0; g < kQG; ++g) {
      const int i = base + g * kThreads + threadIdx.x;
      v[g] = i < nquads ? __ldg(reinterpret_cast<const float4*>(x) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int g = 0; g < kQG; ++g) {
      if (base + g * kThreads < nquads) {  // uniform across the CTA: every lane shuffles
        const int i = base + g * kThreads + threadIdx.x;
        __half dh;
        const int q = quantize_octet(v[g], dh);
        if (i < nquads) {
          reinterpret_cast<int*>(qx)[i] = q;
          if ((i & 7) == 0) dx[i >> 3] = __half2float(dh);
        }
      }
    }
  }
  __syncthreads();

  // ---- 4. rows -------------------------------------------------------------------
  float acc[M];
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = 0.0f;

  for (int it = 0; it < total; ++it) {
    int4 nxt[kUnroll];
    float dnxt[kUnroll];
    if (it + 1 < total) load_batch(it + 1, nxt, dnxt);
    const int row = r0 + warp + (it / nbat) * nwarps;
    const int bj = it % nbat;
    const int c0 = bj * 32 * kUnroll;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      const bool valid = c < nchunk;
      int is[M];
      float dxv[M];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const int4 xv = valid ? *reinterpret_cast<const int4*>(qx + (size_t)m * K + (size_t)c * 16)
                              : make_int4(0, 0, 0, 0);
        dxv[m] = valid ? dx[m * nb + (c >> 1)] : 0.0f;
        is[m] = dot16(cur[u], xv, 0);
      }
#pragma unroll
      for (int m = 0; m < M; ++m) is[m] += __shfl_xor_sync(kFull, is[m], 1);
      if (valid && !(lane & 1)) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float term = __fmul_rn(__fmul_rn(__int2float_rn(is[m]), dcur[u]), dxv[m]);
          acc[m] = __fadd_rn(acc[m], term);
        }
      }
    }
    if (bj == nbat - 1) {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float v = warp_sum(acc[m]);
        if (lane == 0) y[(size_t)m * N + row] = v;
        acc[m] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      cur[u] = nxt[u];
      dcur[u] = dnxt[u];
    }
  }
}

template <int M>
cudaError_t launch_m(const q8lin_weight& w, const float* x, float* y, cudaStream_t s) {
  const int K = (int)w.k, N = (int)w.n;
  const size_t smem = gemv_smem_bytes(M, K);
  // The dynamic shared-memory opt-in is per device context; remember it per device.
  static int configured_smem[128] = {0};
  const int dev = (w.device >= 0 && w.device < 128) ? w.device : 0;
  if ((int)smem > 48 * 1024 && (int)smem > configured_smem[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_q8_0_kernel<M>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured_smem[dev] = (int)smem;
  }
  int grid = 2 * sm_count(w.device);
  if (grid > N) grid = N;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_q8_0_kernel<M>, (const uint8_t*)w.packed, w.row_stride,
                            N, K, x, y);
}

}  // namespace

size_t gemv_smem_bytes(int m, int64_t k) {
  return (((size_t)m * k + 15) / 16) * 16 + (size_t)m * (k / kQK) * sizeof(float);
}

cudaError_t launch_gemv(const q8lin_weight& w, const float* x, float* y, int m, cudaStream_t s) {
  switch (m) {
    case 1: return launch_m<1>(w, x, y, s);
    case 2: return launch_m<2>(w, x, y, s);
    case 3: return launch_m<3>(w, x, y, s);
    case 4: return launch_m<4>(w, x, y, s);
    case 5: return launch_m<5>(w, x, y, s);
    case 6: return launch_m<6>(w, x, y, s);
    case 7: return launch_m<7>(w, x, y, s);
    case 8: return launch_m<8>(w, x, y, s);
    case 9: return launch_m<9>(w, x, y, s);
    case 10: return launch_m<10>(w, x, y, s);
    case 11: return launch_m<11>(w, x, y, s);
    case 12: return launch_m<12>(w, x, y, s);
    case 13: return launch_m<13>(w, x, y, s);
    case 14: return launch_m<14>(w, x, y, s);
    case 15: return launch_m<15>(w, x, y, s);
    case 16: return launch_m<16>(w, x, y, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace q8lin
