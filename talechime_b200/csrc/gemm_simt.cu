// Batched Q8_0 matmul for M > 16 over pre-quantized activations (CUDA cores).
//
// y[m][n] = sum_b (f32(isum[m][n][b]) * dw[n][b]) * dx[m][b], isum exact via dp4a.
// CTA tile: 64 weight rows x 64 activation rows, one 32-value block per K step.
// This is the portable correctness path for the batched case; the tensor-core
// kernel replaces it where it applies.
#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

constexpr int kTile = 64;
constexpr int kRowPad = 48;  // bytes per smem row (32 data + 16 pad)

__global__ void __launch_bounds__(256)
gemm_q8_0_simt_kernel(const uint8_t* __restrict__ W, int64_t S, int N, int K,
                      const int8_t* __restrict__ qx, const float* __restrict__ dx,
                      float* __restrict__ y, int M) {
  __shared__ __align__(16) int8_t sw[kTile * kRowPad];
  __shared__ __align__(16) int8_t sx[kTile * kRowPad];
  __shared__ float sdw[kTile], sdx[kTile];
  const int nb = K >> 5;
  const int n0 = blockIdx.x * kTile, m0 = blockIdx.y * kTile;
  const int t = threadIdx.x;
  const int tx = t & 15, ty = t >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  pdl_wait();
  for (int b = 0; b < nb; ++b) {
    if (t < 128) {
      const int r = t >> 1, h = t & 1;
      int4 v = make_int4(0, 0, 0, 0);
      if (n0 + r < N) v = ld_stream_v4(W + (size_t)(n0 + r) * S + (size_t)b * kQK + h * 16);
      *reinterpret_cast<int4*>(sw + r * kRowPad + h * 16) = v;
    } else {
      const int r = (t - 128) >> 1, h = t & 1;
      int4 v = make_int4(0, 0, 0, 0);
      if (m0 + r < M) v = *reinterpret_cast<const int4*>(qx + (size_t)(m0 + r) * K + (size_t)b * kQK + h * 16);
      *reinterpret_cast<int4*>(sx + r * kRowPad + h * 16) = v;
    }
    if (t < kTile) {
      sdw[t] = (n0 + t < N) ? __half2float(reinterpret_cast<const __half*>(W + (size_t)(n0 + t) * S + K)[b]) : 0.0f;
    } else if (t < 2 * kTile) {
      const int r = t - kTile;
      sdx[r] = (m0 + r < M) ? dx[(size_t)(m0 + r) * nb + b] : 0.0f;
    }
    __syncthreads();
    int4 wv[4][2], xv[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int8_t* pw = sw + (tx + 16 * i) * kRowPad;
      wv[i][0] = *reinterpret_cast<const int4*>(pw);
      wv[i][1] = *reinterpret_cast<const int4*>(pw + 16);
      const int8_t* px = sx + (ty + 16 * i) * kRowPad;
      xv[i][0] = *reinterpret_cast<const int4*>(px);
      xv[i][1] = *reinterpret_cast<const int4*>(px + 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float dwi = sdw[tx + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int is = dot16(wv[i][1], xv[j][1], dot16(wv[i][0], xv[j][0], 0));
        const float term = __fmul_rn(__fmul_rn(__int2float_rn(is), dwi), sdx[ty + 16 * j]);
        acc[i][j] = __fadd_rn(acc[i][j], term);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int m = m0 + ty + 16 * j;
    if (m >= M) continue;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = n0 + tx + 16 * i;
      if (n < N) y[(size_t)m * N + n] = acc[i][j];
    }
  }
}

}  // namespace

cudaError_t launch_gemm(const q8lin_weight& w, const int8_t* qx, const float* dx, float* y,
                        int64_t m, cudaStream_t s) {
  const int N = (int)w.n, K = (int)w.k;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + kTile - 1) / kTile), (unsigned)((m + kTile - 1) / kTile));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemm_q8_0_simt_kernel, (const uint8_t*)w.packed, w.row_stride,
                            N, K, qx, dx, y, (int)m);
}

}  // namespace q8lin
