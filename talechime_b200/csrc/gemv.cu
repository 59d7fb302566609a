// Decode GEMV for 1 <= M <= 16: y[M][N] = Q8_0(x)[M][K] . W^T.
//
// HBM-bound: every launch streams the whole repacked weight (N*K*34/32 bytes)
// once.  Each CTA quantizes all M activation rows into shared memory with candle's
// from_float rules (the activations are tiny next to the weight), then its warps
// walk disjoint weight rows: lanes stride a row in 16-byte chunks with 128-bit
// streaming loads, dp4a the chunk against the quantized activations, join the two
// half-blocks with one shuffle, scale each 32-value block term by f32(dw)*f32(dx)
// and reduce the row across the warp.
//
// Per-term rounding follows candle's scalar vec_dot (f32(isum)*dw, then *dx, each
// rounded); the sum over blocks is a strided tree rather than candle's sequential
// order, so outputs agree within f32 summation tolerance.
//
// Launched with programmatic dependent launch: nothing produced upstream (x) is
// read and nothing (y) is written before griddepcontrol.wait.
#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;  // 16-byte chunks in flight per lane per batch

template <int M>
__global__ void __launch_bounds__(kThreads)
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

  pdl_wait();

  for (int i = threadIdx.x; i < M * nb; i += blockDim.x) {
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)i * kQK);
    float4 v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t);
    int q[8];
    __half dh;
    quantize_block_regs(v, q, dh);
    int4* dst = reinterpret_cast<int4*>(qx + (size_t)i * kQK);
    dst[0] = make_int4(q[0], q[1], q[2], q[3]);
    dst[1] = make_int4(q[4], q[5], q[6], q[7]);
    dx[i] = __half2float(dh);
  }
  __syncthreads();
  pdl_launch_dependents();

  for (int row = r0 + warp; row < r1; row += nwarps) {
    const uint8_t* wr = W + (size_t)row * S;
    const __half* sr = reinterpret_cast<const __half*>(wr + K);
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.0f;

    for (int c0 = 0; c0 < nchunk; c0 += 32 * kUnroll) {
      int4 wv[kUnroll];
      float dw[kUnroll];
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
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32 + lane;
        const bool valid = c < nchunk;
        const int b = c >> 1;
        int is[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const int4 xv = valid ? *reinterpret_cast<const int4*>(qx + (size_t)m * K + (size_t)c * 16)
                                : make_int4(0, 0, 0, 0);
          is[m] = dot16(wv[u], xv, 0);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) is[m] += __shfl_xor_sync(kFull, is[m], 1);
        if (valid && !(lane & 1)) {
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const float term = __fmul_rn(__fmul_rn(__int2float_rn(is[m]), dw[u]), dx[m * nb + b]);
            acc[m] = __fadd_rn(acc[m], term);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float v = warp_sum(acc[m]);
      if (lane == 0) y[(size_t)m * N + row] = v;
    }
  }
}

template <int M>
cudaError_t launch_m(const q8lin_weight& w, const float* x, float* y, cudaStream_t s) {
  const int K = (int)w.k, N = (int)w.n;
  const size_t smem = (((size_t)M * K + 15) / 16) * 16 + (size_t)M * (K / kQK) * sizeof(float);
  // The dynamic shared-memory opt-in is per device context; remember it per device.
  static int configured_smem[128] = {0};
  const int dev = (w.device >= 0 && w.device < 128) ? w.device : 0;
  if ((int)smem > 48 * 1024 && (int)smem > configured_smem[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_q8_0_kernel<M>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured_smem[dev] = (int)smem;
  }
  const int sms = sm_count(w.device);
  int grid = 2 * sms;
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
  cfg.numAttrs = 1;
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
