// Weight repack / export / dequantize and the activation quantizer.
//
// HBM layout of one repacked Q8_0 weight (N rows, K in-features, nb = K/32):
//   row r at packed + r*S, S = packed_row_stride(K):
//     [0, K)               int8 qs, block b at [32b, 32b+32)
//     [K, K + 2*nb)        f16 d, block b at K + 2b
//     [K + 2*nb, S)        zero padding to a 16-byte multiple
// Rows start on 16-byte boundaries, so a row (or a run of rows) streams with 128-bit
// loads or bulk copies, and the int8 plane is a strided 2-D array for tiled copies.
#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

// One thread per GGUF block: 34 bytes {f16 d, int8 qs[32]} at 2-byte alignment.
__global__ void repack_kernel(const uint8_t* __restrict__ gguf, uint8_t* __restrict__ packed,
                              int64_t n, int64_t k, int64_t S) {
  const int64_t nb = k / kQK;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * nb) return;
  const int64_t r = i / nb, b = i - r * nb;
  const uint16_t* src = reinterpret_cast<const uint16_t*>(gguf + i * kBlockBytes);
  uint32_t w[8];
#pragma unroll
  for (int t = 0; t < 8; ++t)
    w[t] = (uint32_t)src[1 + 2 * t] | ((uint32_t)src[2 + 2 * t] << 16);
  uint8_t* row = packed + r * S;
  int4* dq = reinterpret_cast<int4*>(row + b * kQK);
  dq[0] = make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
  dq[1] = make_int4((int)w[4], (int)w[5], (int)w[6], (int)w[7]);
  reinterpret_cast<uint16_t*>(row + k)[b] = src[0];
  if (b == 0) {
    for (int64_t p = k + 2 * nb; p < S; ++p) row[p] = 0;
  }
}

__global__ void unpack_kernel(const uint8_t* __restrict__ packed, uint8_t* __restrict__ gguf,
                              int64_t n, int64_t k, int64_t S) {
  const int64_t nb = k / kQK;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * nb) return;
  const int64_t r = i / nb, b = i - r * nb;
  const uint8_t* row = packed + r * S;
  const uint16_t* q16 = reinterpret_cast<const uint16_t*>(row + b * kQK);
  uint16_t* dst = reinterpret_cast<uint16_t*>(gguf + i * kBlockBytes);
  dst[0] = reinterpret_cast<const uint16_t*>(row + k)[b];
#pragma unroll
  for (int t = 0; t < 16; ++t) dst[1 + t] = q16[t];
}

// One thread per block: x = f32(q) * f32(d).
__global__ void dequantize_kernel(const uint8_t* __restrict__ packed, float* __restrict__ out,
                                  int64_t n, int64_t k, int64_t S) {
  const int64_t nb = k / kQK;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * nb) return;
  const int64_t r = i / nb, b = i - r * nb;
  const uint8_t* row = packed + r * S;
  const float d = __half2float(reinterpret_cast<const __half*>(row + k)[b]);
  const int4* q = reinterpret_cast<const int4*>(row + b * kQK);
  float4* o = reinterpret_cast<float4*>(out + r * k + b * kQK);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int4 v = q[h];
    const int w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float4 f;
      f.x = __fmul_rn((float)(int8_t)(w[t] & 0xff), d);
      f.y = __fmul_rn((float)(int8_t)((w[t] >> 8) & 0xff), d);
      f.z = __fmul_rn((float)(int8_t)((w[t] >> 16) & 0xff), d);
      f.w = __fmul_rn((float)(int8_t)((w[t] >> 24) & 0xff), d);
      o[h * 4 + t] = f;
    }
  }
}

// One thread per (row, block) of the activations.
__global__ void quantize_rows_kernel(const float* __restrict__ x, int64_t m, int64_t k,
                                     int8_t* __restrict__ qs, uint16_t* __restrict__ d_f16,
                                     float* __restrict__ d_f32) {
  const int64_t nb = k / kQK;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  if (i < m * nb) {
    const float4* src = reinterpret_cast<const float4*>(x + i * kQK);
    float4 v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t);
    int q[8];
    __half dh;
    quantize_block_regs(v, q, dh);
    int4* dst = reinterpret_cast<int4*>(qs + i * kQK);
    dst[0] = make_int4(q[0], q[1], q[2], q[3]);
    dst[1] = make_int4(q[4], q[5], q[6], q[7]);
    if (d_f16) d_f16[i] = __half_as_ushort(dh);
    if (d_f32) d_f32[i] = __half2float(dh);
  }
}

inline unsigned blocks_for(int64_t work, int threads) {
  return (unsigned)((work + threads - 1) / threads);
}

}  // namespace

cudaError_t launch_repack(const uint8_t* gguf, uint8_t* packed, int64_t n, int64_t k,
                          int64_t S, cudaStream_t s) {
  const int64_t work = n * (k / kQK);
  if (work == 0) return cudaSuccess;
  repack_kernel<<<blocks_for(work, 256), 256, 0, s>>>(gguf, packed, n, k, S);
  return cudaGetLastError();
}

cudaError_t launch_unpack(const uint8_t* packed, uint8_t* gguf, int64_t n, int64_t k,
                          int64_t S, cudaStream_t s) {
  const int64_t work = n * (k / kQK);
  if (work == 0) return cudaSuccess;
  unpack_kernel<<<blocks_for(work, 256), 256, 0, s>>>(packed, gguf, n, k, S);
  return cudaGetLastError();
}

cudaError_t launch_dequantize(const uint8_t* packed, float* out, int64_t n, int64_t k,
                              int64_t S, cudaStream_t s) {
  const int64_t work = n * (k / kQK);
  if (work == 0) return cudaSuccess;
  dequantize_kernel<<<blocks_for(work, 256), 256, 0, s>>>(packed, out, n, k, S);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const float* x, int64_t m, int64_t k, int8_t* qs,
                                 uint16_t* d_f16, float* d_f32, cudaStream_t s) {
  const int64_t work = m * (k / kQK);
  if (work == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks_for(work, 128));
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, quantize_rows_kernel, x, m, k, qs, d_f16, d_f32);
}

}  // namespace q8lin
