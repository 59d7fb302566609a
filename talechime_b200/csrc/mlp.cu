// SwiGLU between the gate/up and down projections of the VoxCPM MLP
// (crates/voxcpm/src/transformer.rs:147-150: down(silu(gate(h)) * up(h))).
//
// Input gu[M][2I]: columns [0, I) are the gate projection, [I, 2I) the up projection --
// the output of one fused gate+up linear whose weight rows are the gate rows followed by
// the up rows (the same layout per tensor-parallel shard).  Output h[M][I] =
// silu(gate) * up with candle's f32 silu, v / (1 + exp(-v)): each operation rounded to
// f32; exp is CUDA's expf (within 2 ulp of exp), so results agree with the CPU path
// within f32 tolerance rather than bit for bit.
#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

// Four outputs per thread when I is a multiple of 4 (rows then start on 16 bytes).
__global__ void swiglu4_kernel(const float* __restrict__ gu, int64_t m, int64_t inter, float* __restrict__ h) {
  const int64_t q = inter / 4;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  if (i < m * q) {
    const int64_t r = i / q, c = i - r * q;
    const float4 g = reinterpret_cast<const float4*>(gu + r * 2 * inter)[c];
    const float4 u = reinterpret_cast<const float4*>(gu + r * 2 * inter + inter)[c];
    reinterpret_cast<float4*>(h + r * inter)[c] =
        make_float4(silu_mul(g.x, u.x), silu_mul(g.y, u.y), silu_mul(g.z, u.z), silu_mul(g.w, u.w));
  }
}

__global__ void swiglu1_kernel(const float* __restrict__ gu, int64_t m, int64_t inter, float* __restrict__ h) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  if (i < m * inter) {
    const int64_t r = i / inter, c = i - r * inter;
    h[i] = silu_mul(gu[r * 2 * inter + c], gu[r * 2 * inter + inter + c]);
  }
}

}  // namespace

cudaError_t launch_swiglu(const float* gu, int64_t m, int64_t inter, float* h, cudaStream_t s) {
  if (m == 0 || inter == 0) return cudaSuccess;
  const bool vec = (inter % 4) == 0 && (reinterpret_cast<uintptr_t>(gu) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(h) & 15u) == 0;
  const int64_t work = vec ? m * (inter / 4) : m * inter;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((work + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return vec ? cudaLaunchKernelEx(&cfg, swiglu4_kernel, gu, m, inter, h)
             : cudaLaunchKernelEx(&cfg, swiglu1_kernel, gu, m, inter, h);
}

}  // namespace q8lin
