// Prefill kernels of the decoder: B sequences, each with T new rows at positions
// pos0 .. pos0 + T - 1, run as one batched forward (the reference's prompt pass,
// crates/voxcpm/src/model.rs:492-495 -> transformer.rs:107-155 with offset = pos0 and
// t = T).  The linears, norms, SwiGLU and residual adds of that pass are the M = B*T
// entry points of the library; these two kernels are the parts that depend on the
// position:
//   * rope_kv_rows: rotary embedding of q and k of every row at its own position
//     (tables of transformer.rs:44-65, rotate() :159-170: x*[cos,cos] +
//     [second,first]*[-sin,sin], each product rounded), rotated q to q_out, rotated k
//     and v appended to the sequence's f32 KV cache (the cat-growth of :131-139,
//     preallocated);
//   * attention_prefill: causal grouped attention (attention.rs:28-98 with causal = true:
//     key j is excluded for query row i when j > offset + i, :84-95), scores q.k times
//     the f32 rounding of 1/sqrt(128), softmax over the visible keys in f32, times V;
//     kv head = q head / (Hq / Hkv).
// Layouts: qkv [B*T][(Hq + 2 Hkv) D] (row b*T + t), q_out / out [B*T][Hq][D], caches
// [B][Hkv][max_t][D], cos / sin [max_t][D/2].  The host checks pos0 >= 0 and
// pos0 + T <= max_t (the reference's context-limit error) before launching.
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

__global__ void rope_kv_rows_kernel(const float* __restrict__ qkv, int T, int pos0, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, float* __restrict__ kc, float* __restrict__ vc,
                                    int Hq, int Hkv, int D, int max_t, float* __restrict__ q_out) {
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  const int row = blockIdx.x;  // b * T + t
  const int b = row / T, t = row - b * T;
  const int pos = pos0 + t;
  const int head = blockIdx.y;  // 0..Hq+Hkv-1 rotated heads, then Hkv value heads
  const int i = threadIdx.x;
  const int half = D / 2;
  const float* xr = qkv + (size_t)row * (Hq + 2 * Hkv) * D;
  if (i >= D || pos < 0 || pos >= max_t) return;
  if (head < Hq + Hkv) {
    const float* xh = xr + (size_t)head * D;
    const int j = i < half ? i : i - half;
    const float c = cos_t[(size_t)pos * half + j];
    const float sn = sin_t[(size_t)pos * half + j];
    const float r = i < half ? __fadd_rn(__fmul_rn(xh[i], c), __fmul_rn(xh[i + half], -sn))
                             : __fadd_rn(__fmul_rn(xh[i], c), __fmul_rn(xh[i - half], sn));
    if (head < Hq)
      q_out[((size_t)row * Hq + head) * D + i] = r;
    else
      kc[(((size_t)b * Hkv + (head - Hq)) * max_t + pos) * D + i] = r;
  } else if (head < Hq + 2 * Hkv) {
    const int hv = head - Hq - Hkv;
    vc[(((size_t)b * Hkv + hv) * max_t + pos) * D + i] = xr[(size_t)head * D + i];
  }
}

// The same rotation with float4 pieces, one CTA per row (d % 8 == 0, 16-byte aligned
// rows): a thread rotates four dimensions of each half of a head at once, with the
// per-element products and sums of the scalar kernel, so the results are identical.
__global__ void __launch_bounds__(256)
rope_kv_rows_vec_kernel(const float* __restrict__ qkv, int T, int pos0, const float* __restrict__ cos_t,
                        const float* __restrict__ sin_t, float* __restrict__ kc, float* __restrict__ vc, int Hq,
                        int Hkv, int D, int max_t, float* __restrict__ q_out) {
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  const int row = blockIdx.x;
  const int b = row / T, t = row - b * T;
  const int pos = pos0 + t;
  if (pos < 0 || pos >= max_t) return;
  const int half = D / 2, h4 = half / 4, d4 = D / 4;
  const float4* xr = reinterpret_cast<const float4*>(qkv + (size_t)row * (Hq + 2 * Hkv) * D);
  const float4* c4 = reinterpret_cast<const float4*>(cos_t + (size_t)pos * half);
  const float4* s4 = reinterpret_cast<const float4*>(sin_t + (size_t)pos * half);
  const int nrot = (Hq + Hkv) * h4;
  for (int it = threadIdx.x; it < nrot; it += blockDim.x) {
    const int head = it / h4, j = it - head * h4;
    const float4 a = xr[head * d4 + j], o = xr[head * d4 + h4 + j];
    const float4 c = __ldg(c4 + j), sn = __ldg(s4 + j);
    // first half x*cos + second*(-sin); second half x*cos + first*sin
    const float4 lo = make_float4(__fadd_rn(__fmul_rn(a.x, c.x), __fmul_rn(o.x, -sn.x)),
                                  __fadd_rn(__fmul_rn(a.y, c.y), __fmul_rn(o.y, -sn.y)),
                                  __fadd_rn(__fmul_rn(a.z, c.z), __fmul_rn(o.z, -sn.z)),
                                  __fadd_rn(__fmul_rn(a.w, c.w), __fmul_rn(o.w, -sn.w)));
    const float4 hi = make_float4(__fadd_rn(__fmul_rn(o.x, c.x), __fmul_rn(a.x, sn.x)),
                                  __fadd_rn(__fmul_rn(o.y, c.y), __fmul_rn(a.y, sn.y)),
                                  __fadd_rn(__fmul_rn(o.z, c.z), __fmul_rn(a.z, sn.z)),
                                  __fadd_rn(__fmul_rn(o.w, c.w), __fmul_rn(a.w, sn.w)));
    float4* dst = head < Hq ? reinterpret_cast<float4*>(q_out + ((size_t)row * Hq + head) * D)
                            : reinterpret_cast<float4*>(kc + (((size_t)b * Hkv + (head - Hq)) * max_t + pos) * D);
    dst[j] = lo;
    dst[h4 + j] = hi;
  }
  const int nv = Hkv * d4;
  for (int it = threadIdx.x; it < nv; it += blockDim.x) {
    const int hv = it / d4, j = it - hv * d4;
    reinterpret_cast<float4*>(vc + (((size_t)b * Hkv + hv) * max_t + pos) * D)[j] = xr[(Hq + Hkv + hv) * d4 + j];
  }
}

// x[r] += y[r]; h[r] = x[r] / sqrt(sum(x[r]^2) / n + eps) * w  (the residual add and the
// rms_norm that follows it, transformer.rs:146-147 and :107-117 of the next layer), one
// CTA of 256 threads per row, the row held in registers (n % 4 == 0, n <= 8192, 16-byte
// aligned rows); sum of squares per thread, then warps, then the 8 warp sums in order.
constexpr int kArThreads = 256;
constexpr int kArMaxN = 8192;
__global__ void __launch_bounds__(kArThreads)
add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ w, float eps, int n,
                   float* __restrict__ h) {
  constexpr int kV = kArMaxN / 4 / kArThreads;
  __shared__ float red[kArThreads / 32];
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  float4* xr = reinterpret_cast<float4*>(x + (size_t)blockIdx.x * n);
  const float4* yr = reinterpret_cast<const float4*>(y + (size_t)blockIdx.x * n);
  float4* hr = reinterpret_cast<float4*>(h + (size_t)blockIdx.x * n);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const int n4 = n / 4;
  float4 v[kV];
  float sq = 0.0f;
#pragma unroll
  for (int k = 0; k < kV; ++k) {
    const int i = threadIdx.x + k * kArThreads;
    if (i < n4) {
      const float4 a = xr[i], bb = yr[i];
      v[k] = make_float4(__fadd_rn(a.x, bb.x), __fadd_rn(a.y, bb.y), __fadd_rn(a.z, bb.z), __fadd_rn(a.w, bb.w));
      xr[i] = v[k];
      sq = __fadd_rn(sq, __fmul_rn(v[k].x, v[k].x));
      sq = __fadd_rn(sq, __fmul_rn(v[k].y, v[k].y));
      sq = __fadd_rn(sq, __fmul_rn(v[k].z, v[k].z));
      sq = __fadd_rn(sq, __fmul_rn(v[k].w, v[k].w));
    }
  }
  sq = warp_sum(sq);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int i = 0; i < kArThreads / 32; ++i) total = __fadd_rn(total, red[i]);
  const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)n), eps));
#pragma unroll
  for (int k = 0; k < kV; ++k) {
    const int i = threadIdx.x + k * kArThreads;
    if (i < n4) {
      const float4 wv = __ldg(w4 + i);
      hr[i] = make_float4(__fmul_rn(__fdiv_rn(v[k].x, m), wv.x), __fmul_rn(__fdiv_rn(v[k].y, m), wv.y),
                          __fmul_rn(__fdiv_rn(v[k].z, m), wv.z), __fmul_rn(__fdiv_rn(v[k].w, m), wv.w));
    }
  }
}

// ---------------------------------------------------------------------------------
// attention_prefill: grid (ceil(T / 16A), Hq, B), 256 threads; one CTA = 16A query rows
// of one head of one sequence, flash-style over 64-key tiles of the cache:
//   * q rows staged once, K / V tiles double-buffered in shared memory (cp.async, rows
//     past the sequence's pos0 + T valid rows zero-filled, so no stale cache row can
//     reach the sums);
//   * thread (ty, tx) of 16 x 16 holds the scores of rows A*ty + a and keys tx + 16b
//     (a < A, b < 4; q / k rows padded to 132 floats: every 8-lane phase of a 16-byte
//     shared load hits 32 distinct banks) and the output of rows A*ty + a, dimensions
//     tx*4 .. +4 and 64 + tx*4 .. +4; probabilities are stored key-major, so one
//     load gives a key's A rows;
//   * per tile: scores, the causal mask, a running max / sum per row (online softmax,
//     the 16 lanes of a row reduced with xor shuffles), probabilities through shared
//     memory, O += P V;
//   * out = O / sum.  Query tiles are taken longest first (blockIdx.x reversed).
// A rows per thread: 64-row query tiles (A = 4), or 32-row tiles (A = 2) where the
// 64-row grid would occupy fewer than half of the SMs (a short prompt, one sequence).
constexpr int kPfKeys = 64;
constexpr int kPfThreads = 256;
constexpr int kPfD = 128;
constexpr int kPfQStride = 132;

template <int A>
struct PfSmem {
  static constexpr int kRows = 16 * A;
  static constexpr int kPStride = kRows + 4;  // key-major probabilities, padded
  alignas(16) float q[kRows][kPfQStride];
  alignas(16) float k[2][kPfKeys][kPfQStride];
  alignas(16) float v[2][kPfKeys][kPfD];
  alignas(16) float p[kPfKeys][kPStride];
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

template <int A>
__global__ void __launch_bounds__(kPfThreads, 1)
attention_prefill_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                         int T, int pos0, int Hq, int Hkv, int max_t, float scale, float* __restrict__ out) {
  constexpr int kPfRows = PfSmem<A>::kRows;
  extern __shared__ __align__(16) uint8_t pf_smem[];
  PfSmem<A>& sm = *reinterpret_cast<PfSmem<A>*>(pf_smem);
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  const int qt = (int)gridDim.x - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (Hq / Hkv);
  const int q0 = qt * kPfRows;
  const int qrows = min(kPfRows, T - q0);
  const int len = pos0 + T;             // valid cache rows of the sequence after the append
  const int kend = pos0 + q0 + qrows;   // keys [0, kend) are visible to some row of the tile
  const int nkt = (kend + kPfKeys - 1) / kPfKeys;
  const float* kbase = kc + ((size_t)b * Hkv + hk) * (size_t)max_t * kPfD;
  const float* vbase = vc + ((size_t)b * Hkv + hk) * (size_t)max_t * kPfD;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);

  pdl_wait();  // q and the cache rows come from the kernels before this one
  for (int c = tid; c < kPfRows * 32; c += kPfThreads) {
    const int r = c >> 5, ch = c & 31;
    float* dst = &sm.q[r][ch * 4];
    if (r < qrows)
      cp_async16(smem_addr(dst), q + (((size_t)b * T + q0 + r) * Hq + h) * kPfD + ch * 4);
    else
      *reinterpret_cast<float4*>(dst) = zero4;
  }
  auto load_kv = [&](int kt, int buf) {
    for (int c = tid; c < kPfKeys * 32; c += kPfThreads) {
      const int r = c >> 5, ch = c & 31;
      const int j = kt * kPfKeys + r;
      float* dk = &sm.k[buf][r][ch * 4];
      float* dv = &sm.v[buf][r][ch * 4];
      if (j < len) {
        cp_async16(smem_addr(dk), kbase + (size_t)j * kPfD + ch * 4);
        cp_async16(smem_addr(dv), vbase + (size_t)j * kPfD + ch * 4);
      } else {
        *reinterpret_cast<float4*>(dk) = zero4;
        *reinterpret_cast<float4*>(dv) = zero4;
      }
    }
    cp_async_commit();
  };
  load_kv(0, 0);  // the q copies travel in the first group

  float o[A][8];
  float m_run[A], l_run[A];
#pragma unroll
  for (int a = 0; a < A; ++a) {
    m_run[a] = -INFINITY;
    l_run[a] = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[a][e] = 0.0f;
  }

  for (int kt = 0; kt < nkt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < nkt) {
      load_kv(kt + 1, buf ^ 1);  // that buffer's last readers passed the loop-end barrier
      cp_async_wait(1);
    } else {
      cp_async_wait(0);
    }
    __syncthreads();

    // scores of rows A*ty + a against keys tx + 16b
    float s[A][4];
#pragma unroll
    for (int a = 0; a < A; ++a)
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) s[a][bb] = 0.0f;
#pragma unroll 4
    for (int d4 = 0; d4 < kPfD / 4; ++d4) {
      float4 qa[A], kb[4];
#pragma unroll
      for (int a = 0; a < A; ++a) qa[a] = *reinterpret_cast<const float4*>(&sm.q[A * ty + a][d4 * 4]);
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) kb[bb] = *reinterpret_cast<const float4*>(&sm.k[buf][tx + 16 * bb][d4 * 4]);
#pragma unroll
      for (int a = 0; a < A; ++a)
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
          float acc = s[a][bb];
          acc = __fmaf_rn(qa[a].x, kb[bb].x, acc);
          acc = __fmaf_rn(qa[a].y, kb[bb].y, acc);
          acc = __fmaf_rn(qa[a].z, kb[bb].z, acc);
          acc = __fmaf_rn(qa[a].w, kb[bb].w, acc);
          s[a][bb] = acc;
        }
    }

    // causal mask, online softmax; probabilities to shared memory
    const int j0 = kt * kPfKeys;
#pragma unroll
    for (int a = 0; a < A; ++a) {
      const int qpos = pos0 + q0 + A * ty + a;  // absolute position of the row
      float mx = -INFINITY;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const int j = j0 + tx + 16 * bb;
        const float v = (j > qpos) ? -INFINITY : __fmul_rn(s[a][bb], scale);
        s[a][bb] = v;
        mx = fmaxf(mx, v);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      // key 0 is visible to every row, so mn is finite from the first tile on
      const float mn = fmaxf(m_run[a], mx);
      const float corr = expf(m_run[a] - mn);  // 0 on the first tile (m_run = -inf)
      float ps = 0.0f;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const float p = expf(s[a][bb] - mn);  // masked keys: exp(-inf) = 0
        s[a][bb] = p;
        ps = __fadd_rn(ps, p);
      }
      l_run[a] = __fadd_rn(__fmul_rn(l_run[a], corr), ps);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[a][e] = __fmul_rn(o[a][e], corr);
      m_run[a] = mn;
    }
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
      if constexpr (A == 4)
        *reinterpret_cast<float4*>(&sm.p[tx + 16 * bb][4 * ty]) = make_float4(s[0][bb], s[1][bb], s[2][bb], s[3][bb]);
      else
        *reinterpret_cast<float2*>(&sm.p[tx + 16 * bb][2 * ty]) = make_float2(s[0][bb], s[1][bb]);
    }
    __syncthreads();

    // O += P V over the keys of the tile that some row can see
    const int jn = min(kPfKeys, kend - j0);
#pragma unroll 4
    for (int j = 0; j < jn; ++j) {
      const float4 v0 = *reinterpret_cast<const float4*>(&sm.v[buf][j][tx * 4]);
      const float4 v1 = *reinterpret_cast<const float4*>(&sm.v[buf][j][64 + tx * 4]);
      float pj[A];
      if constexpr (A == 4) {
        const float4 p4 = *reinterpret_cast<const float4*>(&sm.p[j][4 * ty]);
        pj[0] = p4.x, pj[1] = p4.y, pj[2] = p4.z, pj[3] = p4.w;
      } else {
        const float2 p2 = *reinterpret_cast<const float2*>(&sm.p[j][2 * ty]);
        pj[0] = p2.x, pj[1] = p2.y;
      }
#pragma unroll
      for (int a = 0; a < A; ++a) {
        const float pa = pj[a];
        o[a][0] = __fmaf_rn(pa, v0.x, o[a][0]);
        o[a][1] = __fmaf_rn(pa, v0.y, o[a][1]);
        o[a][2] = __fmaf_rn(pa, v0.z, o[a][2]);
        o[a][3] = __fmaf_rn(pa, v0.w, o[a][3]);
        o[a][4] = __fmaf_rn(pa, v1.x, o[a][4]);
        o[a][5] = __fmaf_rn(pa, v1.y, o[a][5]);
        o[a][6] = __fmaf_rn(pa, v1.z, o[a][6]);
        o[a][7] = __fmaf_rn(pa, v1.w, o[a][7]);
      }
    }
    __syncthreads();  // the tile's buffers and probabilities are free again
  }

#pragma unroll
  for (int a = 0; a < A; ++a) {
    float l = l_run[a];
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, off));
    const int r = A * ty + a;
    if (r < qrows) {
      float* dst = out + (((size_t)b * T + q0 + r) * Hq + h) * kPfD;
      *reinterpret_cast<float4*>(dst + tx * 4) =
          make_float4(__fdiv_rn(o[a][0], l), __fdiv_rn(o[a][1], l), __fdiv_rn(o[a][2], l), __fdiv_rn(o[a][3], l));
      *reinterpret_cast<float4*>(dst + 64 + tx * 4) =
          make_float4(__fdiv_rn(o[a][4], l), __fdiv_rn(o[a][5], l), __fdiv_rn(o[a][6], l), __fdiv_rn(o[a][7], l));
    }
  }
}

cudaLaunchConfig_t pf_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cfg;
}

}  // namespace

cudaError_t launch_rope_kv_rows(const float* qkv, int batch, int t, int pos0, const float* cos_t, const float* sin_t,
                                float* kc, float* vc, int hq, int hkv, int d, int max_t, float* q_out, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (d % 8 == 0 && a16(qkv) && a16(cos_t) && a16(sin_t) && a16(kc) && a16(vc) && a16(q_out)) {
    cudaLaunchConfig_t cfg = pf_cfg(dim3((unsigned)(batch * t)), dim3(256), 0, s, attr);
    return cudaLaunchKernelEx(&cfg, rope_kv_rows_vec_kernel, qkv, t, pos0, cos_t, sin_t, kc, vc, hq, hkv, d, max_t,
                              q_out);
  }
  cudaLaunchConfig_t cfg = pf_cfg(dim3((unsigned)(batch * t), (unsigned)(hq + 2 * hkv)), dim3((unsigned)d), 0, s, attr);
  return cudaLaunchKernelEx(&cfg, rope_kv_rows_kernel, qkv, t, pos0, cos_t, sin_t, kc, vc, hq, hkv, d, max_t, q_out);
}

cudaError_t launch_add_rmsnorm(float* x, const float* y, const float* w, float eps, int64_t m, int64_t n, float* h,
                               cudaStream_t s) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (n % 4 == 0 && n <= kArMaxN && a16(x) && a16(y) && a16(w) && a16(h)) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pf_cfg(dim3((unsigned)m), dim3(kArThreads), 0, s, attr);
    return cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel, x, y, w, eps, (int)n, h);
  }
  cudaError_t e = launch_add(x, y, m * n, s);
  return e != cudaSuccess ? e : launch_rmsnorm(x, w, eps, m, n, h, s);
}

template <int A>
static cudaError_t launch_attention_prefill_a(const float* q, const float* kc, const float* vc, int batch, int t,
                                             int pos0, int hq, int hkv, int max_t, float* out, int device,
                                             cudaStream_t s) {
  static int configured[128] = {0};
  cudaError_t e =
      ensure_smem((const void*)attention_prefill_kernel<A>, configured, device, sizeof(PfSmem<A>), false);
  if (e != cudaSuccess) return e;
  constexpr int rows = PfSmem<A>::kRows;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pf_cfg(dim3((unsigned)((t + rows - 1) / rows), (unsigned)hq, (unsigned)batch),
                                  dim3(kPfThreads), sizeof(PfSmem<A>), s, attr);
  // candle's `scores / sqrt(width)` multiplies by the f32 rounding of 1/sqrt(width)
  const float scale = (float)(1.0 / std::sqrt(128.0));
  return cudaLaunchKernelEx(&cfg, attention_prefill_kernel<A>, q, kc, vc, t, pos0, hq, hkv, max_t, scale, out);
}

cudaError_t launch_attention_prefill(const float* q, const float* kc, const float* vc, int batch, int t, int pos0,
                                     int hq, int hkv, int max_t, float* out, int device, cudaStream_t s) {
  // measured on B200 (one sequence, 16 heads, us): 32-row tiles take T = 128 from 20.7 to
  // 15.7, but T = 512 from 70.4 to 84.5 and T = 1024 (GQA 16:2) from 210 to 242
  const int64_t ctas64 = (int64_t)((t + 63) / 64) * hq * batch;
  if (2 * ctas64 < (int64_t)sm_count(device))
    return launch_attention_prefill_a<2>(q, kc, vc, batch, t, pos0, hq, hkv, max_t, out, device, s);
  return launch_attention_prefill_a<4>(q, kc, vc, batch, t, pos0, hq, hkv, max_t, out, device, s);
}

}  // namespace q8lin
