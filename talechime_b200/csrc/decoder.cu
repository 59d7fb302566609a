// Decode-step kernels around the Q8_0 linears of the VoxCPM BaseLM-style decoder
// (crates/voxcpm/src/transformer.rs:107-155 and attention.rs:28-98), batch 1, f32.
//
// A decode step reads the token and the position from device memory and the argmax
// writes the next token and advances the position, so one captured CUDA graph of a
// step replays for every token without the host.
//   * embed_rows: dequantize rows of a Q8_0 embedding held as a repacked weight;
//   * rmsnorm: y = x / sqrt(sum(x^2)/n + eps) * w (candle_nn::ops::rms_norm, eps from
//     transformer.rs:92), one CTA per row, tree-ordered sum;
//   * rope_kv: rotary embedding of q and k at the current position with the doubled
//     tables of transformer.rs:44-65 and rotate() :159-170 (x*[cos,cos] +
//     [second,first]*[-sin,sin], each product rounded), rotated q to a buffer, rotated
//     k and v appended to the f32 KV cache (the cat-growth of :131-139 preallocated);
//   * attention_decode: softmax(q k^T * (1/sqrt(d))) v over positions [0, pos] for every
//     query head, kv head = q head / (Hq/Hkv) (grouped heads, attention.rs:52-58),
//     split over position ranges with per-split (max, sum, weighted v) partials merged
//     by the last CTA of each head (deterministic, split order);
//   * add: x += y (residual); argmax: greedy next token (lowest index on ties), then
//     pos += 1.
// Every kernel takes part in programmatic dependent launch (waits before touching data
// an upstream kernel may write, releases dependents at the end).
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

constexpr int kAttnWarps = 4;
constexpr int kAttnPositions = 64;  // positions per attention CTA

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__global__ void embed_rows_kernel(const uint8_t* __restrict__ packed, int64_t S, int K, int vocab,
                                  const int* __restrict__ tokens, int n, float* __restrict__ out) {
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  const int r = blockIdx.x;
  if (r < n) {
    int tok = tokens[r];
    tok = tok < 0 ? 0 : (tok >= vocab ? vocab - 1 : tok);
    const uint8_t* row = packed + (size_t)tok * S;
    const __half* d = reinterpret_cast<const __half*>(row + K);
    for (int i = threadIdx.x; i < K; i += blockDim.x)
      out[(size_t)r * K + i] = __fmul_rn((float)(int8_t)row[i], __half2float(d[i >> 5]));
  }
}

__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps, int n,
                               float* __restrict__ y) {
  __shared__ float red[32];
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  const float* xr = x + (size_t)blockIdx.x * n;
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = __fadd_rn(s, __fmul_rn(xr[i], xr[i]));
  const float sum2 = block_sum(s, red);
  const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum2, (float)n), eps));
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    y[(size_t)blockIdx.x * n + i] = __fmul_rn(__fdiv_rn(xr[i], m), w[i]);
}

// qkv[(Hq + 2 Hkv) * D] of the current token; cos/sin [max_t][D/2]; caches [Hkv][max_t][D].
__global__ void rope_kv_kernel(const float* __restrict__ qkv, const int* __restrict__ pos_dev,
                               const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                               float* __restrict__ kc, float* __restrict__ vc, int Hq, int Hkv, int D, int max_t,
                               float* __restrict__ q_out) {
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  const int pos = *pos_dev;
  const int half = D / 2;
  const int head = blockIdx.x;  // 0..Hq+Hkv-1 rotated heads, then Hkv value heads
  const int i = threadIdx.x;
  if (i < D && pos >= 0 && pos < max_t) {
    if (head < Hq + Hkv) {
      const float* xh = qkv + (size_t)head * D;
      const int j = i < half ? i : i - half;
      const float c = cos_t[(size_t)pos * half + j];
      const float sn = sin_t[(size_t)pos * half + j];
      // x*[cos,cos] + [second,first]*[-sin,sin]
      const float r = i < half ? __fadd_rn(__fmul_rn(xh[i], c), __fmul_rn(xh[i + half], -sn))
                               : __fadd_rn(__fmul_rn(xh[i], c), __fmul_rn(xh[i - half], sn));
      if (head < Hq)
        q_out[(size_t)head * D + i] = r;
      else
        kc[((size_t)(head - Hq) * max_t + pos) * D + i] = r;
    } else if (head < Hq + 2 * Hkv) {
      const int hv = head - Hq - Hkv;
      vc[((size_t)hv * max_t + pos) * D + i] = qkv[(size_t)head * D + i];
    }
  }
}

// grid (Hq, splits); block kAttnWarps warps.  D = 128: four dims per lane.
// part: [Hq][splits][2 + D] (max, sum, acc[D]); cnt: [Hq] arrival counters (zero).
__global__ void __launch_bounds__(kAttnWarps * 32)
attention_decode_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                        const int* __restrict__ pos_dev, int Hq, int Hkv, int max_t, float scale,
                        float* __restrict__ part, unsigned int* __restrict__ cnt, float* __restrict__ out) {
  constexpr int D = 128;
  __shared__ float wm[kAttnWarps], wl[kAttnWarps];
  __shared__ float wacc[kAttnWarps][D];
  __shared__ int last;
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  const int h = blockIdx.x, split = blockIdx.y, splits = gridDim.y;
  const int hk = h / (Hq / Hkv);
  const int len = min(*pos_dev + 1, max_t);  // never past the cache
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float4 q4 = reinterpret_cast<const float4*>(q + (size_t)h * D)[lane];
  const float* kh = kc + (size_t)hk * max_t * D;
  const float* vh = vc + (size_t)hk * max_t * D;
  const int t0 = split * kAttnPositions, t1 = min(len, t0 + kAttnPositions);
  float m = -INFINITY, l = 0.0f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t = t0 + warp; t < t1; t += kAttnWarps) {
    const float4 k4 = reinterpret_cast<const float4*>(kh + (size_t)t * D)[lane];
    float s = __fmul_rn(q4.x, k4.x);
    s = __fadd_rn(s, __fmul_rn(q4.y, k4.y));
    s = __fadd_rn(s, __fmul_rn(q4.z, k4.z));
    s = __fadd_rn(s, __fmul_rn(q4.w, k4.w));
    s = __fmul_rn(warp_sum(s), scale);
    const float mn = fmaxf(m, s);
    const float corr = expf(m - mn);  // 0 on the first position (m = -inf)
    const float p = expf(s - mn);
    const float4 v4 = reinterpret_cast<const float4*>(vh + (size_t)t * D)[lane];
    l = __fadd_rn(__fmul_rn(l, corr), p);
    acc.x = __fadd_rn(__fmul_rn(acc.x, corr), __fmul_rn(p, v4.x));
    acc.y = __fadd_rn(__fmul_rn(acc.y, corr), __fmul_rn(p, v4.y));
    acc.z = __fadd_rn(__fmul_rn(acc.z, corr), __fmul_rn(p, v4.z));
    acc.w = __fadd_rn(__fmul_rn(acc.w, corr), __fmul_rn(p, v4.w));
    m = mn;
  }
  if (lane == 0) {
    wm[warp] = m;
    wl[warp] = l;
  }
  reinterpret_cast<float4*>(wacc[warp])[lane] = acc;
  __syncthreads();
  // merge the warps of the CTA (warp order), one thread per dimension
  float* mine = part + ((size_t)h * splits + split) * (2 + D);
  if (threadIdx.x < D) {
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w]);
    float L = 0.0f, A = 0.0f;
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = (wm[w] == -INFINITY) ? 0.0f : expf(wm[w] - M);
      L = __fadd_rn(L, __fmul_rn(wl[w], f));
      A = __fadd_rn(A, __fmul_rn(wacc[w][threadIdx.x], f));
    }
    mine[2 + threadIdx.x] = A;
    if (threadIdx.x == 0) {
      mine[0] = M;
      mine[1] = L;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(&cnt[h], 1u) == (unsigned)(splits - 1)) ? 1 : 0;
  __syncthreads();
  if (last) {
    __threadfence();
    const float* base = part + (size_t)h * splits * (2 + D);
    if (threadIdx.x < D) {
      float M = -INFINITY;
      for (int s = 0; s < splits; ++s) M = fmaxf(M, base[(size_t)s * (2 + D)]);
      float L = 0.0f, A = 0.0f;
      for (int s = 0; s < splits; ++s) {
        const float ms = base[(size_t)s * (2 + D)];
        const float f = (ms == -INFINITY) ? 0.0f : expf(ms - M);
        L = __fadd_rn(L, __fmul_rn(base[(size_t)s * (2 + D) + 1], f));
        A = __fadd_rn(A, __fmul_rn(base[(size_t)s * (2 + D) + 2 + threadIdx.x], f));
      }
      out[(size_t)h * D + threadIdx.x] = __fdiv_rn(A, L);
    }
    if (threadIdx.x == 0) cnt[h] = 0;
  }
}

// ---------------------------------------------------------------------------------
// RoPE + KV append + attention in one kernel (the decode step's attention block).
// grid (kRaCluster, Hq) with clusters of kRaCluster CTAs: cluster h serves q head h and
// its CTAs split the positions [0, pos] evenly (rank r takes [r*per, (r+1)*per) with
// per = ceil((pos + 1) / kRaCluster)), so the work per CTA follows the current length.
// A CTA:
//   * rotates q of its head and, if its range holds the current position, k and v of
//     the current token straight from the qkv projection (no CTA reads a cache row that
//     another CTA of this launch writes); the first q head of each kv head appends k
//     and v to the cache;
//   * streams its cached K and V rows through a two-slot shared-memory ring of
//     kRaChunk-row chunks (cp.async.bulk from this GPU's memory, mbarrier complete_tx),
//     the copy of chunk c + 2 issued as soon as chunk c is consumed;
//   * per chunk: each warp takes 4 positions and keeps its own online softmax (running
//     max and sum, and the weighted V sum of each lane's 4 dimensions); one barrier per
//     chunk frees the slot; after the last chunk the 8 warps are merged in warp order;
//   * publishes its (max, sum, acc[128]) in shared memory; after a cluster barrier CTA
//     rank 0 reads the partials of the cluster through distributed shared memory, merges
//     them in rank order and writes the output; a second barrier keeps every CTA's
//     shared memory alive until then.
constexpr int kRaCluster = 8;
constexpr int kRaChunk = 32;
constexpr int kRaThreads = 256;

__device__ unsigned int g_attn_fault;

struct RaSmem {
  alignas(16) float k[2][kRaChunk][128];
  alignas(16) float v[2][kRaChunk][128];
  alignas(16) float q[128];
  alignas(16) float kcur[128];
  alignas(16) float vcur[128];
  alignas(16) float pacc[128];  // this CTA's partial: weighted V sum
  alignas(16) float wacc[kRaThreads / 32][128];  // each warp's weighted V sum
  float wm[kRaThreads / 32], wl[kRaThreads / 32];  // each warp's running max and sum
  float stat[4];  // [3]: this CTA's partial max
  float pl;       // partial sum
  alignas(8) uint64_t full[2];
};

// This CTA's wait limit (the kernel's wait_ns argument, set by thread 0 at entry).
__shared__ uint64_t s_ra_wait_ns;

// Bounded wait for this CTA's own bulk copies (false once the limit has passed).
__device__ __forceinline__ bool ra_wait(uint64_t* bar, uint32_t parity) {
  return mb_wait_ns((uint32_t)__cvta_generic_to_shared(bar), parity, s_ra_wait_ns, nullptr);
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kRaThreads)
rope_attention_kernel(const float* __restrict__ qkv, const int* __restrict__ pos_dev, const float* __restrict__ cos_t,
                      const float* __restrict__ sin_t, float* __restrict__ kc, float* __restrict__ vc, int Hq, int Hkv,
                      int max_t, float scale, float* __restrict__ out, int pos_ready, uint64_t wait_ns) {
  constexpr int D = 128, half = 64;
  extern __shared__ __align__(16) uint8_t ra_raw[];
  RaSmem& sm = *reinterpret_cast<RaSmem*>(ra_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.y;
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int group = Hq / Hkv, hk = h / group;
  if (tid == 0) {
    s_ra_wait_ns = wait_ns;
    for (int i = 0; i < 2; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(&sm.full[i])),
                   "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // pos_ready: the position and the cache rows below it were written before the
  // preceding launch began (the decoder's step: the argmax of the previous token is
  // followed by the embedding kernel, whose dependency wait comes before its trigger), so
  // they are read and the first K/V chunks are copied before this launch's dependency
  // wait, overlapping the qkv projection's tail
  if (!pos_ready) {
    pdl_wait();
    // the next linear's CTAs may become resident and fill their weight rings meanwhile
    // (its own dependency wait still covers this grid's writes)
    pdl_launch_dependents();
  }
  const int pos = *pos_dev;
  const int len = pos < 0 ? 0 : min(pos + 1, max_t);  // never past the cache
  const int per = (len + kRaCluster - 1) / kRaCluster;
  const int a = min(len, (int)rank * per), b = min(len, a + per);
  const int nchunks = (b - a + kRaChunk - 1) / kRaChunk;
  const bool cur = a <= pos && pos < b;
  const float* kh = kc + (size_t)hk * max_t * D;
  const float* vh = vc + (size_t)hk * max_t * D;
  // chunk c holds positions [a + c*kRaChunk, ...); its cached rows are those below pos
  auto issue = [&](int c) {
    const int c0 = a + c * kRaChunk, c1 = min(b, c0 + kRaChunk), cached = min(c1, pos) - c0;
    const int slot = c & 1;
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&sm.full[slot]);
    const uint32_t bytes = cached > 0 ? (uint32_t)cached * D * 4 : 0u;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(2 * bytes) : "memory");
    if (bytes) {
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   ::"r"((uint32_t)__cvta_generic_to_shared(&sm.k[slot][0][0])), "l"(kh + (size_t)c0 * D),
                   "r"(bytes), "r"(bar) : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   ::"r"((uint32_t)__cvta_generic_to_shared(&sm.v[slot][0][0])), "l"(vh + (size_t)c0 * D),
                   "r"(bytes), "r"(bar) : "memory");
    }
  };
  __syncthreads();  // barrier init visible before any wait
  if (tid == 0)
    for (int c = 0; c < min(2, nchunks); ++c) issue(c);
  if (pos_ready) {  // qkv comes from the preceding launch
    pdl_wait();
    pdl_launch_dependents();
  }
  // rotation x*[cos,cos] + [second,first]*[-sin,sin] at the current position
  if (tid < D && pos >= 0 && pos < max_t) {
    const int j = tid < half ? tid : tid - half;
    const float c = cos_t[(size_t)pos * half + j], sn = sin_t[(size_t)pos * half + j];
    auto rot = [&](const float* xh) {
      return tid < half ? __fadd_rn(__fmul_rn(xh[tid], c), __fmul_rn(xh[tid + half], -sn))
                        : __fadd_rn(__fmul_rn(xh[tid], c), __fmul_rn(xh[tid - half], sn));
    };
    sm.q[tid] = rot(qkv + (size_t)h * D);
    if (cur) {
      const float kr = rot(qkv + (size_t)(Hq + hk) * D);
      const float vr = qkv[(size_t)(Hq + Hkv + hk) * D + tid];
      sm.kcur[tid] = kr;
      sm.vcur[tid] = vr;
      if (h % group == 0) {  // one writer per kv head
        kc[((size_t)hk * max_t + pos) * D + tid] = kr;
        vc[((size_t)hk * max_t + pos) * D + tid] = vr;
      }
    }
  }
  __syncthreads();
  // Warp w owns positions 4w .. 4w+3 of every chunk and keeps its own online softmax: a
  // running max m and sum l (the same in every lane) and the weighted V sum of the
  // lane's four dimensions; the warps are merged once, after the last chunk.
  const float4 q4 = reinterpret_cast<const float4*>(sm.q)[lane];
  float m = -INFINITY, l = 0.0f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  bool ok = true;
  for (int c = 0; c < nchunks; ++c) {
    const int slot = c & 1, c0 = a + c * kRaChunk, n = min(b - c0, kRaChunk);
    if (!ra_wait(&sm.full[slot], (uint32_t)((c >> 1) & 1))) ok = false;
    float s[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = warp * 4 + u;
      const float* krow = (c0 + j == pos) ? sm.kcur : sm.k[slot][j];
      const float4 k4 = reinterpret_cast<const float4*>(krow)[lane];
      float t = __fmul_rn(q4.x, k4.x);
      t = __fadd_rn(t, __fmul_rn(q4.y, k4.y));
      t = __fadd_rn(t, __fmul_rn(q4.z, k4.z));
      s[u] = __fadd_rn(t, __fmul_rn(q4.w, k4.w));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) s[u] += __shfl_xor_sync(kFull, s[u], o);
    float mx = -INFINITY;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      s[u] = (warp * 4 + u < n) ? __fmul_rn(s[u], scale) : -INFINITY;
      mx = fmaxf(mx, s[u]);
    }
    if (mx != -INFINITY) {  // a warp with no position in this chunk keeps its state
      const float mn = fmaxf(m, mx);
      const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
      float ps = 0.0f;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = warp * 4 + u;
        const float p = (s[u] == -INFINITY) ? 0.0f : expf(s[u] - mn);
        if (p != 0.0f) {
          const float* vrow = (c0 + j == pos) ? sm.vcur : sm.v[slot][j];
          const float4 v4 = reinterpret_cast<const float4*>(vrow)[lane];
          t.x = __fadd_rn(t.x, __fmul_rn(p, v4.x));
          t.y = __fadd_rn(t.y, __fmul_rn(p, v4.y));
          t.z = __fadd_rn(t.z, __fmul_rn(p, v4.z));
          t.w = __fadd_rn(t.w, __fmul_rn(p, v4.w));
        }
        ps = __fadd_rn(ps, p);
      }
      l = __fadd_rn(__fmul_rn(l, corr), ps);
      acc.x = __fadd_rn(__fmul_rn(acc.x, corr), t.x);
      acc.y = __fadd_rn(__fmul_rn(acc.y, corr), t.y);
      acc.z = __fadd_rn(__fmul_rn(acc.z, corr), t.z);
      acc.w = __fadd_rn(__fmul_rn(acc.w, corr), t.w);
      m = mn;
    }
    __syncthreads();  // every warp is done with the slot
    if (tid == 0 && c + 2 < nchunks) issue(c + 2);
  }
  if (!ok && tid == 0) atomicOr(&g_attn_fault, 8u);
  if (lane == 0) {
    sm.wm[warp] = m;
    sm.wl[warp] = l;
  }
  reinterpret_cast<float4*>(sm.wacc[warp])[lane] = acc;
  __syncthreads();
  // this CTA's partial: the warps merged in warp order
  if (tid < D) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kRaThreads / 32; ++w) M = fmaxf(M, sm.wm[w]);
    float L = 0.0f, A = 0.0f;
#pragma unroll
    for (int w = 0; w < kRaThreads / 32; ++w) {
      const float f = (sm.wm[w] == -INFINITY) ? 0.0f : expf(sm.wm[w] - M);
      L = __fadd_rn(L, __fmul_rn(sm.wl[w], f));
      A = __fadd_rn(A, __fmul_rn(sm.wacc[w][tid], f));
    }
    sm.pacc[tid] = A;
    if (tid == 0) {
      sm.stat[3] = M;
      sm.pl = L;
    }
  }
  cluster_sync();  // partials of every CTA of the cluster written
  if (rank == 0 && tid < D) {
    float mr[kRaCluster], lr[kRaCluster], ar[kRaCluster];
    const uint32_t base_m = (uint32_t)__cvta_generic_to_shared(&sm.stat[3]);
    const uint32_t base_l = (uint32_t)__cvta_generic_to_shared(&sm.pl);
    const uint32_t base_a = (uint32_t)__cvta_generic_to_shared(&sm.pacc[tid]);
#pragma unroll
    for (int r = 0; r < kRaCluster; ++r) {
      uint32_t am, al, aa;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(am) : "r"(base_m), "r"(r));
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(al) : "r"(base_l), "r"(r));
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(aa) : "r"(base_a), "r"(r));
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(mr[r]) : "r"(am) : "memory");
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(lr[r]) : "r"(al) : "memory");
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(ar[r]) : "r"(aa) : "memory");
    }
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kRaCluster; ++r) M = fmaxf(M, mr[r]);
    float L = 0.0f, A = 0.0f;
#pragma unroll
    for (int r = 0; r < kRaCluster; ++r) {
      const float f = (mr[r] == -INFINITY) ? 0.0f : expf(mr[r] - M);
      L = __fadd_rn(L, __fmul_rn(lr[r], f));
      A = __fadd_rn(A, __fmul_rn(ar[r], f));
    }
    out[(size_t)h * D + tid] = len > 0 ? __fdiv_rn(A, L) : 0.0f;
  }
  cluster_sync();  // rank 0 has read every partial: shared memory may be released
}

__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t n) {
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __fadd_rn(x[i], y[i]);
}

// Greedy argmax: per-CTA (value, index) partials, the last CTA reduces them (lowest
// index among equal maxima; NaN compares as smaller), writes the token and advances pos.
__global__ void argmax_kernel(const float* __restrict__ logits, int n, float* __restrict__ pv, int* __restrict__ pi,
                              unsigned int* __restrict__ cnt, int* __restrict__ token, int* __restrict__ pos_dev) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ int last;
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  float bv = -INFINITY;
  int bi = n;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float v = logits[i];
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(kFull, bv, o);
    const int oi = __shfl_xor_sync(kFull, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
    pv[blockIdx.x] = bv;
    pi[blockIdx.x] = bi;
    __threadfence();
    last = (atomicAdd(cnt, 1u) == gridDim.x - 1) ? 1 : 0;
  }
  __syncthreads();
  if (last) {
    // the last CTA reduces the per-CTA partials with all of its threads (same order
    // rule: larger value, then lower index)
    __threadfence();
    float v = -INFINITY;
    int ix = n;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
      const float pvb = __ldcg(pv + b);
      const int pib = __ldcg(pi + b);
      if (pvb > v || (pvb == v && pib < ix)) { v = pvb; ix = pib; }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(kFull, v, o);
      const int oi = __shfl_xor_sync(kFull, ix, o);
      if (ov > v || (ov == v && oi < ix)) { v = ov; ix = oi; }
    }
    __syncthreads();  // every thread has read sv / si of the first phase
    if (lane == 0) { sv[warp] = v; si[warp] = ix; }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (sv[w] > v || (sv[w] == v && si[w] < ix)) { v = sv[w]; ix = si[w]; }
      *token = ix < n ? ix : 0;
      if (pos_dev) *pos_dev += 1;
      *cnt = 0;
    }
  }
}

cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, cudaStream_t s, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cfg;
}

}  // namespace

cudaError_t launch_embed_rows(const q8lin_weight& w, const int* tokens, int n, float* out, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3((unsigned)n), dim3(256), s, attr);
  return cudaLaunchKernelEx(&cfg, embed_rows_kernel, (const uint8_t*)w.packed, w.row_stride, (int)w.k, (int)w.n,
                            tokens, n, out);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int64_t m, int64_t n, float* y,
                           cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3((unsigned)m), dim3(256), s, attr);
  return cudaLaunchKernelEx(&cfg, rmsnorm_kernel, x, w, eps, (int)n, y);
}

cudaError_t launch_rope_kv(const float* qkv, const int* pos, const float* cos_t, const float* sin_t, float* kc,
                           float* vc, int hq, int hkv, int d, int max_t, float* q_out, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3((unsigned)(hq + 2 * hkv)), dim3((unsigned)d), s, attr);
  return cudaLaunchKernelEx(&cfg, rope_kv_kernel, qkv, pos, cos_t, sin_t, kc, vc, hq, hkv, d, max_t, q_out);
}

size_t attention_workspace_bytes(int hq, int max_t) {
  const int splits = (max_t + kAttnPositions - 1) / kAttnPositions;
  return ((size_t)hq * splits * (2 + 128) * 4 + 255) / 256 * 256 + ((size_t)hq * 4 + 255) / 256 * 256;
}

cudaError_t launch_attention_decode(const float* q, const float* kc, const float* vc, const int* pos, int hq,
                                    int hkv, int max_t, void* ws, float* out, cudaStream_t s) {
  const int splits = (max_t + kAttnPositions - 1) / kAttnPositions;
  float* part = static_cast<float*>(ws);
  unsigned int* cnt = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(ws) +
                                                      ((size_t)hq * splits * (2 + 128) * 4 + 255) / 256 * 256);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3((unsigned)hq, (unsigned)splits), dim3(kAttnWarps * 32), s, attr);
  // candle's `scores / sqrt(width)` multiplies by the f32 rounding of 1/sqrt(width)
  const float scale = (float)(1.0 / std::sqrt(128.0));
  return cudaLaunchKernelEx(&cfg, attention_decode_kernel, q, kc, vc, pos, hq, hkv, max_t, scale, part, cnt, out);
}

cudaError_t launch_rope_attention(const float* qkv, const int* pos, const float* cos_t, const float* sin_t, float* kc,
                                  float* vc, int hq, int hkv, int max_t, float* out, int device, cudaStream_t s,
                                  bool pos_ready) {
  static int configured[128] = {0};
  cudaError_t e0 = ensure_smem((const void*)rope_attention_kernel, configured, device, sizeof(RaSmem), false);
  if (e0 != cudaSuccess) return e0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kRaCluster, (unsigned)hq);
  cfg.blockDim = dim3(kRaThreads);
  cfg.dynamicSmemBytes = sizeof(RaSmem);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kRaCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  const float scale = (float)(1.0 / std::sqrt(128.0));
  return cudaLaunchKernelEx(&cfg, rope_attention_kernel, qkv, pos, cos_t, sin_t, kc, vc, hq, hkv, max_t, scale, out,
                            pos_ready ? 1 : 0, wait_limit_ns());
}

cudaError_t read_attention_fault(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_attn_fault, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_attn_fault, &z, sizeof(z));
  }
  return e;
}

cudaError_t launch_add(float* x, const float* y, int64_t n, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3((unsigned)((n + 255) / 256)), dim3(256), s, attr);
  return cudaLaunchKernelEx(&cfg, add_kernel, x, y, n);
}

size_t argmax_workspace_bytes() { return 1024 * 8 + 256; }

cudaError_t launch_argmax(const float* logits, int n, void* ws, int* token, int* pos, cudaStream_t s) {
  const int ctas = 296;
  float* pv = static_cast<float*>(ws);
  int* pi = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) + 1024 * 4);
  unsigned int* cnt = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(ws) + 1024 * 8);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(ctas), dim3(256), s, attr);
  return cudaLaunchKernelEx(&cfg, argmax_kernel, logits, n, pv, pi, cnt, token, pos);
}

}  // namespace q8lin
