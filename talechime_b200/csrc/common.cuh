// Device helpers shared by the Q8_0 kernels (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "talechime_b200 kernels target sm_100a only"
#endif

namespace q8lin {

constexpr int kQK = 32;          // values per Q8_0 block
constexpr int kBlockBytes = 34;  // GGUF block bytes
constexpr unsigned kFull = 0xffffffffu;

// Bytes of one repacked weight row: K int8 values, K/32 f16 scales, padded to 16 B.
__host__ __device__ inline int64_t packed_row_stride(int64_t k) {
  return k + (((k / 16) + 15) / 16) * 16;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  No-ops unless the launch set the attribute.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Streaming loads (read-only, no L1 allocation).
__device__ __forceinline__ int4 ld_stream_v4(const void* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Bulk prefetch of [p, p + bytes) into L2 (p and bytes multiples of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------
// Time-bounded waits.  %globaltimer counts nanoseconds; a spin in the kernels gives up
// once the host-set limit (q8lin_set_wait_limit_ns, passed as a kernel argument) has
// passed, or once another warp of the CTA raised the CTA's abort flag.  Waits for a
// CTA's own bulk copies before it exits use the fixed kDrainLimitNs instead, so that a
// tiny limit cannot leave copies in flight into released shared memory.
constexpr uint64_t kDrainLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mb_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

// Wait for the completion of the phase of `bar` with `parity`.  False when `limit_ns`
// passed first or *abort became non-zero (both checked every 16 polls).
__device__ __forceinline__ bool mb_wait_ns(uint32_t bar, uint32_t parity, uint64_t limit_ns,
                                           const volatile int* abort) {
  if (mb_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mb_try(bar, parity)) return true;
    if ((i & 15u) == 0u) {
      if (abort && *abort) return false;
      if (global_ns() - t0 > limit_ns) return false;
    }
  }
}

// 16-byte asynchronous copy global -> shared by the calling thread (L2 only), and its
// commit / wait groups.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// Weights are read once per call: an L2 evict-first policy keeps the streamed rows from
// pushing activations, outputs and caches out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void cp_async16_stream(uint32_t dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(policy)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// All but the newest `n` (0..3) of this thread's copy groups have landed.
__device__ __forceinline__ void cp_async_wait(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
  }
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ int dot16(const int4 a, const int4 b, int c) {
  c = __dp4a(a.x, b.x, c);
  c = __dp4a(a.y, b.y, c);
  c = __dp4a(a.z, b.z, c);
  c = __dp4a(a.w, b.w, c);
  return c;
}

// ---------------------------------------------------------------------------
// Candle's Q8_0 quantization of one value (BlockQ8_0::from_float):
// q = (i8) round_half_away(v * id), saturating, NaN -> 0.
__device__ __forceinline__ int quant_q8(float v, float id) {
  const float p = __fmul_rn(v, id);     // one rounding, never fused
  const float r = roundf(p);            // half away from zero
  int q = __float2int_rz(r);            // saturates; NaN -> 0
  q = max(-128, min(127, q));
  return q;
}

// Per-block quantization parameters: d = amax/127 (IEEE division),
// id = d != 0 ? 1/d : 0, d_f16 = RNE(d).
struct QParams {
  float id;
  __half d_h;
};
__device__ __forceinline__ QParams block_qparams(float amax) {
  QParams p;
  const float d = __fdiv_rn(amax, 127.0f);
  p.id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
  p.d_h = __float2half_rn(d);
  return p;
}

// f32 max that skips NaN (Rust f32::max / C fmaxf semantics).
__device__ __forceinline__ float nan_skip_max(float a, float b) { return fmaxf(a, b); }

// Quantize one 32-value block held as 8 float4 in registers into 8 packed int32.
__device__ __forceinline__ void quantize_block_regs(const float4 (&v)[8], int (&q)[8],
                                                    __half& d_h) {
  float amax = 0.0f;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    amax = nan_skip_max(amax, fabsf(v[t].x));
    amax = nan_skip_max(amax, fabsf(v[t].y));
    amax = nan_skip_max(amax, fabsf(v[t].z));
    amax = nan_skip_max(amax, fabsf(v[t].w));
  }
  const QParams p = block_qparams(amax);
  d_h = p.d_h;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int a = quant_q8(v[t].x, p.id);
    const int b = quant_q8(v[t].y, p.id);
    const int c = quant_q8(v[t].z, p.id);
    const int d = quant_q8(v[t].w, p.id);
    q[t] = (a & 0xff) | ((b & 0xff) << 8) | ((c & 0xff) << 16) | ((d & 0xff) << 24);
  }
}

// Octet-parallel quantization: the 32 values of one block are held by 8 consecutive
// lanes (lane & ~7 aligned), 4 values each.  Every lane of the warp must call this
// (the amax is combined with shuffles).  Returns the lane's 4 int8 packed in an int;
// d_h is the block's f16 scale (identical in the 8 lanes).
__device__ __forceinline__ int quantize_octet(const float4 v, __half& d_h) {
  float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 4));
  amax = fmaxf(amax, 0.0f);  // all-NaN block: candle's running max starts at 0
  const QParams p = block_qparams(amax);
  d_h = p.d_h;
  const int a = quant_q8(v.x, p.id);
  const int b = quant_q8(v.y, p.id);
  const int c = quant_q8(v.z, p.id);
  const int d = quant_q8(v.w, p.id);
  return (a & 0xff) | ((b & 0xff) << 8) | ((c & 0xff) << 16) | ((d & 0xff) << 24);
}

// candle's f32 silu(g) = g / (1 + exp(-g)), times u; each operation rounded (exp is
// CUDA's expf, within 2 ulp of exp).
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// M = 1 row dot products over one 2048-value segment of a repacked row ([int8 K |
// f16 d[K/32]]): lane l holds blocks b0 = 64 seg + l and b1 = b0 + 32 of the segment
// (32 int8 each, two 16-byte units); per block the term is ((f32(isum) * dw) * dx) with
// each product rounded (candle's scalar vec_dot), and the row sum is a tree over the
// lanes.  Two rows at a time share the activation registers.
struct XSeg {
  int4 a0, a1, b0, b1;  // quantized activations of blocks b0 and b1, halves in load order
  float da, db;         // their scales
  bool va, vb;          // blocks inside K
};

// A lane reads the two 16-byte halves of its 32-byte block in the order (lane ^ lane/4)
// & 1 first: within each group of 8 lanes (one shared-memory wavefront of 16-byte
// accesses) the 8 accesses then fall on 8 distinct 4-bank groups, where reading the
// low half first in every lane would put lanes l and l + 4 on the same banks.
__device__ __forceinline__ int half_order(int lane) { return (lane ^ (lane >> 2)) & 1; }

// The warp's activation segment from the quantized vector in shared memory (qx int8
// [K], dx f32 [K/32]; nb = K/32 blocks).
__device__ __forceinline__ XSeg load_xseg(const int8_t* qx, const float* dx, int nb, int seg) {
  const int lane = threadIdx.x & 31, b0 = seg * 64 + lane, b1 = b0 + 32;
  const int h = half_order(lane) * 16;
  XSeg xs;
  xs.va = b0 < nb;
  xs.vb = b1 < nb;
  const int4 z = make_int4(0, 0, 0, 0);
  xs.a0 = xs.va ? *reinterpret_cast<const int4*>(qx + (size_t)b0 * 32 + h) : z;
  xs.a1 = xs.va ? *reinterpret_cast<const int4*>(qx + (size_t)b0 * 32 + (16 - h)) : z;
  xs.b0 = xs.vb ? *reinterpret_cast<const int4*>(qx + (size_t)b1 * 32 + h) : z;
  xs.b1 = xs.vb ? *reinterpret_cast<const int4*>(qx + (size_t)b1 * 32 + (16 - h)) : z;
  xs.da = xs.va ? dx[b0] : 0.0f;
  xs.db = xs.vb ? dx[b1] : 0.0f;
  return xs;
}

// Block `blk` of a row against activations x0 / x1 held in the same half order.
__device__ __forceinline__ float block_term(const uint8_t* row, int K, int blk, const int4& x0, const int4& x1,
                                            float dxs) {
  const int h = half_order(threadIdx.x & 31) * 16;
  const int4 w0 = *reinterpret_cast<const int4*>(row + (size_t)blk * 32 + h);
  const int4 w1 = *reinterpret_cast<const int4*>(row + (size_t)blk * 32 + (16 - h));
  // two independent 4-deep dp4a chains (exact in int32 in any order)
  const int isum = dot16(w0, x0, 0) + dot16(w1, x1, 0);
  const float dw = __half2float(reinterpret_cast<const __half*>(row + K)[blk]);
  return __fmul_rn(__fmul_rn(__int2float_rn(isum), dw), dxs);
}

// This lane's share of segment `seg` of two rows: the sum of its two block terms.
__device__ __forceinline__ void seg_terms2(const uint8_t* wa, const uint8_t* wb, bool has_b, int K, int seg,
                                           const XSeg& xs, float& ta, float& tb) {
  const int lane = threadIdx.x & 31;
  const int b0 = seg * 64 + lane, b1 = b0 + 32;
  ta = 0.0f;
  tb = 0.0f;
  if (xs.va) {
    ta = block_term(wa, K, b0, xs.a0, xs.a1, xs.da);
    if (has_b) tb = block_term(wb, K, b0, xs.a0, xs.a1, xs.da);
  }
  if (xs.vb) {
    ta = __fadd_rn(ta, block_term(wa, K, b1, xs.b0, xs.b1, xs.db));
    if (has_b) tb = __fadd_rn(tb, block_term(wb, K, b1, xs.b0, xs.b1, xs.db));
  }
}

__device__ __forceinline__ void warp_sum2(float& ta, float& tb) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ta += __shfl_xor_sync(kFull, ta, o);
    tb += __shfl_xor_sync(kFull, tb, o);
  }
}

// Sum over the warp of v[m], m < MR, leaving in every lane the total of row mr_index(lane):
// at each of the first log2(MR) levels a lane keeps half of its values and adds the
// partner's copy of them, so MR rows cost MR - 1 + 5 - log2(MR) shuffles over 5 levels
// (one shuffle tree per row would cost 5 MR).
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

// The same arithmetic on rows addressed by their 32-bit shared-memory address, with
// explicit ld.shared loads (a row pointer built with run-time offsets from a dynamic
// shared array otherwise compiles to generic loads).
__device__ __forceinline__ int4 lds128(uint32_t a) {
  int4 v;
  asm volatile("ld.shared.v4.s32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float lds_half_f32(uint32_t a) {
  unsigned short h;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(a));
  return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ float block_term_s(uint32_t row, int K, int blk, const int4& x0, const int4& x1, float dxs) {
  const uint32_t h = (uint32_t)half_order(threadIdx.x & 31) * 16u;
  const uint32_t b = row + (uint32_t)blk * 32u;
  const int4 w0 = lds128(b + h);
  const int4 w1 = lds128(b + (16u - h));
  // two independent 4-deep dp4a chains (exact in int32 in any order)
  const int isum = dot16(w0, x0, 0) + dot16(w1, x1, 0);
  const float dw = lds_half_f32(row + (uint32_t)K + 2u * (uint32_t)blk);
  return __fmul_rn(__fmul_rn(__int2float_rn(isum), dw), dxs);
}
__device__ __forceinline__ float seg_terms1_s(uint32_t row, int K, int seg, const XSeg& xs) {
  const int lane = threadIdx.x & 31;
  const int b0 = seg * 64 + lane, b1 = b0 + 32;
  float t = 0.0f;
  if (xs.va) t = block_term_s(row, K, b0, xs.a0, xs.a1, xs.da);
  if (xs.vb) t = __fadd_rn(t, block_term_s(row, K, b1, xs.b0, xs.b1, xs.db));
  return t;
}
__device__ __forceinline__ void seg_terms2_s(uint32_t wa, uint32_t wb, bool has_b, int K, int seg, const XSeg& xs,
                                             float& ta, float& tb) {
  const int lane = threadIdx.x & 31;
  const int b0 = seg * 64 + lane, b1 = b0 + 32;
  ta = 0.0f;
  tb = 0.0f;
  if (xs.va) {
    ta = block_term_s(wa, K, b0, xs.a0, xs.a1, xs.da);
    if (has_b) tb = block_term_s(wb, K, b0, xs.a0, xs.a1, xs.da);
  }
  if (xs.vb) {
    ta = __fadd_rn(ta, block_term_s(wa, K, b1, xs.b0, xs.b1, xs.db));
    if (has_b) tb = __fadd_rn(tb, block_term_s(wb, K, b1, xs.b0, xs.b1, xs.db));
  }
}
// load_xseg from the quantized activations at shared addresses qx (int8 [K]) and dx
// (f32 [K/32]).
__device__ __forceinline__ XSeg load_xseg_s(uint32_t qx, uint32_t dx, int nb, int seg) {
  const int lane = threadIdx.x & 31, b0 = seg * 64 + lane, b1 = b0 + 32;
  const uint32_t h = (uint32_t)half_order(lane) * 16u;
  XSeg xs;
  xs.va = b0 < nb;
  xs.vb = b1 < nb;
  const int4 z = make_int4(0, 0, 0, 0);
  xs.a0 = xs.va ? lds128(qx + (uint32_t)b0 * 32u + h) : z;
  xs.a1 = xs.va ? lds128(qx + (uint32_t)b0 * 32u + (16u - h)) : z;
  xs.b0 = xs.vb ? lds128(qx + (uint32_t)b1 * 32u + h) : z;
  xs.b1 = xs.vb ? lds128(qx + (uint32_t)b1 * 32u + (16u - h)) : z;
  float da = 0.0f, db = 0.0f;
  if (xs.va) asm volatile("ld.shared.f32 %0, [%1];" : "=f"(da) : "r"(dx + 4u * (uint32_t)b0));
  if (xs.vb) asm volatile("ld.shared.f32 %0, [%1];" : "=f"(db) : "r"(dx + 4u * (uint32_t)b1));
  xs.da = da;
  xs.db = db;
  return xs;
}

// This lane's share of segment `seg` of one row: the sum of its two block terms (the
// same value seg_terms2 gives for either of its rows).
__device__ __forceinline__ float seg_terms1(const uint8_t* w, int K, int seg, const XSeg& xs) {
  const int lane = threadIdx.x & 31;
  const int b0 = seg * 64 + lane, b1 = b0 + 32;
  float t = 0.0f;
  if (xs.va) t = block_term(w, K, b0, xs.a0, xs.a1, xs.da);
  if (xs.vb) t = __fadd_rn(t, block_term(w, K, b1, xs.b0, xs.b1, xs.db));
  return t;
}

__device__ __forceinline__ void seg_dot2(const uint8_t* wa, const uint8_t* wb, bool has_b, int K, int seg,
                                         const XSeg& xs, float& sa, float& sb) {
  float ta, tb;
  seg_terms2(wa, wb, has_b, K, seg, xs, ta, tb);
  warp_sum2(ta, tb);
  sa = ta;
  sb = tb;
}

}  // namespace q8lin
