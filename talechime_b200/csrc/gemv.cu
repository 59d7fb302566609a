// Decode GEMV for 1 <= M <= 16: y[M][N] = Q8_0(x)[M][K] . W^T.
//
// HBM-bound: every launch streams the whole repacked weight (N*K*34/32 bytes) once.
// Two kernels:
//   * M = 1 and K <= 8192: gemv_q8_0_stream_kernel (below), one CTA per SM whose warps
//     stream their rows through private shared-memory rings (cp.async), sized so the
//     next linear's CTA is co-resident and prefetches its weights while this one runs;
//   * otherwise gemv_q8_0_kernel: two 512-thread CTAs per SM; CTA c owns the contiguous
//     weight rows [N*c/G, N*(c+1)/G), its warps take those rows round-robin, and the 32
//     lanes of a warp stride a row in 16-byte chunks (chunk c = half of block c/2) with
//     128-bit streaming loads, four chunks in flight per lane and the next batch issued
//     before the current one is reduced.
//
// Dependent-launch structure of gemv_q8_0_kernel (launched with programmatic stream
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
#include <type_traits>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>

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

// ---------------------------------------------------------------------------------
// M = 1 streaming GEMV with cross-launch weight prefetch: every warp streams its own rows
// through a private shared-memory ring with 16-byte cp.async copies.
//
// Geometry (host: stream_geometry): one CTA per SM owning the contiguous rows [r0, r1),
// 16 warps of which the first `nw` have a ring of `depth` slots; a slot holds `rps`
// consecutive rows (one contiguous byte range of the packed plane).  Slot j of the CTA
// belongs to warp j % nw.  At most 64 registers per thread and ~105 KB of shared memory,
// so two CTAs fit on an SM: the CTA of the next linear in the stream is resident while
// this one runs and fetches its first slots meanwhile.
//
// Why per-warp cp.async: measured on B200, 1-D bulk copies (cp.async.bulk) of one CTA
// complete one after another (~0.35 us each whatever the number in flight: 2 KB copies
// stream at 0.86 TB/s, 8 KB ones at 3.4 TB/s), while 16-byte cp.async copies issued by
// the warps themselves reach 6.9-7.1 TB/s with 16-48 KB in flight per SM.  A warp waits
// for its own copies (cp.async.wait_group) and consumes its slots in order, so the kernel
// has no spin wait and no mbarrier.  (The earlier shared ring, where every warp waited
// on an mbarrier parity only for the chunks holding its rows, let a warp reach the next
// use of a slot before the current use's copy had landed -- the parity test then passes
// at once; private rings consumed in order cannot do that.)
//
// Order of events:
//   1. launch_dependents at once: the next linear's CTAs may become resident and start
//      their own copies while this one computes;
//   2. warps with a ring issue their first `depth` slots -- weights are constant, so this
//      happens before the dependency wait and overlaps the previous linear;
//   3. all 16 warps: griddepcontrol.wait, the optional prologue (rms_norm, SwiGLU), x
//      quantized to Q8_0 in shared memory; warps without a ring leave;
//   4. a ring warp, per slot: wait for its copies, dot products two rows at a time
//      (K <= 2048: x held in registers; longer rows read their 2048-value segments of x
//      from shared memory), refill the slot with the warp's slot `depth` further on, and
//      the lane of each row writes it (+ residual).
// Each block term is ((f32(isum) * dw) * dx) rounded per product as candle's scalar
// vec_dot; sums across blocks are trees, so outputs agree within f32 summation
// tolerance.  The cross-GPU tail's wait for the peers is bounded in time
// (q8lin_set_wait_limit_ns): when it runs out, bit 1 of the fault word is set and the
// CTA's rows are written as NaN.
constexpr int kStreamWarps = 16;
constexpr int kStreamThreads = kStreamWarps * 32;
constexpr int kRingBytes = 96 * 1024;
constexpr int kSlotTargetBytes = 4352;  // two rows of K = 2048
constexpr int kMaxRps = 16;
constexpr int kMaxDepth = 4;
constexpr int kSegValues = 2048;  // x values per warp segment (64 blocks, two per lane)
constexpr int kStreamMaxK = 8192;  // x preparation: four float4 passes of 512 threads

__device__ unsigned int g_gemv_fault;

__host__ __device__ constexpr int64_t round16(int64_t v) { return (v + 15) / 16 * 16; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

struct StreamGeo {
  int rps = 0;         // rows per slot
  int nw = 0;          // warps with a ring
  int depth = 0;       // slots per ring
  int slot_bytes = 0;  // rps * S
};

// kAllreduce: the cross-GPU sum tail (fz.ar_world > 1) is compiled only into its own
// instantiation, so the single-GPU kernel keeps its registers.  kXReg: K <= 2048, the
// warp's x segment lives in registers.
template <bool kAllreduce, bool kXReg>
__global__ void __launch_bounds__(kStreamThreads, 2)
gemv_q8_0_stream_kernel(const uint8_t* __restrict__ W, int64_t S, int N, int K, const float* __restrict__ x,
                        float* __restrict__ y, const StreamGeo geo, const GemvFusion fz, uint64_t wait_ns) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[kStreamWarps];
  const int nb = K >> 5;
  const int r0 = (int)(((int64_t)N * blockIdx.x) / gridDim.x);
  const int r1 = (int)(((int64_t)N * (blockIdx.x + 1)) / gridDim.x);
  const int nrows = r1 - r0;
  const int rps = geo.rps, nw = geo.nw, depth = geo.depth;
  const int nslots = (nrows + rps - 1) / rps;
  // [rings: nw x depth slots | qx: K int8 | dx: nb f32]
  int8_t* qx = reinterpret_cast<int8_t*>(smem + (size_t)nw * depth * geo.slot_bytes);
  float* dx = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(qx) + round16(K));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + (size_t)warp * depth * geo.slot_bytes;  // this warp's ring (warp < nw)

  pdl_launch_dependents();

  // the warp's t-th slot (CTA slot warp + t * nw) into ring position t % depth; one copy
  // group per slot, empty when the warp has no such slot
  const uint64_t l2pol = l2_evict_first_policy();
  auto issue = [&](int t) {
    const int j = warp + t * nw;
    if (j < nslots) {
      const int row = j * rps;
      const int units = (min(rps, nrows - row) * (int)S) >> 4;
      const uint8_t* src = W + (size_t)(r0 + row) * S;
      const uint32_t dst = smem_u32(ring + (size_t)(t % depth) * geo.slot_bytes);
      for (int u = lane; u < units; u += 32) cp_async16_stream(dst + 16u * u, src + 16 * (size_t)u, l2pol);
    }
    cp_async_commit();
  };
  if (warp < nw)
    for (int t = 0; t < depth; ++t) issue(t);

  // Where the prefetched slots (the first `depth` of every ring) hold all of the CTA's
  // rows ("all" mode), every warp takes a share of them once the activations are ready;
  // their shared addresses are tabulated here, before the dependency wait.  Where more
  // rows follow ("own" mode), each ring warp streams its own slots through its ring.
  const int pre_slots = min(nslots, nw * depth);
  const int p1_rows = min(nrows, pre_slots * rps);
  const int p1_cap = nw * depth * rps;
  const bool own = nslots > nw * depth;
  const int nseg = (K + kSegValues - 1) / kSegValues;
  float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(dx) + round16(4 * nb));  // [nseg][p1_rows]
  uint32_t* rowaddr = reinterpret_cast<uint32_t*>(part + (nseg > 1 ? nseg * p1_cap : 0));
  const uint32_t smem_s = smem_u32(smem);
  if (!own) {
    for (int rr = threadIdx.x; rr < p1_rows; rr += kStreamThreads) {
      const int j = rr / rps;
      rowaddr[rr] = smem_s + (uint32_t)(((j % nw) * depth + j / nw) * geo.slot_bytes + (rr - j * rps) * (int)S);
    }
  }

  // ---------------- x -> Q8_0 in shared memory (all 16 warps) ----------------
  {
    // float4 pieces of x, 8 lanes per block; the loads of up to four passes are issued
    // together so K <= 8192 costs one L2 round trip
    constexpr int kT = kStreamThreads;
    constexpr int kQG = (kStreamMaxK / 4 + kT - 1) / kT;
    const int nquads = nb * 8;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4 v[kQG], wn[kQG];
    if (fz.prologue == kPrologueRmsNorm) {  // the norm weight is constant: load it before the wait
      const float4* w4 = reinterpret_cast<const float4*>(fz.norm_w);
#pragma unroll
      for (int g = 0; g < kQG; ++g) {
        const int i = g * kT + threadIdx.x;
        wn[g] = i < nquads ? __ldg(w4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    pdl_wait();
    if (fz.prologue == kPrologueSwiGLU) {
      // x = [gate | up], K values each: the activation is silu(gate) * up
#pragma unroll
      for (int g = 0; g < kQG; ++g) {
        const int i = g * kT + threadIdx.x;
        if (i < nquads) {
          const float4 ga = __ldg(x4 + i), ua = __ldg(x4 + nquads + i);
          v[g] = make_float4(silu_mul(ga.x, ua.x), silu_mul(ga.y, ua.y), silu_mul(ga.z, ua.z), silu_mul(ga.w, ua.w));
        } else {
          v[g] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    } else {
#pragma unroll
      for (int g = 0; g < kQG; ++g) {
        const int i = g * kT + threadIdx.x;
        v[g] = i < nquads ? __ldg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (fz.prologue == kPrologueRmsNorm) {
      // rms_norm over the row: sum of squares across the warps (tree order),
      // m = sqrt(sum/K + eps), x -> (x / m) * w
      float sq = 0.0f;
#pragma unroll
      for (int g = 0; g < kQG; ++g) {
        sq = __fadd_rn(sq, __fmul_rn(v[g].x, v[g].x));
        sq = __fadd_rn(sq, __fmul_rn(v[g].y, v[g].y));
        sq = __fadd_rn(sq, __fmul_rn(v[g].z, v[g].z));
        sq = __fadd_rn(sq, __fmul_rn(v[g].w, v[g].w));
      }
      sq = warp_sum(sq);
      if (lane == 0) red[warp] = sq;
      __syncthreads();
      float total = 0.0f;
#pragma unroll
      for (int i = 0; i < kStreamWarps; ++i) total += red[i];
      const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)K), fz.eps));
#pragma unroll
      for (int g = 0; g < kQG; ++g) {
        const int i = g * kT + threadIdx.x;
        if (i < nquads) {
          const float4 wv = wn[g];
          v[g] = make_float4(__fmul_rn(__fdiv_rn(v[g].x, m), wv.x), __fmul_rn(__fdiv_rn(v[g].y, m), wv.y),
                             __fmul_rn(__fdiv_rn(v[g].z, m), wv.z), __fmul_rn(__fdiv_rn(v[g].w, m), wv.w));
        }
      }
    }
#pragma unroll
    for (int g = 0; g < kQG; ++g) {
      if (g * kT < nquads) {  // uniform across the CTA: every lane shuffles
        const int i = g * kT + threadIdx.x;
        __half dh;
        const int q = quantize_octet(v[g], dh);
        if (i < nquads) {
          reinterpret_cast<int*>(qx)[i] = q;
          if ((i & 7) == 0) dx[i >> 3] = __half2float(dh);
        }
      }
    }
  }
  // the slots issued before the dependency wait are complete for every warp after this
  // barrier (they were issued long before; the wait only matters for a first launch)
  if (warp < nw) cp_async_wait(0);
  __syncthreads();

  // ---------------- rows ----------------
  const uint32_t qx_s = smem_u32(qx), dx_s = smem_u32(dx);
  XSeg xs;
  if constexpr (kXReg) xs = load_xseg_s(qx_s, dx_s, nb, 0);
  // row value `v` of CTA row `rr`: written to y (+ residual), or (cross-GPU sum) staged on
  // every rank.  A row is emitted by exactly one thread, which reads its residual first
  // (the residual may alias y).
  auto emit = [&](int rr, float v) {
    if constexpr (kAllreduce) {
      // the value and this call's epoch in one 64-bit word, one relaxed system-scope store
      // per rank: a reader that sees the epoch sees the value
      const size_t at = ((size_t)(fz.ar_epoch & 1u) * fz.ar_world + fz.ar_rank) * N + r0 + rr;
      const unsigned long long word = ((unsigned long long)fz.ar_epoch << 32) | __float_as_uint(v);
      for (int p = 0; p < fz.ar_world; ++p)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(fz.ar_stage[p] + at), "l"(word) : "memory");
    } else {
      y[r0 + rr] = fz.residual ? __fadd_rn(fz.residual[r0 + rr], v) : v;
    }
  };

  // Phase 1, all mode: items of R rows x one 2048-value segment over the 16 warps (R = 4,
  // 2 or 1, the largest that still gives every warp about one item); each lane sums its
  // two block terms per row and one transposing reduction gives the R row sums.
  // Segment sums of longer rows are added in segment order through shared memory.
  auto all_items = [&](auto rtag) {
    constexpr int R = decltype(rtag)::value;
    const int nitems = ((p1_rows + R - 1) / R) * nseg;
    for (int it = warp; it < nitems; it += kStreamWarps) {
      const int grp = nseg == 1 ? it : it / nseg;
      const int sg = it - grp * nseg, rb = grp * R;
      const int nr = min(R, p1_rows - rb);
      XSeg xsg;
      if constexpr (kXReg) xsg = xs;
      else xsg = load_xseg_s(qx_s, dx_s, nb, sg);
      uint32_t ra[R];
#pragma unroll
      for (int q = 0; q < R; ++q) ra[q] = rowaddr[q < nr ? rb + q : rb];
      float v[R];
#pragma unroll
      for (int q = 0; q < R; ++q) v[q] = q < nr ? seg_terms1_s(ra[q], K, sg, xsg) : 0.0f;
      const float tot = transpose_reduce<R>(v, lane);
      const int q = mr_index<R>(lane);
      if ((lane & (32 / R - 1)) == 0 && q < nr) {  // one lane per row
        if (nseg == 1) emit(rb + q, tot);
        else part[sg * p1_rows + rb + q] = tot;
      }
    }
  };

  if (!own) {
    const int rowsegs = p1_rows * nseg;
    if (rowsegs > 2 * kStreamWarps) all_items(std::integral_constant<int, 4>{});
    else if (rowsegs > kStreamWarps) all_items(std::integral_constant<int, 2>{});
    else all_items(std::integral_constant<int, 1>{});
    if (nseg > 1) {
      __syncthreads();  // every segment sum is in shared memory
      for (int rr = threadIdx.x; rr < p1_rows; rr += kStreamThreads) {
        float v = part[rr];
        for (int sg = 1; sg < nseg; ++sg) v = __fadd_rn(v, part[sg * p1_rows + rr]);
        emit(rr, v);
      }
    }
  } else if (warp < nw) {
    // Own mode: this warp's slots stream through its private ring and are consumed in
    // order, each slot refilled with the warp's slot `depth` further on as soon as it is
    // done (the first `depth` were prefetched before the dependency wait).
    const uint32_t ring_s = smem_u32(ring);
    int pos = 0;  // ring position of slot t (t % depth)
    for (int t = 0, j = warp; j < nslots; ++t, j += nw) {
      cp_async_wait(depth - 1);  // this thread's copies of slot t have landed
      __syncwarp();              // ... and every lane's
      const uint32_t sl = ring_s + (uint32_t)(pos * geo.slot_bytes);
      pos = pos + 1 == depth ? 0 : pos + 1;
      const int row0 = j * rps;
      const int rows = min(rps, nrows - row0);
      float mine = 0.0f;
      for (int i = 0; i < rows; i += 2) {
        const bool has_b = i + 1 < rows;
        const uint32_t wa = sl + (uint32_t)(i * (int)S);
        const uint32_t wb = has_b ? wa + (uint32_t)S : wa;
        float ta = 0.0f, tb = 0.0f;
        for (int sg = 0; sg < nseg; ++sg) {
          XSeg xsg;
          if constexpr (kXReg) xsg = xs;
          else xsg = load_xseg_s(qx_s, dx_s, nb, sg);
          float pa, pb;
          seg_terms2_s(wa, wb, has_b, K, sg, xsg, pa, pb);
          ta = __fadd_rn(ta, pa);
          tb = __fadd_rn(tb, pb);
        }
        warp_sum2(ta, tb);
        if (lane == i) mine = ta;
        if (lane == i + 1) mine = tb;
      }
      __syncwarp();  // every lane is done with the slot before it is refilled
      issue(t + depth);
      if (lane < rows) emit(row0 + lane, mine);
    }
    cp_async_wait(0);  // no copy of this warp outlives it (the trailing groups are empty)
  }
  if constexpr (kAllreduce) {
    // ---- cross-GPU sum of this CTA's rows (the same row range on every rank) ----
    // Each thread waits for the staged words of its rows from every rank -- a word whose
    // tag is this call's epoch holds this call's value -- and adds them in rank order.  No
    // fence and no flag: on B200 a system-scope fence after the peer stores took ~3.6 us
    // and each release store of a flag ~3.5 us more.  The wait is bounded in time; rows
    // whose peers never arrive are written as NaN and bit 1 of the fault word is set.
    const unsigned long long* stage = fz.ar_stage[fz.ar_rank] + (size_t)(fz.ar_epoch & 1u) * fz.ar_world * N;
    const float nan = __int_as_float(0x7fc00000);
    const uint64_t t0 = global_ns();
    bool ok = true;
    for (int rr = threadIdx.x; rr < nrows; rr += kStreamThreads) {
      float v = 0.0f;
      for (int p = 0; p < fz.ar_world && ok; ++p) {
        const unsigned long long* a = stage + (size_t)p * N + r0 + rr;
        unsigned long long wv = 0;
        for (uint32_t i = 0;; ++i) {
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(wv) : "l"(a) : "memory");
          if ((int)((unsigned)(wv >> 32) - fz.ar_epoch) >= 0) break;  // this call's word (or a later one)
          if ((i & 15u) == 15u && global_ns() - t0 > wait_ns) {
            ok = false;
            break;
          }
          if (i > 64) __nanosleep(32);
        }
        const float pv = __uint_as_float((unsigned)wv);
        v = p == 0 ? pv : __fadd_rn(v, pv);
      }
      y[r0 + rr] = !ok ? nan : (fz.residual ? __fadd_rn(fz.residual[r0 + rr], v) : v);
    }
    if (!ok) atomicOr(&g_gemv_fault, 2u);
  }
}

// Slot geometry of the M = 1 streaming kernel for this K (nw == 0: the kernel does not
// apply): slots of about two K = 2048 rows, depth 2, as many ring warps as the ~96 KB of
// ring allow (measured on B200 in CUDA graphs against 1-row slots and deeper rings:
// 2 rows x 11 warps x depth 2 streams the decode chain fastest at K = 2048, and 1 row x
// 7 warps x depth 2 at K = 6144).  Q8LIN_STREAM_GEO=rps:nw:depth overrides it where the
// ring fits (experiments).
StreamGeo stream_geometry(int64_t k, int64_t S) {
  StreamGeo g;
  if (k > kStreamMaxK || k % kQK) return g;
  int64_t rps = kSlotTargetBytes / S;
  rps = rps < 1 ? 1 : (rps > kMaxRps ? kMaxRps : rps);
  int depth = 2;
  int64_t nw = kRingBytes / (rps * S) / depth;
  if (nw > kStreamWarps) nw = kStreamWarps;
  static const int* over = [] {
    static int v[3] = {0, 0, 0};
    const char* e = getenv("Q8LIN_STREAM_GEO");
    if (!e || sscanf(e, "%d:%d:%d", &v[0], &v[1], &v[2]) != 3) v[0] = 0;
    return v;
  }();
  if (over[0] >= 1 && over[0] <= kMaxRps && over[1] >= 1 && over[1] <= kStreamWarps && over[2] >= 2 &&
      over[2] <= kMaxDepth && (int64_t)over[0] * S * over[1] * over[2] <= kRingBytes) {
    rps = over[0];
    nw = over[1];
    depth = over[2];
  }
  if (nw < 1) return g;
  g.rps = (int)rps;
  g.nw = (int)nw;
  g.depth = depth;
  g.slot_bytes = (int)(rps * S);
  return g;
}

size_t stream_smem_bytes(const StreamGeo& g, int64_t k) {
  const int64_t nseg = (k + kSegValues - 1) / kSegValues;
  const size_t p1_cap = (size_t)g.nw * g.depth * g.rps;  // prefetched rows at most
  const size_t part = nseg > 1 ? (size_t)nseg * p1_cap * sizeof(float) : 0;
  return (size_t)g.nw * g.depth * g.slot_bytes + round16(k) + round16(4 * (k / kQK)) + part +
         p1_cap * sizeof(uint32_t);
}

template <bool kAllreduce, bool kXReg>
cudaError_t launch_stream_t(const q8lin_weight& w, const float* x, float* y, const StreamGeo& g, cudaStream_t s,
                            const GemvFusion& fz) {
  const int K = (int)w.k, N = (int)w.n;
  const size_t smem = stream_smem_bytes(g, K);
  static int configured[128] = {0};
  auto fn = gemv_q8_0_stream_kernel<kAllreduce, kXReg>;
  cudaError_t e = ensure_smem((const void*)fn, configured, w.device, smem, true);
  if (e != cudaSuccess) return e;
  int grid = sm_count(w.device);
  if (grid > N) grid = N;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, fn, (const uint8_t*)w.packed, w.row_stride, N, K, x, y, g, fz, wait_limit_ns());
}

cudaError_t launch_stream(const q8lin_weight& w, const float* x, float* y, const StreamGeo& g, cudaStream_t s,
                          const GemvFusion& fz = GemvFusion()) {
  const bool xreg = w.k <= kSegValues;
  if (fz.ar_world > 1)
    return xreg ? launch_stream_t<true, true>(w, x, y, g, s, fz) : launch_stream_t<true, false>(w, x, y, g, s, fz);
  return xreg ? launch_stream_t<false, true>(w, x, y, g, s, fz) : launch_stream_t<false, false>(w, x, y, g, s, fz);
}

template <int M>
cudaError_t launch_m(const q8lin_weight& w, const float* x, float* y, cudaStream_t s) {
  const int K = (int)w.k, N = (int)w.n;
  const size_t smem = gemv_smem_bytes(M, K);
  // The dynamic shared-memory opt-in is per device context; remember it per device.
  static int configured_smem[128] = {0};
  if (smem > 48 * 1024) {
    cudaError_t e = ensure_smem((const void*)gemv_q8_0_kernel<M>, configured_smem, w.device, smem, false);
    if (e != cudaSuccess) return e;
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

// Whether the M = 1 streaming kernel serves K.
bool stream_applies(int64_t k) { return stream_geometry(k, packed_row_stride(k)).nw > 0; }

size_t gemv_smem_bytes(int m, int64_t k) {
  return (((size_t)m * k + 15) / 16) * 16 + (size_t)m * (k / kQK) * sizeof(float);
}

cudaError_t read_gemv_fault(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_gemv_fault, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_gemv_fault, &z, sizeof(z));
  }
  return e;
}

cudaError_t launch_gemv_fused(const q8lin_weight& w, const float* x, float* y, const GemvFusion& f, cudaStream_t s) {
  const StreamGeo g = stream_geometry(w.k, w.row_stride);
  if (g.nw == 0 || w.k > kFusedMaxK) return cudaErrorInvalidValue;
  return launch_stream(w, x, y, g, s, f);
}

cudaError_t launch_gemv(const q8lin_weight& w, const float* x, float* y, int m, cudaStream_t s) {
  if (m == 1) {
    const StreamGeo g = stream_geometry(w.k, w.row_stride);
    if (g.nw > 0) return launch_stream(w, x, y, g, s);
  }
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
