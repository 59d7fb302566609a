// Decode GEMV for 1 <= M <= 16: y[M][N] = Q8_0(x)[M][K] . W^T.
//
// HBM-bound: every launch streams the whole repacked weight (N*K*34/32 bytes) once.
// Two kernels:
//   * M = 1 and K <= 8192: gemv_q8_0_stream_kernel (below), one CTA per SM with a
//     shared-memory ring filled by bulk copies, sized so the next linear's CTA is
//     co-resident and prefetches its weights while this one computes;
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
// M = 1 streaming GEMV with cross-launch weight prefetch.
//
// Geometry: one CTA per SM owning the contiguous rows [r0, r1): 16 consumer warps and
// one producer warp, at most 56 registers per thread and ~100 KB of shared memory, so
// two CTAs fit on an SM -- the CTA of the next linear in the stream is resident while
// this one runs.  The CTA's rows are one contiguous byte range of the packed plane,
// copied into a shared-memory ring of `rpc`-row chunks with 1-D bulk copies
// (cp.async.bulk from this GPU's own memory).
//
// Order of events:
//   1. launch_dependents at once: the next linear's CTAs may become resident and start
//      their own copies while this one computes;
//   2. producer warp: copies of the first `slots` chunks -- weights are constant, so
//      they are issued before the dependency wait and overlap the previous linear --
//      then one refill per chunk whose rows have all been reduced (empty barrier);
//   3. consumer warps: griddepcontrol.wait, x quantized to Q8_0 in shared memory, then
//      each warp keeps its 2048-value segment of x (four 16-byte units per lane) and
//      the block scales in registers.  A row of K values is reduced by
//      ceil(K / 2048) warps, one segment each, straight from the ring; with several
//      segments the partial sums meet in shared memory and the last warp to arrive
//      adds them in segment order.  No CTA-wide barrier per chunk.
// Each block term is ((f32(isum) * dw) * dx) rounded per product as candle's scalar
// vec_dot; sums across blocks are trees, so outputs agree within f32 summation
// tolerance.  Every wait is bounded: on timeout bit 1 of the fault word is set and the
// waiting warp stops; the producer waits (bounded) for its last copies before it exits.
constexpr int kConsumerWarps = 16;
constexpr int kStreamThreads = (kConsumerWarps + 1) * 32;
constexpr int kRingBytes = 96 * 1024;
constexpr int kMaxSlots = 16;
constexpr int kMaxRpc = 4;
constexpr int kUnitsPerLane = 4;
constexpr int kSegUnits = 32 * kUnitsPerLane;  // 16-byte units per row segment (2048 values)
constexpr int kMaxSegs = 4;
constexpr int kStreamMaxK = kMaxSegs * kSegUnits * 16;
constexpr uint32_t kWaitLimit = 1u << 24;
constexpr int kStreamResRows = 512;  // residual rows staged in shared memory
constexpr uint32_t kPeerWaitLimit = 1u << 20;  // polls of a peer's flag (~1 s with the back-off)

__device__ unsigned int g_gemv_fault;

__host__ __device__ constexpr int64_t round16(int64_t v) { return (v + 15) / 16 * 16; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    if (ok) return true;
  }
  atomicOr(&g_gemv_fault, 2u);
  return false;
}

// kAllreduce: the cross-GPU sum tail (fz.ar_world > 1) is compiled only into its own
// instantiation, so the single-GPU kernel keeps its registers and shared memory.
template <bool kAllreduce>
__global__ void __launch_bounds__(kStreamThreads, 2)
gemv_q8_0_stream_kernel(const uint8_t* __restrict__ W, int64_t S, int N, int K, const float* __restrict__ x,
                        float* __restrict__ y, int rpc, int slots, const GemvFusion fz) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = K >> 5;
  const int nunits = K >> 4;  // 16-byte units per row; unit u is half of block u / 2
  const int nseg = (nunits + kSegUnits - 1) / kSegUnits;  // warps per row
  const int ngroups = kConsumerWarps / nseg;               // rows in flight
  const int r0 = (int)(((int64_t)N * blockIdx.x) / gridDim.x);
  const int r1 = (int)(((int64_t)N * (blockIdx.x + 1)) / gridDim.x);
  const int nchunks = (r1 - r0 + rpc - 1) / rpc;
  const size_t chunk_bytes = (size_t)rpc * S;
  // [ring | qx: K int8 | dx: nb f32 | part: [slot][row][seg] f32 | cnt: [slot][row] |
  //  full, empty: kMaxSlots mbarriers each], every region on 16 bytes
  uint8_t* ring = smem;
  int8_t* qx = reinterpret_cast<int8_t*>(smem + kRingBytes);
  float* dx = reinterpret_cast<float*>(smem + kRingBytes + round16(K));
  float* part = reinterpret_cast<float*>(smem + kRingBytes + round16(K) + round16(4 * nb));
  int* cnt = reinterpret_cast<int*>(part + kMaxSlots * kMaxRpc * kMaxSegs);
  uint64_t* full = reinterpret_cast<uint64_t*>(cnt + kMaxSlots * kMaxRpc);
  uint64_t* empty = full + kMaxSlots;
  float* res_s = reinterpret_cast<float*>(empty + kMaxSlots);  // [kStreamResRows] residual rows of the CTA
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < slots; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&full[i])), "r"(1) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&empty[i])), "r"(rpc * nseg)
                   : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = threadIdx.x; i < kMaxSlots * kMaxRpc; i += kStreamThreads) cnt[i] = 0;
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < nchunks; ++j) {
        const int slot = j % slots;
        if (j >= slots && !bar_wait(&empty[slot], (uint32_t)((j / slots - 1) & 1))) break;
        const int row = r0 + j * rpc;
        const uint32_t bytes = (uint32_t)(min(rpc, r1 - row) * S);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&full[slot])),
                     "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(smem_u32(ring + (size_t)slot * chunk_bytes)), "l"(W + (size_t)row * S), "r"(bytes),
                     "r"(smem_u32(&full[slot]))
                     : "memory");
        issued = j + 1;
      }
      // the copies must land before the CTA's shared memory is released
      for (int j = (issued > slots ? issued - slots : 0); j < issued; ++j)
        bar_wait(&full[j % slots], (uint32_t)((j / slots) & 1));
    }
    return;
  }

  // ---------------- consumers ----------------
  {
    // float4 pieces of x, 8 lanes per block; the loads of up to four passes are issued
    // together so K <= 8192 costs one L2 round trip
    constexpr int kT = kConsumerWarps * 32;
    constexpr int kQG = 4;
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
    if (fz.residual && r1 - r0 <= kStreamResRows && (int)threadIdx.x < r1 - r0)
      res_s[threadIdx.x] = fz.residual[r0 + threadIdx.x];  // read before any row of this CTA is written
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
      // rms_norm over the row: sum of squares across the consumer warps (tree order),
      // m = sqrt(sum/K + eps), x -> (x / m) * w
      __shared__ float red[kConsumerWarps];
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
      asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
      float total = 0.0f;
#pragma unroll
      for (int i = 0; i < kConsumerWarps; ++i) total += red[i];
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
      if (g * kT < nquads) {  // uniform across the warps: every lane shuffles
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
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");  // consumer warps only

  const int seg = warp % nseg, grp = warp / nseg;
  const int nrows = r1 - r0;
  const bool res_from_smem = nrows <= kStreamResRows;
  // the row's value: written to y, or (cross-GPU sum) staged on every rank
  auto emit = [&](int rr, float v) {
    if constexpr (kAllreduce) {
      const size_t at = ((size_t)(fz.ar_epoch & 1u) * fz.ar_world + fz.ar_rank) * N + r0 + rr;
      for (int p = 0; p < fz.ar_world; ++p) fz.ar_stage[p][at] = v;
    } else {
      y[r0 + rr] = fz.residual ? __fadd_rn(res_from_smem ? res_s[rr] : fz.residual[r0 + rr], v) : v;
    }
  };
  // finalize row segment `rr` (chunk slot `slot`, row `ri` in the chunk) and release it
  auto finish = [&](int rr, int slot, int ri, float v) {
    if (nseg == 1) {
      emit(rr, v);
    } else {
      float* pr = part + (slot * kMaxRpc + ri) * kMaxSegs;
      pr[seg] = v;
      __threadfence_block();
      if (atomicAdd(&cnt[slot * kMaxRpc + ri], 1) == nseg - 1) {
        __threadfence_block();
        float sum = pr[0];
        for (int q = 1; q < nseg; ++q) sum += pr[q];
        emit(rr, sum);
        cnt[slot * kMaxRpc + ri] = 0;
      }
    }
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[slot])) : "memory");
  };
  // Ring position of a row, advanced incrementally (no division in the loop).
  struct Pos {
    int ri, slot;
    uint32_t parity;
  };
  auto advance = [&](Pos p, int rows) {
    p.ri += rows;
    while (p.ri >= rpc) {
      p.ri -= rpc;
      if (++p.slot == slots) {
        p.slot = 0;
        p.parity ^= 1u;
      }
    }
    return p;
  };
  // two rows in flight per warp: rr and rr + ngroups (the ring holds every chunk the
  // rows in flight of all warps can touch; checked by stream_plan's caller)
  // K = 6144: one warp of the sixteen has no segment and skips the rows (it stays for the
  // cross-GPU tail's barriers)
  if (!kAllreduce && grp >= ngroups) return;
  const XSeg xs = load_xseg(qx, dx, nb, grp < ngroups ? seg : 0);
  Pos pa = advance(Pos{0, 0, 0u}, grp);
  for (int rr = grp < ngroups ? grp : nrows; rr < nrows; rr += 2 * ngroups, pa = advance(pa, 2 * ngroups)) {
    const int rb = rr + ngroups;
    const bool has_b = rb < nrows;
    if (!bar_wait(&full[pa.slot], pa.parity)) break;
    const Pos pb = has_b ? advance(pa, ngroups) : pa;
    if (has_b && !bar_wait(&full[pb.slot], pb.parity)) break;
    const uint8_t* wa = ring + (size_t)pa.slot * chunk_bytes + (size_t)pa.ri * S;
    const uint8_t* wb = ring + (size_t)pb.slot * chunk_bytes + (size_t)pb.ri * S;
    float va, vb;
    seg_dot2(wa, wb, has_b, K, seg, xs, va, vb);
    __syncwarp();
    if (lane == 0) {
      finish(rr, pa.slot, pa.ri, va);
      if (has_b) finish(rb, pb.slot, pb.ri, vb);
    }
  }
  if constexpr (kAllreduce) {
  // ---- cross-GPU sum of this CTA's rows (the same row range on every rank) ----
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");  // all rows staged
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    __threadfence_system();  // the peer stores of this CTA before its flags
    const unsigned slot = blockIdx.x * (unsigned)fz.ar_world + (unsigned)fz.ar_rank;
    for (int p = 0; p < fz.ar_world; ++p)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(fz.ar_flags[p] + slot), "r"(fz.ar_epoch) : "memory");
    const unsigned* mine = fz.ar_flags[fz.ar_rank] + blockIdx.x * (unsigned)fz.ar_world;
    int ok = 1;
    for (int p = 0; p < fz.ar_world && ok; ++p) {
      ok = 0;
      for (uint32_t i = 0; i < kPeerWaitLimit; ++i) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + p) : "memory");
        if ((int)(v - fz.ar_epoch) >= 0) {  // this call's flag or a later one
          ok = 1;
          break;
        }
        if (i > 64) __nanosleep(64);
      }
    }
    if (!ok) atomicOr(&g_gemv_fault, 2u);
    s_ok = ok;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
  if (!s_ok) return;
  const float* stage = fz.ar_stage[fz.ar_rank] + (size_t)(fz.ar_epoch & 1u) * fz.ar_world * N;
  for (int rr = threadIdx.x; rr < nrows; rr += kConsumerWarps * 32) {
    float v = __ldcv(stage + r0 + rr);  // rank 0's rows, then rank 1's, ... (fixed order)
    for (int p = 1; p < fz.ar_world; ++p) v = __fadd_rn(v, __ldcv(stage + (size_t)p * N + r0 + rr));
    y[r0 + rr] = fz.residual ? __fadd_rn(res_from_smem ? res_s[rr] : fz.residual[r0 + rr], v) : v;
  }
  }
}

// Rows per chunk and ring slots of the M = 1 streaming kernel for this K (slots 0: the
// kernel does not apply).  Chunks shrink until at least 8 fit in the ring.
void stream_plan(int64_t k, int64_t S, int* rpc, int* slots) {
  *rpc = kMaxRpc;
  *slots = 0;
  if (k > kStreamMaxK) return;
  while (*rpc > 1 && kRingBytes / (*rpc * S) < 8) *rpc /= 2;
  const int64_t s = kRingBytes / (*rpc * S);
  *slots = s < 2 ? 0 : (int)(s > kMaxSlots ? kMaxSlots : s);
}

size_t stream_smem_bytes(int64_t k) {
  return (size_t)(kRingBytes + round16(k) + round16(4 * (k / kQK)) + kMaxSlots * kMaxRpc * kMaxSegs * 4 +
                  kMaxSlots * kMaxRpc * 4 + 2 * kMaxSlots * 8 + kStreamResRows * 4);
}

cudaError_t launch_stream(const q8lin_weight& w, const float* x, float* y, int rpc, int slots, cudaStream_t s,
                          const GemvFusion& fz = GemvFusion()) {
  const int K = (int)w.k, N = (int)w.n;
  const size_t smem = stream_smem_bytes(K);
  static int configured_smem[128] = {0};
  const int dev = (w.device >= 0 && w.device < 128) ? w.device : 0;
  if ((int)smem > configured_smem[dev]) {
    // the largest shared-memory carveout, so that two CTAs (this launch's and the
    // next one's) fit on an SM
    for (const void* fn : {(const void*)gemv_q8_0_stream_kernel<false>, (const void*)gemv_q8_0_stream_kernel<true>}) {
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return e;
    }
    configured_smem[dev] = (int)smem;
  }
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
  if (fz.ar_world > 1)
    return cudaLaunchKernelEx(&cfg, gemv_q8_0_stream_kernel<true>, (const uint8_t*)w.packed, w.row_stride, N, K, x,
                              y, rpc, slots, fz);
  return cudaLaunchKernelEx(&cfg, gemv_q8_0_stream_kernel<false>, (const uint8_t*)w.packed, w.row_stride, N, K, x, y,
                            rpc, slots, fz);
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

// Whether the M = 1 streaming kernel serves K (its ring holds at least two chunks).
bool stream_applies(int64_t k) {
  int rpc, slots;
  stream_plan(k, packed_row_stride(k), &rpc, &slots);
  return slots > 0;
}

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
  int rpc, slots;
  stream_plan(w.k, w.row_stride, &rpc, &slots);
  if (slots == 0 || w.k > kFusedMaxK) return cudaErrorInvalidValue;
  return launch_stream(w, x, y, rpc, slots, s, f);
}

cudaError_t launch_gemv(const q8lin_weight& w, const float* x, float* y, int m, cudaStream_t s) {
  if (m == 1) {
    int rpc, slots;
    stream_plan(w.k, w.row_stride, &rpc, &slots);
    if (slots > 0) return launch_stream(w, x, y, rpc, slots, s);
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
