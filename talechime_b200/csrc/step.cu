// Persistent decode-step kernel: one cooperative launch runs a whole program of
// operations -- Q8_0 GEMVs (M = 1, with rms_norm / SwiGLU prologues and residual,
// SwiGLU and argmax epilogues), RoPE + KV append + attention, the embedding gather and
// the greedy argmax -- that the multi-launch decode step runs as ~140 kernels.
//
// Why: a decode step is a chain of ~113 weight-streaming GEMVs, each of which needs the
// previous one's full output.  With one kernel per operation every boundary costs a
// dependency release, the activation load and its quantization, during which HBM
// idles.  Here the weights -- constant -- never wait for the data:
//   * one CTA per SM (cooperative launch, so every CTA is resident), 15 consumer warps
//     and one producer warp;
//   * the producer walks the program's GEMVs in order and streams this CTA's rows of
//     each weight through a shared-memory ring (14 slots of 13,056 bytes: 6 rows of K =
//     2048, 2 rows of K = 6144) with cp.async.bulk, never waiting on activations, so
//     it runs up to ~180 KB ahead across operation boundaries and attention phases;
//   * the consumers run the operations in order; operation i starts when every CTA has
//     finished operation i - 1 (a per-operation arrival counter: release add by one
//     thread of each CTA after a CTA barrier, acquire poll by one thread of the waiting
//     CTA before a CTA barrier), the only synchronisation between CTAs;
//   * every consumer warp consumes every ring chunk in order -- waits for it, does its
//     pairs if it has any -- and arrives on the chunk's empty barrier, which counts all
//     consumer warps: the producer is then never more than one ring ahead of any warp,
//     so the parity a warp waits on always names the chunk it wants.  (Waiting only for
//     the chunks holding its own rows let a warp test the next use of a slot whose
//     current copy had not landed, where the parity test passes at once.)
// GEMV work split: CTA c owns rows [N c / G, N (c + 1) / G) (with the SwiGLU epilogue:
// pairs (gate i, up i) for i in [I c / G, I (c + 1) / G), the gate and up rows of a pair
// copied into the same ring chunk).  A row's K values form ceil(K / 2048) segments;
// warp w keeps segment w % nseg of the quantized activations in registers (lane l:
// blocks l and l + 32 of the segment) and takes every ngroups-th pair of rows of the
// CTA (two rows in flight per warp); segments of a row are combined in segment order.
// Attention: units (q head, split) with 8 splits per head over the current length;
// each unit writes a (max, sum, acc[128]) partial and the last unit of a head to
// arrive merges the head's partials in split order into the output.
// Counters are reset by the last CTA to finish, so the next launch starts from zero.
// Every wait is bounded: on timeout bit 4 of the fault word is set, the other CTAs
// stop waiting soon after, and the kernel ends without hanging (outputs invalid).
#include <cmath>

#include <climits>

#include "common.cuh"
#include "internal.h"

namespace q8lin {

namespace {

constexpr int kSWarps = 15;                    // consumer warps (17 warps would cap registers at 96)
constexpr int kSConsumers = kSWarps * 32;      // 480
constexpr int kSThreads = kSConsumers + 32;    // + producer warp
constexpr int kSlotBytes = 13056;              // 6 x 2176 = 2 x 6528
constexpr int kSlots = 14;
constexpr int kRingBytes = kSlots * kSlotBytes;
constexpr int kSMaxRpc = 8;
constexpr int kSMaxSegs = 4;
constexpr int kSMaxResidualRows = kSConsumers;
constexpr int kSplits = 8;                     // attention splits per q head

__device__ unsigned int g_step_fault;

struct SmemLayout {
  static constexpr int ring = 0;
  static constexpr int qx = ring + kRingBytes;                     // int8 [kStepMaxK]
  static constexpr int dx = qx + kStepMaxK;                        // f32 [kStepMaxK / 32]
  static constexpr int part = dx + kStepMaxK / 32 * 4;             // f32 [kSlots][kSMaxRpc][kSMaxSegs]
  static constexpr int cnt = part + kSlots * kSMaxRpc * kSMaxSegs * 4;  // int [kSlots][kSMaxRpc]
  static constexpr int res = cnt + kSlots * kSMaxRpc * 4;          // f32 [kSMaxResidualRows]
  static constexpr int red = res + (kSMaxResidualRows + 3) / 4 * 16;  // f32 [32]
  static constexpr int amv = red + 32 * 4;                         // f32 [kSWarps], 16 slots
  static constexpr int ami = amv + 16 * 4;                         // int [kSWarps], 16 slots
  static constexpr int aq = ami + 16 * 4;                          // f32 [128] rotated q
  static constexpr int akc = aq + 128 * 4;                         // f32 [128] current k
  static constexpr int avc = akc + 128 * 4;                        // f32 [128] current v
  static constexpr int awp = avc + 128 * 4;                        // f32 [kSWarps][132] warp partials
  static constexpr int flag = awp + kSWarps * 132 * 4;             // int [4]
  static constexpr int tally = flag + 16;                          // int [kSlots] (spare)
  static constexpr int full = tally + (kSlots * 4 + 15) / 16 * 16;  // u64 [kSlots]
  static constexpr int empty = full + kSlots * 8;                  // u64 [kSlots]
  static constexpr int bytes = empty + kSlots * 8;
};
static_assert(SmemLayout::full % 8 == 0, "mbarriers need 8-byte alignment");
static_assert(SmemLayout::aq % 16 == 0 && SmemLayout::awp % 16 == 0, "float4 scratch alignment");
static_assert(SmemLayout::bytes <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// After any wait of any CTA has timed out, the others stop waiting too (within ~1k polls).
__device__ __forceinline__ bool step_aborted() { return (*(volatile unsigned*)&g_step_fault & 16u) != 0u; }

// This CTA's wait limit (the kernel's wait_ns argument, set by thread 0 at entry).
__shared__ uint64_t s_step_wait_ns;

__device__ __noinline__ bool mbar_wait_slow(uint32_t a, uint32_t parity) {
  const uint64_t t0 = global_ns(), lim = s_step_wait_ns;
  for (uint32_t i = 1;; ++i) {
    if (mb_try(a, parity)) return true;
    if ((i & 15u) == 0u) {
      if (step_aborted()) return false;
      if (global_ns() - t0 > lim) break;
    }
  }
  atomicOr(&g_step_fault, 16u);
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = su32(bar);
  return mb_try(a, parity) || mbar_wait_slow(a, parity);
}
// Wait for this CTA's own bulk copies before it exits: the fixed drain bound.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
  return mb_wait_ns(su32(bar), parity, kDrainLimitNs, nullptr);
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release(unsigned* p) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(1u) : "memory");
}

// One thread waits until the counter reaches `target` (bounded in time).
__device__ __forceinline__ void wait_count(const unsigned* p, unsigned target) {
  const uint64_t t0 = global_ns(), lim = s_step_wait_ns;
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire(p) >= target) return;
    if (i > 256) __nanosleep(20);
    if ((i & 15u) == 15u) {
      if (step_aborted()) return;
      if (global_ns() - t0 > lim) break;
    }
  }
  atomicOr(&g_step_fault, 16u);
}

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(kSConsumers) : "memory");
}

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// Rows (or, with the SwiGLU epilogue, gate/up pairs) [n c / g, n (c + 1) / g) of CTA c.
__device__ __forceinline__ void cta_range(int n, int c, int g, int& r0, int& r1) {
  r0 = (int)(((int64_t)n * c) / g);
  r1 = (int)(((int64_t)n * (c + 1)) / g);
}

// Units of the CTA's share of a GEMV: rows, or pairs with the SwiGLU epilogue.
__device__ __forceinline__ int gemv_units(const StepOp& op) { return op.epilogue == kStepEpilogueSwiGLU ? op.n / 2 : op.n; }
// Units per ring chunk.
__device__ __forceinline__ int chunk_units(const StepOp& op) {
  return op.epilogue == kStepEpilogueSwiGLU ? op.rpc / 2 : op.rpc;
}

// ---------------------------------------------------------------------------------
// Consumer phases.

// Activation prologue + Q8_0 quantization of x into qx/dx (all consumers).  `wn` holds
// this thread's rms_norm weights, loaded before the dependency wait.
constexpr int kQuadGroups = (kStepMaxK / 4 + kSConsumers - 1) / kSConsumers;

__device__ void gemv_prologue(const StepOp& op, const float4 (&wn)[kQuadGroups], uint8_t* sm) {
  constexpr int kQG = (kStepMaxK / 4 + kSConsumers - 1) / kSConsumers;
  const int tid = threadIdx.x;
  const int K = op.k, nb = K >> 5, nquads = nb * 8;
  float4 v[kQG];
  if (op.prologue == kStepPrologueSwiGLU) {
#pragma unroll
    for (int g = 0; g < kQG; ++g) {
      const int i = g * kSConsumers + tid;
      if (i < nquads) {
        const float4 ga = ldcg4(op.x + 4 * i), ua = ldcg4(op.x + K + 4 * i);
        v[g] = make_float4(silu_mul(ga.x, ua.x), silu_mul(ga.y, ua.y), silu_mul(ga.z, ua.z), silu_mul(ga.w, ua.w));
      } else {
        v[g] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  } else {
#pragma unroll
    for (int g = 0; g < kQG; ++g) {
      const int i = g * kSConsumers + tid;
      v[g] = i < nquads ? ldcg4(op.x + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (op.prologue == kStepPrologueRmsNorm) {
    float* red = reinterpret_cast<float*>(sm + SmemLayout::red);
    float sq = 0.0f;
#pragma unroll
    for (int g = 0; g < kQG; ++g) {
      if (g * kSConsumers >= nquads) break;  // uniform: zero groups add nothing
      sq = __fadd_rn(sq, __fmul_rn(v[g].x, v[g].x));
      sq = __fadd_rn(sq, __fmul_rn(v[g].y, v[g].y));
      sq = __fadd_rn(sq, __fmul_rn(v[g].z, v[g].z));
      sq = __fadd_rn(sq, __fmul_rn(v[g].w, v[g].w));
    }
    sq = warp_sum(sq);
    if ((tid & 31) == 0) red[tid >> 5] = sq;
    consumers_sync();
    float total = 0.0f;
#pragma unroll
    for (int i = 0; i < kSWarps; ++i) total += red[i];
    const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)K), op.eps));
#pragma unroll
    for (int g = 0; g < kQG; ++g) {
      if (g * kSConsumers + tid < nquads) {  // the IEEE divisions only where there are values
        const float4 wv = wn[g];
        v[g] = make_float4(__fmul_rn(__fdiv_rn(v[g].x, m), wv.x), __fmul_rn(__fdiv_rn(v[g].y, m), wv.y),
                           __fmul_rn(__fdiv_rn(v[g].z, m), wv.z), __fmul_rn(__fdiv_rn(v[g].w, m), wv.w));
      }
    }
  }
  int8_t* qx = reinterpret_cast<int8_t*>(sm + SmemLayout::qx);
  float* dx = reinterpret_cast<float*>(sm + SmemLayout::dx);
#pragma unroll
  for (int g = 0; g < kQG; ++g) {
    if (g * kSConsumers < nquads) {  // uniform across the consumers: every lane shuffles
      const int i = g * kSConsumers + tid;
      __half dh;
      const int q = quantize_octet(v[g], dh);
      if (i < nquads) {
        reinterpret_cast<int*>(qx)[i] = q;
        if ((i & 7) == 0) dx[i >> 3] = __half2float(dh);
      }
    }
  }
}

// One GEMV operation on the consumer side.  `seq` is the ring position of its first
// chunk.  Every consumer warp waits for every chunk in order and arrives once on its
// empty barrier; warps beyond the op's groups (K = 8192) only wait and arrive.
__device__ void gemv_consume(const StepOp& op, int c, int g, int seq, uint8_t* sm, float* am_v, int* am_i) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool swi = op.epilogue == kStepEpilogueSwiGLU;
  int u0, u1;
  cta_range(gemv_units(op), c, g, u0, u1);
  const int nunits_cta = u1 - u0, cu = chunk_units(op), K = op.k, nb = K >> 5;
  const int64_t S = op.S;
  const int nseg = (nb + 63) >> 6, ngroups = kSWarps / nseg;
  const int seg = warp % nseg, grp = warp / nseg;
  const bool idle = grp >= ngroups;  // K = 6144 with 15 warps uses all; K = 8192: three idle warps
  const int nchunks = (nunits_cta + cu - 1) / cu;
  float* part = reinterpret_cast<float*>(sm + SmemLayout::part);
  int* cnt = reinterpret_cast<int*>(sm + SmemLayout::cnt);
  const float* res = reinterpret_cast<const float*>(sm + SmemLayout::res);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + SmemLayout::full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(sm + SmemLayout::empty);
  const bool res_smem = op.residual && nunits_cta <= kSMaxResidualRows;
  const float* residual = op.residual;
  float* y = op.y;
  const XSeg xs = load_xseg(reinterpret_cast<const int8_t*>(sm + SmemLayout::qx),
                            reinterpret_cast<const float*>(sm + SmemLayout::dx), nb, seg);
  float bv = -INFINITY;
  int bi = op.n;
  // finalize one row value (row index `r` within the CTA's rows)
  auto finish = [&](int r, float val) {
    const int grow = u0 + r;
    if (residual) val = __fadd_rn(res_smem ? res[r] : __ldcg(residual + grow), val);
    y[grow] = val;
    if (val > bv || (val == bv && grow < bi)) {
      bv = val;
      bi = grow;
    }
  };
  int off = idle ? INT_MAX / 2 : grp;  // this warp's first pair in the current chunk: pairs go round-robin
  for (int jj = 0; jj < nchunks; ++jj) {
    const int i0 = jj * cu, nu = min(cu, nunits_cta - i0);
    const int npairs = swi ? nu : (nu + 1) >> 1;
    const int j = seq + jj, slot = j % kSlots;
    mbar_wait(&full[slot], (uint32_t)((j / kSlots) & 1));
    const uint8_t* chunk = sm + SmemLayout::ring + (size_t)slot * kSlotBytes;
    int done_pairs = 0;
    int p = off;
    for (; p < npairs; p += ngroups, ++done_pairs) {
      const int ra = swi ? p : 2 * p;
      const int rb = swi ? nu + p : 2 * p + 1;
      const bool has_b = swi || rb < nu;
      float sa, sb;
      seg_dot2(chunk + (size_t)ra * S, chunk + (size_t)rb * S, has_b, K, seg, xs, sa, sb);
      if (lane == 0) {
        if (nseg == 1) {
          if (swi) {
            y[u0 + i0 + p] = silu_mul(sa, sb);  // gate i, up i -> h[i]
          } else {
            finish(i0 + ra, sa);
            if (has_b) finish(i0 + rb, sb);
          }
        } else {
          // segments of a row meet in shared memory; the last warp adds them in order
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int ri = h ? rb : ra;
            if (h && !has_b) break;
            float* pr = part + (slot * kSMaxRpc + ri) * kSMaxSegs;
            pr[seg] = h ? sb : sa;
            __threadfence_block();
            if (atomicAdd(&cnt[slot * kSMaxRpc + ri], 1) == nseg - 1) {
              __threadfence_block();
              float sum = pr[0];
              for (int q = 1; q < nseg; ++q) sum += pr[q];
              cnt[slot * kSMaxRpc + ri] = 0;
              finish(i0 + ri, sum);
            }
          }
        }
      }
    }
    if (!idle) off = p - npairs;
    (void)done_pairs;
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&empty[slot])) : "memory");
  }
  if (op.argmax && lane == 0) {
    am_v[warp] = bv;
    am_i[warp] = bi;
  }
}

// RoPE + KV append + partial attention for unit (h, split); the last unit of head h
// merges the head (all consumers).
// The first group of K and V rows of a warp (up to four cached positions), loaded before
// the dependency wait: cached rows below pos were written by earlier launches.
struct KVFirst {
  float4 k[4], v[4];
};

__device__ __forceinline__ void attention_unit_range(int len, int split, int& a, int& b) {
  const int per = (len + kSplits - 1) / kSplits;
  a = min(len, split * per);
  b = min(len, a + per);
}

__device__ void attention_prefetch(const StepOp* gop, int unit, int pos, KVFirst& f) {
  constexpr int D = 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = __ldg(&gop->hq), hkv = __ldg(&gop->hkv), max_t = __ldg(&gop->max_t);
  const int h = unit / kSplits, split = unit % kSplits, hk = h / (hq / hkv);
  const int len = pos < 0 ? 0 : min(pos + 1, max_t);
  int a, b;
  attention_unit_range(len, split, a, b);
  const float* kh = gop->kc + (size_t)hk * max_t * D;
  const float* vh = gop->vc + (size_t)hk * max_t * D;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int t = a + warp + u * kSWarps;
    if (t < b && t != pos) {
      f.k[u] = ldcg4(kh + (size_t)t * D + 4 * lane);
      f.v[u] = ldcg4(vh + (size_t)t * D + 4 * lane);
    } else {
      f.k[u] = f.v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

__device__ void attention_unit(const StepOp& op, int unit, int pos, uint8_t* sm, const KVFirst* first) {
  constexpr int D = 128, half = 64;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = unit / kSplits, split = unit % kSplits;
  const int Hq = op.hq, Hkv = op.hkv, group = Hq / Hkv, hk = h / group, max_t = op.max_t;
  float* aq = reinterpret_cast<float*>(sm + SmemLayout::aq);
  float* akc = reinterpret_cast<float*>(sm + SmemLayout::akc);
  float* avc = reinterpret_cast<float*>(sm + SmemLayout::avc);
  float* awp = reinterpret_cast<float*>(sm + SmemLayout::awp);
  int* flag = reinterpret_cast<int*>(sm + SmemLayout::flag);
  const int len = pos < 0 ? 0 : min(pos + 1, max_t);
  int a, b;
  attention_unit_range(len, split, a, b);
  const bool cur = a <= pos && pos < b;
  if (tid < D && pos >= 0 && pos < max_t) {
    const int j = tid < half ? tid : tid - half;
    const float c = __ldg(op.cos_t + (size_t)pos * half + j), sn = __ldg(op.sin_t + (size_t)pos * half + j);
    auto rot = [&](const float* xh) {
      return tid < half ? __fadd_rn(__fmul_rn(__ldcg(xh + tid), c), __fmul_rn(__ldcg(xh + tid + half), -sn))
                        : __fadd_rn(__fmul_rn(__ldcg(xh + tid), c), __fmul_rn(__ldcg(xh + tid - half), sn));
    };
    aq[tid] = rot(op.x + (size_t)h * D);
    if (cur) {
      const float kr = rot(op.x + (size_t)(Hq + hk) * D);
      const float vr = __ldcg(op.x + (size_t)(Hq + Hkv + hk) * D + tid);
      akc[tid] = kr;
      avc[tid] = vr;
      if (h % group == 0) {  // one writer per kv head
        op.kc[((size_t)hk * max_t + pos) * D + tid] = kr;
        op.vc[((size_t)hk * max_t + pos) * D + tid] = vr;
      }
    }
  }
  consumers_sync();
  const float4 q4 = reinterpret_cast<const float4*>(aq)[lane];
  const float* kh = op.kc + (size_t)hk * max_t * D;
  const float* vh = op.vc + (size_t)hk * max_t * D;
  float m = -INFINITY, l = 0.0f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  // warp w: positions a + w, a + w + 16, ...; four positions' K and V rows in flight
  for (int t0 = a + warp; t0 < b; t0 += 4 * kSWarps) {
    float4 k4[4], v4[4];
    const bool pre = first && t0 == a + warp;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + u * kSWarps;
      if (t >= b) {
        k4[u] = v4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      } else if (t == pos) {  // the current token: rotated in this launch, not read back from the cache
        k4[u] = reinterpret_cast<const float4*>(akc)[lane];
        v4[u] = reinterpret_cast<const float4*>(avc)[lane];
      } else if (pre) {
        k4[u] = first->k[u];
        v4[u] = first->v[u];
      } else {
        k4[u] = ldcg4(kh + (size_t)t * D + 4 * lane);
        v4[u] = ldcg4(vh + (size_t)t * D + 4 * lane);
      }
    }
    float s[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float d = __fmul_rn(q4.x, k4[u].x);
      d = __fadd_rn(d, __fmul_rn(q4.y, k4[u].y));
      d = __fadd_rn(d, __fmul_rn(q4.z, k4[u].z));
      s[u] = __fadd_rn(d, __fmul_rn(q4.w, k4[u].w));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) s[u] += __shfl_xor_sync(kFull, s[u], o);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (t0 + u * kSWarps < b) {
        const float sc = __fmul_rn(s[u], op.scale);
        const float mn = fmaxf(m, sc);
        const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
        const float p = expf(sc - mn);
        l = __fadd_rn(__fmul_rn(l, corr), p);
        acc.x = __fadd_rn(__fmul_rn(acc.x, corr), __fmul_rn(p, v4[u].x));
        acc.y = __fadd_rn(__fmul_rn(acc.y, corr), __fmul_rn(p, v4[u].y));
        acc.z = __fadd_rn(__fmul_rn(acc.z, corr), __fmul_rn(p, v4[u].z));
        acc.w = __fadd_rn(__fmul_rn(acc.w, corr), __fmul_rn(p, v4[u].w));
        m = mn;
      }
    }
  }
  float* wp = awp + warp * 132;
  if (lane == 0) {
    wp[0] = m;
    wp[1] = l;
  }
  reinterpret_cast<float4*>(wp + 4)[lane] = acc;
  consumers_sync();
  // merge the warps (warp order), one thread per dimension, into the unit's partial
  float* hp = op.attn_part + (size_t)h * kSplits * 132;
  if (tid < D) {
    float M = -INFINITY;
    for (int w = 0; w < kSWarps; ++w) M = fmaxf(M, awp[w * 132]);
    float L = 0.0f, A = 0.0f;
    for (int w = 0; w < kSWarps; ++w) {
      const float mw = awp[w * 132];
      const float f = (mw == -INFINITY) ? 0.0f : expf(mw - M);
      L = __fadd_rn(L, __fmul_rn(awp[w * 132 + 1], f));
      A = __fadd_rn(A, __fmul_rn(awp[w * 132 + 4 + tid], f));
    }
    float* dst = hp + split * 132;
    dst[4 + tid] = A;
    if (tid == 0) {
      dst[0] = M;
      dst[1] = L;
    }
  }
  consumers_sync();
  if (tid == 0) {
    __threadfence();
    flag[0] = atomicAdd(op.head_cnt + h, 1u) == (unsigned)(kSplits - 1);
    if (flag[0]) __threadfence();
  }
  consumers_sync();
  if (flag[0]) {  // last unit of head h: merge the splits in order
    if (tid < D) {
      float ms[kSplits];
      float M = -INFINITY;
#pragma unroll
      for (int s = 0; s < kSplits; ++s) {
        ms[s] = __ldcg(hp + s * 132);
        M = fmaxf(M, ms[s]);
      }
      float L = 0.0f, A = 0.0f;
#pragma unroll
      for (int s = 0; s < kSplits; ++s) {
        const float f = (ms[s] == -INFINITY) ? 0.0f : expf(ms[s] - M);
        L = __fadd_rn(L, __fmul_rn(__ldcg(hp + s * 132 + 1), f));
        A = __fadd_rn(A, __fmul_rn(__ldcg(hp + s * 132 + 4 + tid), f));
      }
      op.y[(size_t)h * D + tid] = L > 0.0f ? __fdiv_rn(A, L) : 0.0f;
    }
    if (tid == 0) op.head_cnt[h] = 0;
  }
}

}  // namespace

__global__ void __launch_bounds__(kSThreads, 1)
decode_step_kernel(const StepOp* __restrict__ ops, int nops, int* __restrict__ pos_dev, int* __restrict__ token,
                   unsigned* __restrict__ done, float* __restrict__ am_gv, int* __restrict__ am_gi, uint64_t wait_ns) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, g = gridDim.x;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + SmemLayout::full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(sm + SmemLayout::empty);
  if (tid == 0) {
    s_step_wait_ns = wait_ns;
    for (int i = 0; i < kSlots; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&full[i])), "r"(1) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&empty[i])), "r"(kSWarps) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  int* cnt = reinterpret_cast<int*>(sm + SmemLayout::cnt);
  for (int i = tid; i < kSlots * kSMaxRpc; i += kSThreads) cnt[i] = 0;
  __syncthreads();

  if (warp == kSWarps) {
    // ---------------- producer: every GEMV's rows of this CTA, in program order ----------------
    if (lane == 0) {
      int j = 0;
      bool ok = true;
      for (int o = 0; o < nops && ok; ++o) {
        const StepOp& op = ops[o];
        if (op.kind != kStepOpGemv) continue;
        const bool swi = op.epilogue == kStepEpilogueSwiGLU;
        const int cu = chunk_units(op), half_n = op.n / 2;
        const int64_t S = op.S;
        int u0, u1;
        cta_range(gemv_units(op), c, g, u0, u1);
        for (int u = u0; u < u1; u += cu, ++j) {
          const int slot = j % kSlots;
          if (j >= kSlots && !mbar_wait(&empty[slot], (uint32_t)(((j / kSlots) - 1) & 1))) {
            ok = false;
            break;
          }
          const int nu = min(cu, u1 - u);
          const uint32_t part_bytes = (uint32_t)(nu * S);
          const uint32_t dst = su32(sm + SmemLayout::ring + (size_t)slot * kSlotBytes);
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[slot])),
                       "r"(swi ? 2 * part_bytes : part_bytes) : "memory");
          asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                       ::"r"(dst), "l"(op.W + (size_t)u * S), "r"(part_bytes), "r"(su32(&full[slot])) : "memory");
          if (swi)  // the up rows of the same pairs, right after the gate rows
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                         ::"r"(dst + part_bytes), "l"(op.W + (size_t)(half_n + u) * S), "r"(part_bytes),
                         "r"(su32(&full[slot])) : "memory");
        }
      }
      // the copies must land before the CTA's shared memory is released
      for (int i = (j > kSlots ? j - kSlots : 0); i < j; ++i) mbar_drain(&full[i % kSlots], (uint32_t)((i / kSlots) & 1));
    }
    return;
  }

  // ---------------- consumers ----------------
  // The operation descriptor is copied to shared memory before the dependency wait: the
  // acquire of the wait discards L1, and the descriptor is read again after every
  // barrier wait of the ring, so global reads of it would cost L2 round trips.
  __shared__ __align__(16) StepOp s_op[2];  // double-buffered: op o + 1 is written while slow threads may still read op o
  constexpr int kOpWords = (int)(sizeof(StepOp) / 4);
  static_assert(sizeof(StepOp) % 4 == 0 && kOpWords <= kSConsumers, "descriptor copy");
  float* am_v = reinterpret_cast<float*>(sm + SmemLayout::amv);
  int* am_i = reinterpret_cast<int*>(sm + SmemLayout::ami);
  float* res = reinterpret_cast<float*>(sm + SmemLayout::res);
  // the position of this step: written only by the ARGMAX operation at the end of the
  // launch, so one read serves every operation
  const int pos = __ldcg(pos_dev);
  int seq = 0;
  for (int o = 0; o < nops; ++o) {
    if (tid < kOpWords)
      reinterpret_cast<uint32_t*>(&s_op[o & 1])[tid] = __ldg(reinterpret_cast<const uint32_t*>(ops + o) + tid);
    // constant inputs first: they do not depend on the previous operation
    float4 wn[kQuadGroups];
    {
      const int kind = __ldg(&ops[o].kind), pro = __ldg(&ops[o].prologue);
      if (kind == kStepOpGemv && pro == kStepPrologueRmsNorm) {
        const int nquads = __ldg(&ops[o].k) >> 2;
        const float4* w4 = reinterpret_cast<const float4*>(ops[o].norm_w);
#pragma unroll
        for (int q = 0; q < kQuadGroups; ++q) {
          const int i = q * kSConsumers + tid;
          wn[q] = i < nquads ? __ldg(w4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    KVFirst kvf;
    const bool attn_first = __ldg(&ops[o].kind) == kStepOpAttention && c < __ldg(&ops[o].hq) * kSplits;
    if (attn_first) attention_prefetch(ops + o, c, pos, kvf);
    const StepOp& op = s_op[o & 1];
    if (tid == 0 && o > 0) wait_count(done + o - 1, (unsigned)g);
    consumers_sync();
    if (op.kind == kStepOpGemv) {
      int u0, u1;
      cta_range(gemv_units(op), c, g, u0, u1);
      if (op.residual && u1 - u0 <= kSMaxResidualRows && tid < u1 - u0) res[tid] = __ldcg(op.residual + u0 + tid);
      if (op.argmax && lane == 0) {
        am_v[warp] = -INFINITY;
        am_i[warp] = op.n;
      }
      gemv_prologue(op, wn, sm);
      consumers_sync();
      gemv_consume(op, c, g, seq, sm, am_v, am_i);
      seq += (u1 - u0 + chunk_units(op) - 1) / chunk_units(op);
      consumers_sync();
      if (op.argmax && tid == 0) {
        float bv = am_v[0];
        int bi = am_i[0];
        for (int w = 1; w < kSWarps; ++w)
          if (am_v[w] > bv || (am_v[w] == bv && am_i[w] < bi)) {
            bv = am_v[w];
            bi = am_i[w];
          }
        am_gv[c] = bv;
        am_gi[c] = bi;
      }
    } else if (op.kind == kStepOpAttention) {
      for (int unit = c; unit < op.hq * kSplits; unit += g) {
        attention_unit(op, unit, pos, sm, unit == c && attn_first ? &kvf : nullptr);
        consumers_sync();
      }
    } else if (op.kind == kStepOpEmbed) {
      int r0, r1;
      cta_range(op.k, c, g, r0, r1);
      int tok = __ldcg(token);
      tok = tok < 0 ? 0 : (tok >= op.n ? op.n - 1 : tok);
      const uint8_t* row = op.W + (size_t)tok * op.S;
      const __half* d = reinterpret_cast<const __half*>(row + op.k);
      for (int i = r0 + tid; i < r1; i += kSConsumers)
        op.y[i] = __fmul_rn((float)(int8_t)row[i], __half2float(d[i >> 5]));
      consumers_sync();
    } else if (op.kind == kStepOpArgmax && c == 0) {
      // lowest index among equal maxima; NaN compares as smaller
      float bv = -INFINITY;
      int bi = op.n;
      for (int i = tid; i < g; i += kSConsumers) {
        const float v = __ldcg(am_gv + i);
        const int ix = __ldcg(am_gi + i);
        if (v > bv || (v == bv && ix < bi)) {
          bv = v;
          bi = ix;
        }
      }
      for (int s = 16; s > 0; s >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, s);
        const int oi = __shfl_xor_sync(kFull, bi, s);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        am_v[warp] = bv;
        am_i[warp] = bi;
      }
      consumers_sync();
      if (tid == 0) {
        for (int w = 1; w < kSWarps; ++w)
          if (am_v[w] > bv || (am_v[w] == bv && am_i[w] < bi)) {
            bv = am_v[w];
            bi = am_i[w];
          }
        *token = bi;
        *pos_dev = pos + 1;
      }
      consumers_sync();
    }
    if (tid == 0) red_release(done + o);  // after the CTA barrier that ended the operation
  }
  // the last CTA to finish resets the counters for the next launch
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(done + nops, 1u) == (unsigned)(g - 1)) {
      for (int o = 0; o <= nops; ++o) done[o] = 0;
      __threadfence();
    }
  }
}

size_t step_smem_bytes() { return SmemLayout::bytes; }

int step_rows_per_chunk(int64_t k) {
  const int64_t S = packed_row_stride(k);
  if (S > kSlotBytes) return 0;
  const int64_t r = kSlotBytes / S;
  return (int)(r > kSMaxRpc ? kSMaxRpc : r);
}

int step_splits() { return kSplits; }

namespace {
cudaError_t configure(int device) {
  static int configured[128] = {0};
  const int dev = (device >= 0 && device < 128) ? device : 0;
  if (configured[dev]) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)SmemLayout::bytes);
  if (e == cudaSuccess) configured[dev] = 1;
  return e;
}
}  // namespace

cudaError_t launch_decode_step(const StepOp* ops, int nops, int* pos, int* token, unsigned* done, float* am_gv,
                               int* am_gi, int grid, int device, cudaStream_t s) {
  cudaError_t e = configure(device);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = SmemLayout::bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_step_kernel, ops, nops, pos, token, done, am_gv, am_gi, wait_limit_ns());
}

cudaError_t step_max_grid(int device, int* grid) {
  cudaError_t e = configure(device);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kSThreads, SmemLayout::bytes);
  if (e != cudaSuccess) return e;
  *grid = per_sm >= 1 ? sm_count(device) : 0;
  return cudaSuccess;
}

cudaError_t read_step_fault(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_step_fault, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_step_fault, &z, sizeof(z));
  }
  return e;
}

}  // namespace q8lin
