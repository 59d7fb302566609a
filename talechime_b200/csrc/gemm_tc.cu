// Batched Q8_0 matmul on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// y[m][n] = sum_b dx[m][b] * dw[n][b] * I[m][n][b],  I = exact int dot of one 32-value
// block.  The per-block scales forbid accumulating across blocks inside the MMA, so
// every 32-value block gets its own tensor-core products and the rescale happens in
// registers:
//   * A = activations (MMA M = 128 rows of x), f16 holding the exact Q8_0 integers
//     (written by quantize_rows_f16t), 128B-swizzled tiles loaded by TMA;
//   * B = weights (MMA N = 128 rows of W), int8 tiles loaded by TMA from the packed
//     plane and widened to f16 integers in shared memory by converter warps (same
//     swizzled K-major layout);
//   * per block: two tcgen05.mma kind::f16 (K = 16 each) give I in a TMEM buffer (f32;
//     products of |q| <= 127 and their 32-term sums are exact integers), and a third
//     MMA gives the scale product P[m][n] = dx[m] * dw[n] next to it: its operands are
//     K = 16 tiles whose only non-zero column holds the f16 scales, so P is the outer
//     product, exact in f32 (11-bit x 11-bit significands);
//   * epilogue warps read I and P with tcgen05.ld and accumulate acc += I * P with
//     packed f32x2 FMAs: no shared-memory traffic and no broadcast of scales per
//     column, which is what bounds a register-side rescale.
// TMEM holds two blocks (2 x (I + P) = 512 columns), so the MMAs of block b + 1 run
// while block b is rescaled.  One CTA owns a 128 (m) x 128 (n) output tile over a range
// of K.
//
// Split-K: when the output has too few tiles to occupy the SMs (M = 64..256 against a
// 2048-row weight gives 16-48 tiles), grid.z splits K into ranges of whole scale groups
// (8 blocks); each CTA writes the valid rows of its partial tile to the workspace and a
// second kernel (tc_split_reduce_kernel, all SMs) adds the partials in split order, so
// the result does not depend on which CTA finishes first.  (Adding them in the last
// CTA of each tile left one SM doing a tile's whole reduction after the others were
// done: 22 us of a 36 us call at M = 64, N = K = 2048.)
//
// Rings (a stage = 64 K values = 2 blocks):
//   operand ring (kStages): A f16 tile + B int8 tile + activation scales;
//   converted ring (2 slots): f16 weight tile + the two blocks' scale operands;
//   one MMA commit per stage (consumed[s % kStages]) frees both slots of stage s.
//
// Warp roles (448 threads):
//   warp 0      TMA producer (waits on the upstream kernel before loading activations)
//   warp 1      TMEM allocation and MMA issue (one elected lane)
//   warps 2-5   int8 -> f16 conversion of the weight tile; scale operands
//   warps 6-13  epilogue: TMEM lane quadrant (warp % 4) x 64-column half ((warp - 6) / 4)
//
// Every mbarrier wait is bounded; a wait that runs out sets a fault word that the host
// reads with q8lin_fault_status and makes the CTA drain and return.
#include <cuda.h>

#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace q8lin {

__device__ unsigned int g_tc_fault;  // bit 0: a bounded wait ran out

namespace {

constexpr int kBM = 128;          // activation rows per tile (MMA M)
constexpr int kBN = 128;          // weight rows per tile (MMA N)
constexpr int kBK = 64;           // K values per stage (two Q8_0 blocks)
constexpr int kStages = 6;        // operand ring
constexpr int kBSlots = 2;        // converted ring
constexpr int kConvWarps = 4;     // warps 2..5
constexpr int kConvThreads = kConvWarps * 32;
constexpr int kEpiWarps = 8;      // warps 6..13
constexpr int kEpiCols = kBN / (kEpiWarps / 4);  // TMEM columns per epilogue warp
constexpr int kEpiWarp0 = 2 + kConvWarps;
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;  // two blocks x (I: kBN columns + P: kBN columns)
constexpr int kSplitMaxCtas = 148;  // tiles x splits bound when splitting (one wave)
constexpr int kGroupStages = 4;     // stages per 8-block scale group: split boundaries

constexpr int kAStageBytes = kBM * kBK * 2;   // 16 KB f16
constexpr int kBStageBytes = kBN * kBK * 2;   // 16 KB f16
constexpr int kB8StageBytes = kBN * kBK;      //  8 KB int8
constexpr int kDxStageBytes = 2 * kBM * 4;    //  1 KB f32
constexpr int kScaleTileBytes = 128 * 16 * 2; //  4 KB: 128 rows x K = 16 f16, no swizzle

static_assert(kConvThreads == kBN && kConvThreads == kBM, "one converter thread per tile row");

struct Smem {
  alignas(1024) uint8_t a[kStages][kAStageBytes];
  alignas(1024) uint8_t b[kBSlots][kBStageBytes];
  alignas(1024) uint8_t sx[kBSlots][2][kScaleTileBytes];  // activation-scale operand of each block
  alignas(1024) uint8_t sw[kBSlots][2][kScaleTileBytes];  // weight-scale operand of each block
  alignas(128) uint8_t b8[kStages][kB8StageBytes];
  alignas(128) float dx[kStages][2][kBM];   // activation scales of a stage's two blocks (TMA)
  alignas(8) uint64_t full[kStages];        // A + B int8 + activation scales landed
  alignas(8) uint64_t consumed[kStages];    // MMAs of stage s done: its operand slot and its
                                            // converted slot are free (one commit serves both)
  alignas(8) uint64_t bfull[kBSlots];       // converted B and scale operands written
  alignas(8) uint64_t acc_full[2];          // a block's I and P ready in TMEM buffer j
  alignas(8) uint64_t acc_empty[2];         // epilogue done reading buffer j
  alignas(8) uint64_t mma_done;             // every MMA this CTA issued has completed
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
// This CTA's wait limit (the kernel's wait_ns argument, set by thread 0 at entry).
__shared__ uint64_t s_wait_ns;

// Bounded wait for the phase with the given parity; false (and the fault flag) once the
// limit has passed, or false at once when the CTA aborted.  The spin lives out of line so
// that the many call sites keep their registers; the first poll is inline.
__device__ __noinline__ bool mbar_wait_slow(uint32_t a, uint32_t parity, volatile int* abort) {
  const uint64_t t0 = global_ns(), lim = s_wait_ns;
  for (uint32_t i = 1;; ++i) {
    if (mb_try(a, parity)) return true;
    if ((i & 15u) == 0u) {
      if (*abort) return false;
      if (global_ns() - t0 > lim) break;
    }
  }
  *abort = 1;
  atomicOr(&g_tc_fault, 1u);
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  const uint32_t a = su32(b);
  return mb_try(a, parity) || mbar_wait_slow(a, parity, abort);
}
// Wait for this CTA's own copies / MMAs before it exits: the fixed drain bound.
__device__ __forceinline__ bool mbar_drain(uint64_t* b, uint32_t parity) {
  return mb_wait_ns(su32(b), parity, kDrainLimitNs, nullptr);
}
// Every lane waits (and so acquires); the verdict is made warp-uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  return __all_sync(0xffffffffu, mbar_wait(b, parity, abort));
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(su32(bar))
      : "memory");
}

// K-major, 128B-swizzled UMMA shared-memory descriptor (8-row atoms of 128 B, SBO 1024 B).
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* base) {
  const uint64_t addr = su32(base);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;           // start address
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                 // layout: SWIZZLE_128B
  return d;
}

// K-major, unswizzled descriptor of a scale tile: core matrices of 8 rows x 16 B stored
// as 128 contiguous bytes; the two core matrices along K are 128 B apart (leading byte
// offset) and consecutive 8-row groups 256 B apart (stride byte offset).
__device__ __forceinline__ uint64_t umma_desc_plain(const void* base) {
  const uint64_t addr = su32(base);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;
  d |= (uint64_t)(128 >> 4) << 16;
  d |= (uint64_t)(256 >> 4) << 32;
  d |= (uint64_t)1 << 46;                 // layout field 0: no swizzle
  return d;
}
// Byte offset of element (row r, k = 0) in a scale tile.
__device__ __forceinline__ uint32_t scale_tile_offset(int r) { return (uint32_t)((r >> 3) * 256 + (r & 7) * 16); }

// Instruction descriptor: kind::f16, A/B f16, D f32, both K-major, M = 128, N = kBN.
constexpr uint32_t kIdesc = (1u << 4)                    // D format f32
                          | (0u << 7) | (0u << 10)       // A, B f16
                          | ((uint32_t)(kBN >> 3) << 17)  // N >> 3
                          | ((uint32_t)(kBM >> 4) << 24); // M >> 4

// MMA and commit are called by a converged warp; one elected lane issues them.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n elect.sync _|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}" ::"r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 16 consecutive f32 columns of TMEM -> 16 registers per thread.  Issue only:
// the values are valid after tcgen05.wait::ld.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
  float2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(reinterpret_cast<uint64_t&>(d))
      : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)),
        "l"(reinterpret_cast<const uint64_t&>(c)));
  return d;
}

// Four int8 -> four f16 holding the same integers: byte b becomes f16(1024 + (b ^ 0x80)),
// then 1152 is subtracted (exact at this exponent).
__device__ __forceinline__ uint2 i8x4_to_f16x4(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t lo = __byte_perm(u, 0x64646464u, 0x5140);
  const uint32_t hi = __byte_perm(u, 0x64646464u, 0x7362);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  const __half2 l = __hsub2(*reinterpret_cast<const __half2*>(&lo), bias);
  const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&hi), bias);
  uint2 r;
  r.x = *reinterpret_cast<const uint32_t*>(&l);
  r.y = *reinterpret_cast<const uint32_t*>(&h);
  return r;
}

__global__ void __launch_bounds__(kThreads, 1)
gemm_q8_0_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_dx, const uint8_t* __restrict__ W, int64_t S, int N,
                    int K, float* __restrict__ y, int M, int splits, float* __restrict__ part, uint64_t wait_ns) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN;
  const int m0 = blockIdx.y * kBM;
  const int nb = K >> 5;
  const int nstages_all = (K + kBK - 1) / kBK;
  // this CTA's stages [sbeg, sbeg + nstages): whole scale groups, split blockIdx.z of splits
  const int ngroups_all = (nstages_all + kGroupStages - 1) / kGroupStages;
  const int split = blockIdx.z;
  const int gbeg = (int)(((int64_t)ngroups_all * split) / splits);
  const int gend = (int)(((int64_t)ngroups_all * (split + 1)) / splits);
  const int sbeg = gbeg * kGroupStages;
  const int nstages = min(gend * kGroupStages, nstages_all) - sbeg;
  volatile int* abort = &sm.abort;

  if (threadIdx.x == 0) {
    s_wait_ns = wait_ns;
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 3);  // the three copies of a stage, each from its own lane
      mbar_init(&sm.consumed[i], 1);
    }
    for (int i = 0; i < kBSlots; ++i) mbar_init(&sm.bfull[i], kConvWarps);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], kEpiWarps);
    }
    mbar_init(&sm.mma_done, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // The scale tiles are zero except column 0, which the converters rewrite per block.
  {
    uint4* zx = reinterpret_cast<uint4*>(&sm.sx[0][0][0]);
    uint4* zw = reinterpret_cast<uint4*>(&sm.sw[0][0][0]);
    constexpr int kN16 = (int)(sizeof(Smem::sx) / 16);
    for (int i = threadIdx.x; i < kN16; i += kThreads) {
      zx[i] = make_uint4(0, 0, 0, 0);
      zw[i] = make_uint4(0, 0, 0, 0);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&sm.tmem_base)),
                 "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // Measured on B200: the TMA copies one thread issues complete one after another
    // (~0.4 us each up to 16 KB, however many are in flight), while copies from different
    // threads -- lanes of one warp included -- proceed side by side.  So the three copies
    // of a stage (A, int8 B, activation scales) come from three lanes, rotating over
    // kIssueTriples lane triples: each lane issues one copy every fourth stage.
    constexpr int kIssueTriples = 4;
    pdl_wait();  // activations come from the upstream quantize kernel
    int issued = 0;
    for (int s = 0; s < nstages; ++s) {
      const int st = s % kStages;
      if (s >= kStages && !warp_wait(&sm.consumed[st], ((s / kStages) - 1) & 1, abort)) break;
      const int gs = sbeg + s;
      const int l0 = 3 * (s % kIssueTriples);
      if (lane == l0) {
        mbar_expect_tx(&sm.full[st], kAStageBytes);
        tma_load_2d(sm.a[st], &map_a, gs * kBK, m0, &sm.full[st]);
      } else if (lane == l0 + 1) {
        mbar_expect_tx(&sm.full[st], kB8StageBytes);
        tma_load_2d(sm.b8[st], &map_b, gs * kBK, n0, &sm.full[st]);
      } else if (lane == l0 + 2) {
        mbar_expect_tx(&sm.full[st], kDxStageBytes);
        tma_load_2d(sm.dx[st], &map_dx, m0, 2 * gs, &sm.full[st]);
      }
      issued = s + 1;
    }
    // Every copy this CTA issued must land before it can exit (on the normal path these
    // waits return at once; after an abort they drain the copies).
    if (lane == 0) {
      for (int s = (issued > kStages ? issued - kStages : 0); s < issued; ++s)
        mbar_drain(&sm.full[s % kStages], (s / kStages) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issue ----------------
    // The whole warp runs the loop and waits; one elected lane issues each MMA and
    // commit.  Issuing from a converged warp with straight-line descriptor arithmetic
    // keeps the issue cost of one 128x128x16 MMA near its 64-cycle execution time.
    for (int s = 0; s < nstages; ++s) {
      const int st = s % kStages, bs = s % kBSlots;
      if (!warp_wait(&sm.full[st], (s / kStages) & 1, abort)) break;
      if (!warp_wait(&sm.bfull[bs], (s / kBSlots) & 1, abort)) break;
      tc_fence_after();
      const uint64_t adesc = umma_desc_sw128(sm.a[st]);
      const uint64_t bdesc = umma_desc_sw128(sm.b[bs]);
      bool stop = false;
      // block 2s + sub goes to TMEM buffer sub: I in columns [256 sub, 256 sub + 128),
      // P in the next 128.  K offsets within the 128 B swizzled row: 64 B per block,
      // 32 B per MMA.
      for (int sub = 0; sub < 2; ++sub) {
        if (2 * (sbeg + s) + sub >= nb) break;
        if (s >= 1 && !warp_wait(&sm.acc_empty[sub], (s - 1) & 1, abort)) {
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)sub * 2 * kBN;
        const uint64_t off = (uint64_t)(sub * 4);
        umma_f16(d, adesc + off, bdesc + off, 0);
        umma_f16(d, adesc + off + 2, bdesc + off + 2, 1);
        umma_f16(d + kBN, umma_desc_plain(sm.sx[bs][sub]), umma_desc_plain(sm.sw[bs][sub]), 0);
        umma_commit(&sm.acc_full[sub]);
      }
      umma_commit(&sm.consumed[st]);
      if (stop) break;
    }
    // all MMAs this warp issued have completed before TMEM is released
    umma_commit(&sm.mma_done);
    __all_sync(0xffffffffu, mbar_drain(&sm.mma_done, 0));
  } else if (warp < kEpiWarp0) {
    // ---------------- int8 -> f16 conversion, scale operands ----------------
    const int ct = threadIdx.x - 64;  // 0..127: also the weight row n0 + ct and activation row m0 + ct
    // Thread ct reads the scales of weight row n0 + ct 8 blocks (16 bytes) at a time, two
    // groups ahead of the stage being converted, so no global load latency sits on the
    // per-stage path.  A group index below ceil(nb/8) stays inside the row (its scale
    // area is padded to 16 bytes).
    // Groups are counted from this split's first one (sbeg is a multiple of 4 stages).
    const bool sload = n0 + ct < N;
    const int ngroups = (nb + 7) / 8 - gbeg;
    const uint8_t* sbase = W + (size_t)(sload ? n0 + ct : 0) * S + K + 16 * (size_t)gbeg;
    const int4 z4 = make_int4(0, 0, 0, 0);
    int4 g0 = (sload && 0 < ngroups) ? ld_stream_v4(sbase) : z4;
    int4 g1 = (sload && 1 < ngroups) ? ld_stream_v4(sbase + 16) : z4;
    int4 g2 = (sload && 2 < ngroups) ? ld_stream_v4(sbase + 32) : z4;
    const uint32_t soff = scale_tile_offset(ct);
    for (int s = 0; s < nstages && !*abort; ++s) {
      const int st = s % kStages, bs = s % kBSlots;
      if ((s & 3) == 0 && s > 0) {
        const int g = s >> 2;
        g0 = g1;
        g1 = g2;
        g2 = (sload && g + 2 < ngroups) ? ld_stream_v4(sbase + 16 * (g + 2)) : z4;
      }
      if (!mbar_wait(&sm.full[st], (s / kStages) & 1, abort)) break;
      // converted slot bs is free once the MMAs of stage s - kBSlots are done
      if (s >= kBSlots) {
        const int sp = s - kBSlots;
        if (!mbar_wait(&sm.consumed[sp % kStages], (sp / kStages) & 1, abort)) break;
      }
      // weight tile: 16-byte output chunk (8 values) per item, all loads first
      constexpr int kItems = kBN * 8 / kConvThreads;
      uint2 src[kItems];
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        const int it = ct + i * kConvThreads;
        src[i] = *reinterpret_cast<const uint2*>(sm.b8[st] + (it >> 3) * kBK + (it & 7) * 8);
      }
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        const int it = ct + i * kConvThreads, r = it >> 3, c = it & 7;
        const uint2 lo = i8x4_to_f16x4(src[i].x);
        const uint2 hi = i8x4_to_f16x4(src[i].y);
        uint8_t* dst = sm.b[bs] + r * 128 + ((c ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(lo.x, lo.y, hi.x, hi.y);
      }
      // scale operands of blocks 2s and 2s + 1: weight scales are halves 2(s%4) and
      // 2(s%4)+1 of group s/4 (raw f16 bits); activation scales are f16 values held as f32
      const int q = s & 3;
      const uint32_t two = (uint32_t)(q == 0 ? g0.x : q == 1 ? g0.y : q == 2 ? g0.z : g0.w);
      *reinterpret_cast<uint16_t*>(sm.sw[bs][0] + soff) = (uint16_t)(two & 0xffffu);
      *reinterpret_cast<uint16_t*>(sm.sw[bs][1] + soff) =
          (2 * (sbeg + s) + 1 < nb) ? (uint16_t)(two >> 16) : (uint16_t)0;
      *reinterpret_cast<__half*>(sm.sx[bs][0] + soff) = __float2half_rn(sm.dx[st][0][ct]);
      *reinterpret_cast<__half*>(sm.sx[bs][1] + soff) = __float2half_rn(sm.dx[st][1][ct]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.bfull[bs]);
    }
  } else {
    // ---------------- epilogue ----------------
    const int ew = warp - kEpiWarp0;
    const int quad = warp & 3;
    const int cg = ew >> 2;  // column group: kEpiCols columns of the tile
    const int m = m0 + quad * 32 + lane;
    const bool mvalid = m < M;
    pdl_wait();  // y may still be read by the upstream kernel; write it only after the wait
    float2 acc[kEpiCols / 2];
#pragma unroll
    for (int j = 0; j < kEpiCols / 2; ++j) acc[j] = make_float2(0.f, 0.f);
    for (int s = 0; s < nstages && !*abort; ++s) {
      for (int sub = 0; sub < 2; ++sub) {
        if (2 * (sbeg + s) + sub >= nb) break;
        if (!mbar_wait(&sm.acc_full[sub], s & 1, abort)) break;
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)sub * 2 * kBN + cg * kEpiCols;
        // 32 columns of I and of P per TMEM wait
#pragma unroll
        for (int c = 0; c < kEpiCols; c += 32) {
          float iv[32], pv[32];
          tmem_ld16_issue(taddr + c, iv);
          tmem_ld16_issue(taddr + c + 16, iv + 16);
          tmem_ld16_issue(taddr + kBN + c, pv);
          tmem_ld16_issue(taddr + kBN + c + 16, pv + 16);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if (c + 32 == kEpiCols) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[sub]);
          }
#pragma unroll
          for (int p = 0; p < 16; ++p)
            acc[c / 2 + p] = f2_fma(make_float2(iv[2 * p], iv[2 * p + 1]), make_float2(pv[2 * p], pv[2 * p + 1]),
                                    acc[c / 2 + p]);
        }
      }
    }
    const bool ok = !*abort;
    const int nbase = n0 + cg * kEpiCols;
    float* const yr = y + (size_t)m * N + nbase;
    if (splits == 1) {
      if (mvalid && ok) {
        if ((N & 3) == 0 && nbase + kEpiCols <= N) {
#pragma unroll
          for (int j = 0; j < kEpiCols / 4; ++j)
            reinterpret_cast<float4*>(yr)[j] =
                make_float4(acc[2 * j].x, acc[2 * j].y, acc[2 * j + 1].x, acc[2 * j + 1].y);
        } else {
#pragma unroll
          for (int j = 0; j < kEpiCols / 2; ++j) {
            if (nbase + 2 * j < N) yr[2 * j] = acc[j].x;
            if (nbase + 2 * j + 1 < N) yr[2 * j + 1] = acc[j].y;
          }
        }
      }
    } else if (mvalid && ok) {
      // Row r of this split's partial tile [128 rows][128 columns]; rows >= M are not
      // written (nor read by the reduction).
      const int tile = blockIdx.y * gridDim.x + blockIdx.x;
      float4* mine = reinterpret_cast<float4*>(part + (size_t)(tile * splits + split) * (kBM * kBN) +
                                               (quad * 32 + lane) * kBN + cg * kEpiCols);
#pragma unroll
      for (int j = 0; j < kEpiCols / 4; ++j)
        mine[j] = make_float4(acc[2 * j].x, acc[2 * j].y, acc[2 * j + 1].x, acc[2 * j + 1].y);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Quantize x rows for the tensor-core path: f16 integers [M][K] and transposed f32
// scales dxT[K/32][Mp] (rows padded to Mp = round_up(M, 4) so every row of the scale
// tensor starts on 16 bytes, as TMA requires).  Thread i handles block b = i / M of
// row m = i % M, so consecutive threads write consecutive scales.
__global__ void quantize_rows_f16t_kernel(const float* __restrict__ x, int M, int Mp, int K,
                                          __half* __restrict__ qh, float* __restrict__ dxT) {
  const int nb = K >> 5;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  if (i < (int64_t)M * nb) {
    const int b = (int)(i / M), m = (int)(i % M);
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)m * K + (size_t)b * kQK);
    float4 v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t);
    int q[8];
    __half dh;
    quantize_block_regs(v, q, dh);
    uint4* dst = reinterpret_cast<uint4*>(qh + (size_t)m * K + (size_t)b * kQK);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint2 a = i8x4_to_f16x4((uint32_t)q[2 * t]);
      const uint2 c = i8x4_to_f16x4((uint32_t)q[2 * t + 1]);
      dst[t] = make_uint4(a.x, a.y, c.x, c.y);
    }
    dxT[(size_t)b * Mp + m] = __half2float(dh);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------------
// Exact-halves variant (gemm_q8_0_split_kernel): no per-block rescale inside the loop.
//
// Every dequantized Q8_0 value v = q * d (q int8, d f16) has at most 8 + 11 significant
// bits, so after a power-of-two scale 2^e it is EXACTLY hi + lo with hi = f16(v 2^e) and
// lo = f16(v 2^e - hi) -- as long as both halves stay normal f16 numbers, which the scale
// ensures for every value within 2^-25 of the row's largest (smaller ones are off by at
// most 2^-25 of that largest, far below f32 rounding of the sums).  Then
//   y[m][n] = sum_k x[m][k] w[n][k] = 2^-(ea[m] + eb[n]) sum_k (xh + xl)(wh + wl)
// and sum_k (xh wh + xh wl + xl wh) differs from the exact sum only by the xl wl terms
// (each below 2^-22 of its product) and the tensor cores' f32 accumulation.  So one
// 128 x 128 tile accumulates over all of K in TMEM with three kind::f16 MMAs per 16 K
// values, and the epilogue runs once per chunk of `chunk_stages` stages (0: the whole K
// range) instead of once per 32-value block.
//   * activations: quantize_rows_split_kernel quantizes each row with candle's Q8_0 rules,
//     picks ea[m] from the row's largest block scale and writes the hi and lo planes
//     (f16 [M][K] each) and 2^-ea[m];
//   * weights: the converter warps widen the int8 tile, multiply by the block scale and
//     the row's 2^eb[n] (exact in f32) and write the hi and lo f16 tiles (128B-swizzled,
//     K-major) that the MMAs read;
//   * epilogue: y = chunk sums (f32, in chunk order) * 2^-ea[m] * 2^-eb[n] (exact).
// Rings: TMA (kSpStages): A hi + A lo + B int8; converted (kSpBSlots): B hi + B lo.
constexpr int kSpStages = 3;
constexpr int kSpBSlots = 3;
constexpr uint32_t kSpTmemCols = 2 * kBN;  // two chunk accumulators of kBN columns

struct SpSmem {
  alignas(1024) uint8_t a[kSpStages][2][kAStageBytes];  // [hi, lo] f16 tiles, swizzled
  alignas(1024) uint8_t b[kSpBSlots][2][kBStageBytes];  // [hi, lo] f16 tiles, swizzled
  alignas(128) uint8_t b8[kSpStages][kB8StageBytes];
  alignas(16) float col_scale[kBN];  // 2^-eb of each weight row of the tile
  alignas(8) uint64_t full[kSpStages];
  alignas(8) uint64_t consumed[kSpStages];
  alignas(8) uint64_t bfull[kSpBSlots];
  alignas(8) uint64_t acc_full[2];
  alignas(8) uint64_t acc_empty[2];
  alignas(8) uint64_t scales_ready;
  alignas(8) uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

// 2^e for |e| <= 126 (exact).
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }

// Scale exponent of a row whose values are q * d with |q| <= 128 and |d| <= dmax:
// 128 * dmax * 2^e < 2^15, so hi halves stay below the f16 maximum.
__device__ __forceinline__ int split_exponent(float dmax) {
  if (!(dmax > 0.0f)) return 0;
  int e;
  frexpf(dmax, &e);  // dmax = f * 2^e, 0.5 <= f < 1
  return 8 - e;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// The same halves in f16x2 arithmetic (converter warps): q as exact f16 integers,
// hi = f16(q * s) (one rounding of the exact product) and lo = fma(q, s, -hi): the fused
// f16 FMA forms q * s - hi exactly and that remainder fits an f16, so both halves equal
// the f32 route's bit for bit.  s = d * 2^e as an f16 (exact while it stays normal; a
// block whose scale is 2^-14 below f16's range is 2^-29 below the row's largest).
__device__ __forceinline__ void split8_h(uint32_t w0, uint32_t w1, __half2 s2, uint4& hi, uint4& lo) {
  const uint2 a = i8x4_to_f16x4(w0), b = i8x4_to_f16x4(w1);
  const uint32_t q[4] = {a.x, a.y, b.x, b.y};
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 qv = *reinterpret_cast<const __half2*>(&q[i]);
    const __half2 hv = __hmul2(qv, s2);
    const __half2 lv = __hfma2(qv, s2, __hneg2(hv));
    h[i] = *reinterpret_cast<const uint32_t*>(&hv);
    l[i] = *reinterpret_cast<const uint32_t*>(&lv);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Eight products q * s (q from two int8 words, s = d * 2^e) -> hi and lo f16x8.
__device__ __forceinline__ void split8(uint32_t w0, uint32_t w1, float s, uint4& hi, uint4& lo) {
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = __fmul_rn((float)(int8_t)(w0 >> (8 * i)), s);
    v[4 + i] = __fmul_rn((float)(int8_t)(w1 >> (8 * i)), s);
  }
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[i] = pack_h2(v[2 * i], v[2 * i + 1]);
    const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
    l[i] = pack_h2(__fsub_rn(v[2 * i], hf.x), __fsub_rn(v[2 * i + 1], hf.y));
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__global__ void __launch_bounds__(kThreads, 1)
gemm_q8_0_split_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                       const __grid_constant__ CUtensorMap map_b, const uint8_t* __restrict__ W, int64_t S, int N,
                       int K, const float* __restrict__ row_scale, float* __restrict__ y, int M, int splits,
                       float* __restrict__ part, int chunk_stages, uint64_t wait_ns) {
  extern __shared__ uint8_t smem_raw[];
  SpSmem& sm = *reinterpret_cast<SpSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN;
  const int m0 = blockIdx.y * kBM;
  const int nb = K >> 5;
  const int nstages_all = (K + kBK - 1) / kBK;
  const int ngroups_all = (nstages_all + kGroupStages - 1) / kGroupStages;
  const int split = blockIdx.z;
  const int gbeg = (int)(((int64_t)ngroups_all * split) / splits);
  const int gend = (int)(((int64_t)ngroups_all * (split + 1)) / splits);
  const int sbeg = gbeg * kGroupStages;
  const int nstages = min(gend * kGroupStages, nstages_all) - sbeg;
  const int cs = (chunk_stages > 0 && chunk_stages < nstages) ? chunk_stages : max(nstages, 1);
  const int nchunks = (nstages + cs - 1) / cs;
  volatile int* abort = &sm.abort;

  if (threadIdx.x == 0) {
    s_wait_ns = wait_ns;
    for (int i = 0; i < kSpStages; ++i) {
      mbar_init(&sm.full[i], 3);  // A hi, A lo, B int8: each from its own lane
      mbar_init(&sm.consumed[i], 1);
    }
    for (int i = 0; i < kSpBSlots; ++i) mbar_init(&sm.bfull[i], kConvWarps);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], kEpiWarps);
    }
    mbar_init(&sm.scales_ready, kConvWarps);
    mbar_init(&sm.mma_done, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&sm.tmem_base)),
                 "r"(kSpTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer (three lanes per stage, rotating) ----------------
    constexpr int kIssueTriples = 4;
    pdl_wait();  // the activation planes come from the upstream quantize kernel
    int issued = 0;
    for (int s = 0; s < nstages; ++s) {
      const int st = s % kSpStages;
      if (s >= kSpStages && !warp_wait(&sm.consumed[st], ((s / kSpStages) - 1) & 1, abort)) break;
      const int gs = sbeg + s;
      const int l0 = 3 * (s % kIssueTriples);
      if (lane == l0) {
        mbar_expect_tx(&sm.full[st], kAStageBytes);
        tma_load_2d(sm.a[st][0], &map_ahi, gs * kBK, m0, &sm.full[st]);
      } else if (lane == l0 + 1) {
        mbar_expect_tx(&sm.full[st], kAStageBytes);
        tma_load_2d(sm.a[st][1], &map_alo, gs * kBK, m0, &sm.full[st]);
      } else if (lane == l0 + 2) {
        mbar_expect_tx(&sm.full[st], kB8StageBytes);
        tma_load_2d(sm.b8[st], &map_b, gs * kBK, n0, &sm.full[st]);
      }
      issued = s + 1;
    }
    if (lane == 0) {
      for (int s = (issued > kSpStages ? issued - kSpStages : 0); s < issued; ++s)
        mbar_drain(&sm.full[s % kSpStages], (s / kSpStages) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issue: 3 MMAs per 16 K into the chunk's accumulator ----------------
    for (int s = 0; s < nstages; ++s) {
      const int st = s % kSpStages, bs = s % kSpBSlots;
      const int c = s / cs, buf = c & 1;
      const bool first = (s % cs) == 0;
      if (!warp_wait(&sm.full[st], (s / kSpStages) & 1, abort)) break;
      if (!warp_wait(&sm.bfull[bs], (s / kSpBSlots) & 1, abort)) break;
      if (first && c >= 2 && !warp_wait(&sm.acc_empty[buf], ((c >> 1) - 1) & 1, abort)) break;
      tc_fence_after();
      const uint64_t ah = umma_desc_sw128(sm.a[st][0]), al = umma_desc_sw128(sm.a[st][1]);
      const uint64_t bh = umma_desc_sw128(sm.b[bs][0]), bl = umma_desc_sw128(sm.b[bs][1]);
      const uint32_t d = tmem + (uint32_t)buf * kBN;
      // a stage holding one block (odd nb, last stage) has zero K values 32..63 (TMA
      // fill and zero weights): their MMAs are skipped
      const int kk_end = (2 * (sbeg + s) + 1 < nb) ? 4 : 2;
      for (int kk = 0; kk < kk_end; ++kk) {
        const uint64_t off = (uint64_t)(kk * 2);  // 32 B of a 128 B swizzled row per 16 K
        umma_f16(d, ah + off, bh + off, (first && kk == 0) ? 0u : 1u);
        umma_f16(d, ah + off, bl + off, 1u);
        umma_f16(d, al + off, bh + off, 1u);
      }
      umma_commit(&sm.consumed[st]);
      if ((s + 1) % cs == 0 || s + 1 == nstages) umma_commit(&sm.acc_full[buf]);
    }
    umma_commit(&sm.mma_done);
    __all_sync(0xffffffffu, mbar_drain(&sm.mma_done, 0));
  } else if (warp < kEpiWarp0) {
    // ---------------- weight conversion: thread ct owns weight row n0 + ct ----------------
    const int ct = threadIdx.x - 64;
    const bool rvalid = n0 + ct < N;
    const uint8_t* srow = W + (size_t)(rvalid ? n0 + ct : 0) * S + K;  // the row's f16 scales
    // the row's scale exponent from its largest block scale (8 scales per 16-byte load;
    // the scale area is padded to 16 bytes, lanes past the last block are masked)
    const int ngroups_row = (nb + 7) / 8;
    float dmax = 0.0f;
    if (rvalid) {
#pragma unroll 4
      for (int g = 0; g < ngroups_row; ++g) {
        const int4 v = ld_stream_v4(srow + 16 * g);
        const uint32_t u[4] = {(uint32_t)v.x, (uint32_t)v.y, (uint32_t)v.z, (uint32_t)v.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (8 * g + i < nb)
            dmax = fmaxf(dmax, fabsf(__half2float(__ushort_as_half((unsigned short)(u[i >> 1] >> (16 * (i & 1)))))));
      }
    }
    const int eb = split_exponent(dmax);
    const float up = exp2i(eb);
    sm.col_scale[ct] = exp2i(-eb);
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.scales_ready);
    // the stages' block scales: 8-block groups (4 stages each) loaded two groups ahead,
    // counted from this split's first group (sbeg is a multiple of 4 stages)
    const int ngroups = ngroups_row - gbeg;
    const uint8_t* sbase = srow + 16 * (size_t)gbeg;
    const int4 z4 = make_int4(0, 0, 0, 0);
    int4 g0 = (rvalid && 0 < ngroups) ? ld_stream_v4(sbase) : z4;
    int4 g1 = (rvalid && 1 < ngroups) ? ld_stream_v4(sbase + 16) : z4;
    int4 g2 = (rvalid && 2 < ngroups) ? ld_stream_v4(sbase + 32) : z4;
    for (int s = 0; s < nstages && !*abort; ++s) {
      const int st = s % kSpStages, bs = s % kSpBSlots;
      const int gb = 2 * (sbeg + s);  // first block of the stage
      if ((s & 3) == 0 && s > 0) {
        const int g = s >> 2;
        g0 = g1;
        g1 = g2;
        g2 = (rvalid && g + 2 < ngroups) ? ld_stream_v4(sbase + 16 * (g + 2)) : z4;
      }
      const int q = s & 3;
      const uint32_t two = (uint32_t)(q == 0 ? g0.x : q == 1 ? g0.y : q == 2 ? g0.z : g0.w);
      const __half2 s0 = __half2half2(
          __float2half_rn(__fmul_rn(__half2float(__ushort_as_half((unsigned short)(two & 0xffffu))), up)));
      const __half2 s1 = __half2half2(__float2half_rn(
          (gb + 1 < nb) ? __fmul_rn(__half2float(__ushort_as_half((unsigned short)(two >> 16))), up) : 0.0f));
      if (!mbar_wait(&sm.full[st], (s / kSpStages) & 1, abort)) break;
      if (s >= kSpBSlots) {
        const int sp = s - kSpBSlots;
        if (!mbar_wait(&sm.consumed[sp % kSpStages], (sp / kSpStages) & 1, abort)) break;
      }
      const uint32_t* b8row = reinterpret_cast<const uint32_t*>(sm.b8[st] + ct * kBK);
      uint8_t* dh = sm.b[bs][0] + ct * 128;
      uint8_t* dl = sm.b[bs][1] + ct * 128;
      // 8 chunks of 8 values; chunks 0-3 are block gb, 4-7 block gb + 1.  The chunk order
      // rotates with the row so that lanes read different banks.
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = (i + ct) & 7;
        const uint2 w = *reinterpret_cast<const uint2*>(b8row + 2 * c);
        uint4 hi, lo;
        split8_h(w.x, w.y, c < 4 ? s0 : s1, hi, lo);
        const int sw = (c ^ (ct & 7)) << 4;
        *reinterpret_cast<uint4*>(dh + sw) = hi;
        *reinterpret_cast<uint4*>(dl + sw) = lo;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.bfull[bs]);
    }
  } else {
    // ---------------- epilogue: chunk sums in order, then the exact 2^-(ea + eb) ----------------
    const int ew = warp - kEpiWarp0;
    const int quad = warp & 3;
    const int cg = ew >> 2;
    const int m = m0 + quad * 32 + lane;
    const bool mvalid = m < M;
    pdl_wait();  // row_scale comes from the quantize kernel; y may still be read upstream
    float acc[kEpiCols];
#pragma unroll
    for (int j = 0; j < kEpiCols; ++j) acc[j] = 0.0f;
    for (int c = 0; c < nchunks && !*abort; ++c) {
      const int buf = c & 1;
      if (!mbar_wait(&sm.acc_full[buf], (c >> 1) & 1, abort)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)buf * kBN + cg * kEpiCols;
#pragma unroll
      for (int cc = 0; cc < kEpiCols; cc += 32) {
        float v[32];
        tmem_ld16_issue(taddr + cc, v);
        tmem_ld16_issue(taddr + cc + 16, v + 16);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[cc + j] = __fadd_rn(acc[cc + j], v[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
    }
    const bool ok = !*abort && mbar_wait(&sm.scales_ready, 0, abort);
    const float rs = mvalid ? row_scale[m] : 0.0f;
#pragma unroll
    for (int j = 0; j < kEpiCols; ++j) acc[j] = __fmul_rn(acc[j], __fmul_rn(rs, sm.col_scale[cg * kEpiCols + j]));
    const int nbase = n0 + cg * kEpiCols;
    float* const yr = y + (size_t)m * N + nbase;
    if (splits == 1) {
      if (mvalid && ok) {
        if ((N & 3) == 0 && nbase + kEpiCols <= N) {
#pragma unroll
          for (int j = 0; j < kEpiCols / 4; ++j)
            reinterpret_cast<float4*>(yr)[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < kEpiCols; ++j)
            if (nbase + j < N) yr[j] = acc[j];
        }
      }
    } else if (mvalid && ok) {
      const int tile = blockIdx.y * gridDim.x + blockIdx.x;
      float4* mine = reinterpret_cast<float4*>(part + (size_t)(tile * splits + split) * (kBM * kBN) +
                                               (quad * 32 + lane) * kBN + cg * kEpiCols);
#pragma unroll
      for (int j = 0; j < kEpiCols / 4; ++j)
        mine[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kSpTmemCols) : "memory");
  }
}

// Activation rows -> Q8_0 (candle's rules) -> exact hi / lo f16 planes of q * d * 2^ea[m]
// and rs[m] = 2^-ea[m].  One CTA per row: pass 1 finds the row's largest block scale,
// pass 2 quantizes again (the row is in L2) and writes the planes.
constexpr int kSqThreads = 256;
__global__ void __launch_bounds__(kSqThreads)
quantize_rows_split_kernel(const float* __restrict__ x, int K, __half* __restrict__ ahi, __half* __restrict__ alo,
                           float* __restrict__ rs) {
  __shared__ float red[kSqThreads / 32];
  pdl_launch_dependents();  // the matmul's CTAs may become resident and start their weight work
  pdl_wait();
  const int m = blockIdx.x;
  const int nb = K >> 5;
  const float* xr = x + (size_t)m * K;
  float dmax = 0.0f;
  for (int b = threadIdx.x; b < nb; b += kSqThreads) {
    float4 v[8];
    const float4* src = reinterpret_cast<const float4*>(xr + (size_t)b * kQK);
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t);
    int q[8];
    __half dh;
    quantize_block_regs(v, q, dh);
    dmax = fmaxf(dmax, fabsf(__half2float(dh)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dmax = fmaxf(dmax, __shfl_xor_sync(0xffffffffu, dmax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = dmax;
  __syncthreads();
  dmax = 0.0f;
#pragma unroll
  for (int i = 0; i < kSqThreads / 32; ++i) dmax = fmaxf(dmax, red[i]);
  const int ea = split_exponent(dmax);
  const float up = exp2i(ea);
  if (threadIdx.x == 0) rs[m] = exp2i(-ea);
  for (int b = threadIdx.x; b < nb; b += kSqThreads) {
    float4 v[8];
    const float4* src = reinterpret_cast<const float4*>(xr + (size_t)b * kQK);
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t);
    int q[8];
    __half dh;
    quantize_block_regs(v, q, dh);
    const float sc = __fmul_rn(__half2float(dh), up);
    uint4* dhi = reinterpret_cast<uint4*>(ahi + (size_t)m * K + (size_t)b * kQK);
    uint4* dlo = reinterpret_cast<uint4*>(alo + (size_t)m * K + (size_t)b * kQK);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      uint4 hi, lo;
      split8((uint32_t)q[2 * t], (uint32_t)q[2 * t + 1], sc, hi, lo);
      dhi[t] = hi;
      dlo[t] = lo;
    }
  }
}

// y[m][n] = sum over splits, in split order, of the partial tiles the split-K matmul
// wrote: part[tile][split][128][128], tile = (m / 128) * tiles_n + n / 128.  Thread i
// sums four consecutive columns of one row (tile rows are 128 columns wide, so the
// four are always inside the partial buffer; only columns < N are stored).
__global__ void tc_split_reduce_kernel(const float* __restrict__ part, int splits, int M, int N, int tiles_n,
                                       float* __restrict__ y) {
  const int quads = tiles_n * (kBN / 4);  // column quads per row, partial-tile padded
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();  // the matmul's partials
  if (i < (int64_t)M * quads) {
    const int m = (int)(i / quads), q = (int)(i % quads);
    const int n = q * 4;
    const int tile = (m / kBM) * tiles_n + n / kBN;
    const float4* src = reinterpret_cast<const float4*>(part + (size_t)tile * splits * (kBM * kBN) +
                                                        (m % kBM) * kBN + n % kBN);
    float4 t = src[0];
    for (int sp = 1; sp < splits; ++sp) {
      const float4 v = src[(size_t)sp * (kBM * kBN / 4)];
      t.x += v.x;
      t.y += v.y;
      t.z += v.z;
      t.w += v.w;
    }
    float* yr = y + (size_t)m * N + n;
    if ((N & 3) == 0 && n + 4 <= N) {
      *reinterpret_cast<float4*>(yr) = t;
    } else {
      if (n < N) yr[0] = t.x;
      if (n + 1 < N) yr[1] = t.y;
      if (n + 2 < N) yr[2] = t.z;
      if (n + 3 < N) yr[3] = t.w;
    }
  }
  pdl_launch_dependents();
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType type, void* base, uint64_t d0, uint64_t d1,
               uint64_t stride1_bytes, uint32_t b0, uint32_t b1, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {d0, d1};
  const cuuint64_t strides[1] = {stride1_bytes};
  const cuuint32_t box[2] = {b0, b1};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, type, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline int64_t padded_rows(int64_t m) { return (m + 3) / 4 * 4; }
inline size_t up256(size_t v) { return (v + 255) / 256 * 256; }

// Split count for a (M, N, K) problem: enough CTAs for one wave of kSplitMaxCtas when the
// output has fewer than half that many tiles, each split at least one scale group.
int tc_splits(int M, int N, int K) {
  const int tiles = ((N + kBN - 1) / kBN) * ((M + kBM - 1) / kBM);
  if (2 * tiles > kSplitMaxCtas) return 1;
  const int ngroups = ((K + kBK - 1) / kBK + kGroupStages - 1) / kGroupStages;
  int splits = kSplitMaxCtas / tiles;
  if (splits > ngroups) splits = ngroups;
  return splits < 1 ? 1 : splits;
}

}  // namespace

size_t gemm_tc_smem_bytes() { return sizeof(Smem) + 1024; }

// Which f16 tensor-core kernel serves M > 32: the per-block rescale kernel (default,
// faster on B200: gate_up 2048 -> 12288 at M = 4096 in 752 us against 1047 us) or the
// exact-halves kernel (Q8LIN_F16_GEMM=split).  Read once.
bool f16_split_enabled() {
  static const bool on = [] {
    const char* v = getenv("Q8LIN_F16_GEMM");
    return v && v[0] == 's';
  }();
  return on;
}
// Stages per TMEM chunk of the exact-halves kernel.  The tensor cores' f32 accumulation
// over one long K range loses accuracy (measured against the oracle: rel-L2 7e-6 at
// K = 2048 and 2.1e-5 at K = 6144 in one chunk); chunks of 4 stages (256 K values) added
// on the CUDA cores keep it near 1e-6 at every K.  Q8LIN_SPLIT_CHUNK overrides (0: one
// chunk).
int split_chunk_stages() {
  static const int c = [] {
    const char* v = getenv("Q8LIN_SPLIT_CHUNK");
    return v ? atoi(v) : 4;
  }();
  return c;
}

// per-block kernel: [qh f16 M x K][dxT f32 nb x Mp][split partials: one wave of tiles];
// exact-halves kernel: [a_hi f16 M x K][a_lo f16 M x K][2^-ea f32 M][split partials]
size_t gemm_tc_workspace_bytes(int64_t m, int64_t k) {
  const size_t partials = (size_t)kSplitMaxCtas * kBM * kBN * 4;
  if (f16_split_enabled()) return 2 * up256((size_t)(m * k) * 2) + up256((size_t)m * 4) + partials;
  const size_t qh = up256((size_t)(m * k) * 2);
  const size_t dx = up256((size_t)(padded_rows(m) * (k / kQK)) * 4);
  return qh + dx + partials;
}

static cudaError_t launch_gemm_split(const q8lin_weight& w, const float* x, void* workspace, float* y, int64_t m,
                                     cudaStream_t s) {
  const int M = (int)m, K = (int)w.k, N = (int)w.n;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t plane = up256((size_t)M * K * 2);
  __half* ahi = reinterpret_cast<__half*>(ws);
  __half* alo = reinterpret_cast<__half*>(ws + plane);
  float* rs = reinterpret_cast<float*>(ws + 2 * plane);
  float* part = reinterpret_cast<float*>(ws + 2 * plane + up256((size_t)M * 4));
  const int splits = tc_splits(M, N, K);

  CUtensorMap map_ahi, map_alo, map_b;
  if (!encode_2d(&map_ahi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ahi, K, M, (uint64_t)K * 2, kBK, kBM,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&map_alo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, alo, K, M, (uint64_t)K * 2, kBK, kBM,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.packed, K, N, (uint64_t)w.row_stride, kBK, kBN,
                 CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)M);
    cfg.blockDim = dim3(kSqThreads);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, quantize_rows_split_kernel, x, K, ahi, alo, rs);
    if (e != cudaSuccess) return e;
  }
  const size_t smem = sizeof(SpSmem) + 1024;
  static int configured[128] = {0};
  {
    cudaError_t e = ensure_smem((const void*)gemm_q8_0_split_kernel, configured, w.device, smem, false);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + kBN - 1) / kBN), (unsigned)((M + kBM - 1) / kBM), (unsigned)splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_q8_0_split_kernel, map_ahi, map_alo, map_b,
                                     (const uint8_t*)w.packed, w.row_stride, N, K, (const float*)rs, y, M, splits,
                                     part, split_chunk_stages(), wait_limit_ns());
  if (e != cudaSuccess || splits == 1) return e;
  const int tiles_n = (N + kBN - 1) / kBN;
  const int64_t work = (int64_t)M * tiles_n * (kBN / 4);
  cudaLaunchConfig_t rcfg = {};
  rcfg.gridDim = dim3((unsigned)((work + 255) / 256));
  rcfg.blockDim = dim3(256);
  rcfg.stream = s;
  rcfg.attrs = attr;
  rcfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&rcfg, tc_split_reduce_kernel, (const float*)part, splits, M, N, tiles_n, y);
}

cudaError_t launch_gemm_tc(const q8lin_weight& w, const float* x, void* workspace, float* y, int64_t m,
                           cudaStream_t s) {
  if (f16_split_enabled()) return launch_gemm_split(w, x, workspace, y, m, s);
  const int M = (int)m, K = (int)w.k, N = (int)w.n;
  const int Mp = (int)padded_rows(m);
  const int nb = K / kQK;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __half* qh = reinterpret_cast<__half*>(ws);
  float* dxT = reinterpret_cast<float*>(ws + up256((size_t)M * K * 2));
  float* part = reinterpret_cast<float*>(ws + up256((size_t)M * K * 2) + up256((size_t)Mp * nb * 4));
  const int splits = tc_splits(M, N, K);

  CUtensorMap map_a, map_b, map_dx;
  if (!encode_2d(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, qh, K, M, (uint64_t)K * 2, kBK, kBM,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.packed, K, N, (uint64_t)w.row_stride, kBK, kBN,
                 CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(&map_dx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dxT, M, nb, (uint64_t)Mp * 4, kBM, 2,
                 CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;

  // 1. quantize
  {
    const int64_t work = (int64_t)M * nb;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((work + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, quantize_rows_f16t_kernel, x, M, Mp, K, qh, dxT);
    if (e != cudaSuccess) return e;
  }
  // 2. tensor-core matmul
  const size_t smem = gemm_tc_smem_bytes();
  static int configured[128] = {0};
  {
    cudaError_t e = ensure_smem((const void*)gemm_q8_0_tc_kernel, configured, w.device, smem, false);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + kBN - 1) / kBN), (unsigned)((M + kBM - 1) / kBM), (unsigned)splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_q8_0_tc_kernel, map_a, map_b, map_dx, (const uint8_t*)w.packed,
                                     w.row_stride, N, K, y, M, splits, part, wait_limit_ns());
  if (e != cudaSuccess || splits == 1) return e;
  // 3. split-K: add the partials
  const int tiles_n = (N + kBN - 1) / kBN;
  const int64_t work = (int64_t)M * tiles_n * (kBN / 4);
  cudaLaunchConfig_t rcfg = {};
  rcfg.gridDim = dim3((unsigned)((work + 255) / 256));
  rcfg.blockDim = dim3(256);
  rcfg.stream = s;
  rcfg.attrs = attr;
  rcfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&rcfg, tc_split_reduce_kernel, (const float*)part, splits, M, N, tiles_n, y);
}

cudaError_t read_tc_fault(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_tc_fault, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_tc_fault, &z, sizeof(z));
  }
  return e;
}

}  // namespace q8lin
