// Q8_0 matmul for small batches (M <= 32) on the tensor cores with int8 MMAs.
//
// y[m][n] = sum_b dx[m][b] * dw[n][b] * I[n][m][b],  I = exact int dot of one 32-value
// block.  With few activation rows the matmul is a weight stream (HBM-bound), so the
// weights take the MMA's 128-row side and the activations the narrow side:
//   * A = 128 weight rows x 128 K bytes, int8 straight from the packed plane by TMA
//     (128B swizzle) -- no conversion;
//   * B = Np activation rows (M rounded up to 16) x 128 K bytes of the Q8_0-quantized
//     x, int8, by TMA;
//   * one tcgen05.mma kind::i8 (M = 128, N = Np, K = 32) per Q8_0 block writes the
//     block's int32 dot products to its own TMEM buffer (Np columns);
//   * epilogue warps (one TMEM lane = one weight row each) add the block terms in block
//     order exactly as candle's scalar vec_dot does: acc += (f32(I) * dw) * dx, every
//     product rounded, the weight scale held in a register and the Np activation scales
//     of the block read from shared memory.  A CTA that covers the whole K therefore
//     reproduces the CPU result bit for bit.
// Split-K: when the weight has too few 128-row tiles to occupy the SMs, grid.y splits
// the blocks; each CTA writes its partial sums to the workspace and a second kernel
// (skinny_split_reduce_kernel, all SMs) adds the partials in split order --
// deterministic, no atomics.
//
// A stage is 4 blocks (128 K bytes).  Warp roles (192 threads):
//   warp 0      TMA producer (weights, activations, activation scales)
//   warp 1      TMEM allocation and MMA issue (converged warp, one elected lane)
//   warps 2-5   epilogue: TMEM lane quadrant warp % 4
// The operand slot of a stage is released by the MMA commit and by the four epilogue
// warps (which read its activation scales).  Every wait is bounded; on timeout bit 2 of
// the fault word is set and the CTA drains and returns.
#include <cuda.h>

#include "common.cuh"
#include "internal.h"

namespace q8lin {

__device__ unsigned int g_skinny_fault;

namespace {

constexpr int kRows = 128;
constexpr int kBlocksPerStage = 4;
constexpr int kStageK = kBlocksPerStage * kQK;  // 128 bytes of K
constexpr int kStages = 6;
constexpr int kMaxNp = kSkinnyMaxM;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxTbufs = 8;
constexpr int kTargetCtas = 148;

constexpr int kAStageBytes = kRows * kStageK;     // 16 KB
constexpr int kBStageBytes = kMaxNp * kStageK;    //  8 KB at Np = 64
constexpr int kDxStageFloats = kBlocksPerStage * kMaxNp;

struct Smem {
  alignas(1024) uint8_t a[kStages][kAStageBytes];
  alignas(1024) uint8_t b[kStages][kBStageBytes];
  alignas(16) float dx[kStages][kDxStageFloats];  // [block of stage][m], Np per block
  alignas(8) uint64_t full[kStages];
  alignas(8) uint64_t consumed[kStages];  // MMA commit + kEpiWarps epilogue arrivals
  alignas(8) uint64_t acc_full[kMaxTbufs];
  alignas(8) uint64_t acc_empty[kMaxTbufs];
  alignas(8) uint64_t mma_done;
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
  atomicOr(&g_skinny_fault, 4u);
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
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  return __all_sync(0xffffffffu, mbar_wait(b, parity, abort));
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(su32(bar))
      : "memory");
}

// K-major, 128B-swizzled UMMA shared-memory descriptor (8-row atoms of 128 B).
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* base) {
  const uint64_t addr = su32(base);
  return ((addr >> 4) & 0x3FFFull) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)2 << 61);
}

// kind::i8 MMA (signed int8 x signed int8 -> int32), issued by one elected lane of a
// converged warp.  idesc: D s32, A and B s8, K-major, N = Np, M = 128.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
  // enable-input-d false: every block writes a fresh int32 result
  asm volatile(
      "{\n .reg .pred p, e;\n elect.sync _|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(0u)
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

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

struct Params {
  const uint8_t* W;  // packed plane (for the weight scales)
  int64_t S;
  int N, K, M, Np;
  int splits, tbufs;
  uint32_t idesc;
  float* y;
  float* part;       // [tile][split][Np][128] partial sums (splits > 1)
  uint64_t wait_ns;  // limit of the bounded waits (q8lin_set_wait_limit_ns)
};

template <int NP>
__global__ void __launch_bounds__(kThreads, 1)
gemm_q8_0_skinny_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                        const __grid_constant__ CUtensorMap map_dx, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n0 = tile * kRows;
  const int nb = p.K / kQK;
  const int b0 = (int)(((int64_t)nb * split) / p.splits);
  const int b1 = (int)(((int64_t)nb * (split + 1)) / p.splits);
  const int nst = (b1 - b0 + kBlocksPerStage - 1) / kBlocksPerStage;
  volatile int* abort = &sm.abort;

  if (threadIdx.x == 0) {
    s_wait_ns = p.wait_ns;
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 3);  // the three copies of a stage, each from its own lane
      mbar_init(&sm.consumed[i], 1 + kEpiWarps);
    }
    for (int i = 0; i < kMaxTbufs; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], kEpiWarps);
    }
    mbar_init(&sm.mma_done, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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
    // The TMA copies one thread issues complete one after another (measured on B200:
    // ~0.4 us each up to 16 KB), copies from different lanes side by side: the three
    // copies of a stage come from three lanes, rotating over four lane triples.
    constexpr int kIssueTriples = 4;
    pdl_wait();  // the quantized activations come from the upstream kernel
    int issued = 0;
    for (int s = 0; s < nst; ++s) {
      const int st = s % kStages;
      if (s >= kStages && !warp_wait(&sm.consumed[st], ((s / kStages) - 1) & 1, abort)) break;
      const int kb = (b0 + s * kBlocksPerStage) * kQK;
      const int l0 = 3 * (s % kIssueTriples);
      if (lane == l0) {
        mbar_expect_tx(&sm.full[st], kAStageBytes);
        tma_load_2d(sm.a[st], &map_w, kb, n0, &sm.full[st]);
      } else if (lane == l0 + 1) {
        mbar_expect_tx(&sm.full[st], NP * kStageK);
        tma_load_2d(sm.b[st], &map_x, kb, 0, &sm.full[st]);
      } else if (lane == l0 + 2) {
        mbar_expect_tx(&sm.full[st], kBlocksPerStage * NP * 4);
        tma_load_2d(sm.dx[st], &map_dx, 0, b0 + s * kBlocksPerStage, &sm.full[st]);
      }
      issued = s + 1;
    }
    if (lane == 0) {
      for (int s = (issued > kStages ? issued - kStages : 0); s < issued; ++s)
        mbar_drain(&sm.full[s % kStages], (s / kStages) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issue ----------------
    for (int s = 0; s < nst; ++s) {
      const int st = s % kStages, tb = s % p.tbufs;
      if (!warp_wait(&sm.full[st], (s / kStages) & 1, abort)) break;
      if (s >= p.tbufs && !warp_wait(&sm.acc_empty[tb], ((s / p.tbufs) - 1) & 1, abort)) break;
      tc_fence_after();
      const uint64_t ad = umma_desc_sw128(sm.a[st]);
      const uint64_t bd = umma_desc_sw128(sm.b[st]);
#pragma unroll
      for (int j = 0; j < kBlocksPerStage; ++j) {
        if (b0 + s * kBlocksPerStage + j >= b1) break;
        // block j: 32 bytes along K within the 128 B swizzled rows
        umma_i8(tmem + (uint32_t)((tb * kBlocksPerStage + j) * NP), ad + (uint64_t)(2 * j), bd + (uint64_t)(2 * j),
                p.idesc);
      }
      umma_commit(&sm.acc_full[tb]);
      umma_commit(&sm.consumed[st]);
    }
    umma_commit(&sm.mma_done);
    __all_sync(0xffffffffu, mbar_drain(&sm.mma_done, 0));
  } else {
    // ---------------- epilogue ----------------
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // row within the tile = TMEM lane
    const int n = n0 + r;
    const bool nvalid = n < p.N;
    // weight scales of row n, 8 blocks (16 bytes) per group, two groups ahead; a group
    // index below ceil(nb/8) stays inside the row's padded scale area
    const uint8_t* sbase = p.W + (size_t)(nvalid ? n : 0) * p.S + p.K;
    const int ng = (nb + 7) / 8;
    const int4 z4 = make_int4(0, 0, 0, 0);
    int g_lo = b0 >> 3;
    int4 g0 = (nvalid && g_lo < ng) ? ld_stream_v4(sbase + 16 * g_lo) : z4;
    int4 g1 = (nvalid && g_lo + 1 < ng) ? ld_stream_v4(sbase + 16 * (g_lo + 1)) : z4;
    int4 g2 = (nvalid && g_lo + 2 < ng) ? ld_stream_v4(sbase + 16 * (g_lo + 2)) : z4;
    pdl_wait();  // y and the workspace may still be in use upstream
    float acc[NP];
#pragma unroll
    for (int m = 0; m < NP; ++m) acc[m] = 0.0f;
    for (int s = 0; s < nst && !*abort; ++s) {
      const int st = s % kStages, tb = s % p.tbufs;
      if (!mbar_wait(&sm.acc_full[tb], (s / p.tbufs) & 1, abort)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(tb * kBlocksPerStage * NP);
#pragma unroll
      for (int j = 0; j < kBlocksPerStage; ++j) {
        const int b = b0 + s * kBlocksPerStage + j;
        if (b >= b1) break;
        while ((b >> 3) > g_lo) {  // advance the scale groups
          ++g_lo;
          g0 = g1;
          g1 = g2;
          g2 = (nvalid && g_lo + 2 < ng) ? ld_stream_v4(sbase + 16 * (g_lo + 2)) : z4;
        }
        const int q = (b & 7) >> 1;
        const uint32_t two = (uint32_t)(q == 0 ? g0.x : q == 1 ? g0.y : q == 2 ? g0.z : g0.w);
        const float dw = __half2float(__ushort_as_half((unsigned short)((b & 1) ? (two >> 16) : (two & 0xffff))));
        int iv[NP];
#pragma unroll
        for (int c = 0; c < NP; c += 16) tmem_ld16(taddr + (uint32_t)(j * NP + c), iv + c);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const float* dxb = &sm.dx[st][j * NP];
#pragma unroll
        for (int m = 0; m < NP; m += 4) {
          const float4 d4 = *reinterpret_cast<const float4*>(dxb + m);  // same 16 bytes for every lane
          acc[m] = __fadd_rn(acc[m], __fmul_rn(__fmul_rn(__int2float_rn(iv[m]), dw), d4.x));
          acc[m + 1] = __fadd_rn(acc[m + 1], __fmul_rn(__fmul_rn(__int2float_rn(iv[m + 1]), dw), d4.y));
          acc[m + 2] = __fadd_rn(acc[m + 2], __fmul_rn(__fmul_rn(__int2float_rn(iv[m + 2]), dw), d4.z));
          acc[m + 3] = __fadd_rn(acc[m + 3], __fmul_rn(__fmul_rn(__int2float_rn(iv[m + 3]), dw), d4.w));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.acc_empty[tb]);
        mbar_arrive(&sm.consumed[st]);  // done with the stage's activation scales
      }
    }
    const bool ok = !*abort;
    if (p.splits == 1) {
      if (ok && nvalid) {
#pragma unroll
        for (int m = 0; m < NP; ++m)
          if (m < p.M) p.y[(size_t)m * p.N + n] = acc[m];
      }
    } else {
      float* mine = p.part + ((size_t)(tile * p.splits + split) * NP) * kRows;
      if (ok) {
#pragma unroll
        for (int m = 0; m < NP; ++m)
          if (m < p.M) mine[(size_t)m * kRows + r] = acc[m];
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Activations -> Q8_0 for the int8 path: qx int8 [M][K] and transposed f32 scales
// dxT[K/32][Mp] (Mp = M rounded up to 16).
__global__ void quantize_rows_i8t_kernel(const float* __restrict__ x, int M, int Mp, int K, int8_t* __restrict__ qx,
                                         float* __restrict__ dxT) {
  const int nb = K >> 5;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();
  if (i < (int64_t)Mp * nb) {
    const int b = (int)(i / Mp), m = (int)(i % Mp);
    if (m < M) {
      const float4* src = reinterpret_cast<const float4*>(x + (size_t)m * K + (size_t)b * kQK);
      float4 v[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t);
      int q[8];
      __half dh;
      quantize_block_regs(v, q, dh);
      int4* dst = reinterpret_cast<int4*>(qx + (size_t)m * K + (size_t)b * kQK);
      dst[0] = make_int4(q[0], q[1], q[2], q[3]);
      dst[1] = make_int4(q[4], q[5], q[6], q[7]);
      dxT[(size_t)b * Mp + m] = __half2float(dh);
    } else {
      dxT[(size_t)b * Mp + m] = 0.0f;
    }
  }
}

// y[m][n] = sum over splits, in split order, of the split-K partials
// part[tile][split][Np][128] (tile = n / 128); one thread per output, consecutive
// threads on consecutive n.
__global__ void skinny_split_reduce_kernel(const float* __restrict__ part, int splits, int Np, int M, int N,
                                           float* __restrict__ y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_launch_dependents();  // dependents may become resident now; they wait for this grid
  pdl_wait();  // the matmul's partials
  if (i < (int64_t)M * N) {
    const int m = (int)(i / N), n = (int)(i % N);
    const float* src = part + ((size_t)(n / kRows) * splits * Np + m) * kRows + (n % kRows);
    float sum = src[0];
    for (int sp = 1; sp < splits; ++sp) sum += src[(size_t)sp * Np * kRows];
    y[i] = sum;
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(ptr);
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

inline int np_of(int64_t m) { return (int)((m + 15) / 16 * 16); }
inline size_t up256(size_t v) { return (v + 255) / 256 * 256; }
constexpr int kMaxCtasWs = 2 * kTargetCtas;  // bound on tiles x splits when splits > 1

template <int NP>
cudaError_t launch_np(const CUtensorMap& mw, const CUtensorMap& mx, const CUtensorMap& md, const Params& p,
                      int tiles, int dev, cudaStream_t s) {
  const size_t smem = sizeof(Smem) + 1024;
  static int configured[128] = {0};
  cudaError_t e0 = ensure_smem((const void*)gemm_q8_0_skinny_kernel<NP>, configured, dev, smem, false);
  if (e0 != cudaSuccess) return e0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)tiles, (unsigned)p.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemm_q8_0_skinny_kernel<NP>, mw, mx, md, p);
}

}  // namespace

cudaError_t launch_quantize_rows_i8t(const float* x, int M, int Mp, int K, int8_t* qx, float* dxT, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const int64_t work = (int64_t)Mp * (K / kQK);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((work + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, quantize_rows_i8t_kernel, x, M, Mp, K, qx, dxT);
}

size_t gemm_skinny_workspace_bytes(int64_t m, int64_t k) {
  const int Np = np_of(m);
  const int64_t nb = k / kQK;
  return up256((size_t)(m * k)) + up256((size_t)Np * nb * 4) + (size_t)kMaxCtasWs * Np * kRows * 4;
}

cudaError_t launch_gemm_skinny(const q8lin_weight& w, const float* x, void* workspace, float* y, int64_t m,
                               cudaStream_t s) {
  const int M = (int)m, K = (int)w.k, N = (int)w.n, Np = np_of(m);
  const int nb = K / kQK;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int8_t* qx = reinterpret_cast<int8_t*>(ws);
  float* dxT = reinterpret_cast<float*>(ws + up256((size_t)M * K));
  float* part = reinterpret_cast<float*>(ws + up256((size_t)M * K) + up256((size_t)Np * nb * 4));

  const int tiles = (N + kRows - 1) / kRows;
  int splits = (kTargetCtas + tiles / 2) / tiles;
  if (splits > nb / 8) splits = nb / 8;
  if (splits < 1) splits = 1;
  if (tiles * splits > kMaxCtasWs) splits = kMaxCtasWs / tiles;
  if (splits < 1) splits = 1;

  Params p;
  p.W = static_cast<const uint8_t*>(w.packed);
  p.S = w.row_stride;
  p.N = N;
  p.K = K;
  p.M = M;
  p.Np = Np;
  p.splits = splits;
  p.tbufs = (int)(kTmemCols / (kBlocksPerStage * Np));
  if (p.tbufs > kMaxTbufs) p.tbufs = kMaxTbufs;
  p.idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(Np >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
  p.y = y;
  p.part = part;
  p.wait_ns = wait_limit_ns();

  CUtensorMap mw, mx, md;
  if (!encode_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.packed, K, N, (uint64_t)w.row_stride, kStageK, kRows,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_UINT8, qx, K, M, (uint64_t)K, kStageK, Np, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dxT, Np, nb, (uint64_t)Np * 4, Np, kBlocksPerStage,
                 CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  {
    const int64_t work = (int64_t)Np * nb;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((work + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, quantize_rows_i8t_kernel, x, M, Np, K, qx, dxT);
    if (e != cudaSuccess) return e;
  }
  const int dev = (w.device >= 0 && w.device < 128) ? w.device : 0;
  static_assert(kMaxNp == 32, "instantiations below cover Np = 16 and 32");
  cudaError_t e;
  switch (Np) {
    case 16: e = launch_np<16>(mw, mx, md, p, tiles, dev, s); break;
    case 32: e = launch_np<32>(mw, mx, md, p, tiles, dev, s); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess || splits == 1) return e;
  // split-K: add the partials
  const int64_t outs = (int64_t)M * N;
  cudaLaunchConfig_t rcfg = {};
  rcfg.gridDim = dim3((unsigned)((outs + 255) / 256));
  rcfg.blockDim = dim3(256);
  rcfg.stream = s;
  rcfg.attrs = attr;
  rcfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&rcfg, skinny_split_reduce_kernel, (const float*)part, splits, Np, M, N, y);
}

cudaError_t read_skinny_fault(unsigned int* flags, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_skinny_fault, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_skinny_fault, &z, sizeof(z));
  }
  return e;
}

}  // namespace q8lin
