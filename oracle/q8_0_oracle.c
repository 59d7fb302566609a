/*
 * q8_0_oracle.c -- CPU restatement of candle-core 0.11.0's CPU Q8_0 quantized matmul.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path in
 * talechime_b200/csrc; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it.  The product library never
 * links or calls it.
 *
 * What it restates
 * ----------------
 * talechime's VoxCPM BaseLM keeps every Q8_0 GGUF projection as
 * `QMatMul::QTensor(Arc<QTensor>)` (crates/voxcpm/src/weights.rs:98-117) and calls
 * `QMatMul::forward(&x[rows, in])` from `Linear::forward`
 * (crates/voxcpm/src/weights.rs:213-229).  The arithmetic lives in the third-party
 * crate candle-core 0.11.0 (workspace pin Cargo.toml:20, fork rev
 * 884b359895a16c8fbd3647789b1f7c7974894708 at Cargo.toml:94-98; its patches are
 * Metal-only, so the CPU quantized code is upstream 0.11.0).  Candle's source is not
 * part of the reference tree; what follows restates its published algorithm:
 *
 *   Q8_0 block (GGUF/ggml format): 34 bytes = { f16 d (little endian); int8 qs[32] }.
 *   dequantize:  x[j] = f32(qs[j]) * f32(d)
 *   quantize (BlockQ8_0::from_float, used for both GGUF weights and the f32
 *   activations of the matmul):
 *       amax = max_j |x[j]|           (f32 max; a NaN element is skipped)
 *       d    = amax / 127             (f32 division, correctly rounded)
 *       id   = d != 0 ? 1 / d : 0     (reciprocal of the f32 d, *before* f16 rounding)
 *       qs[j]= (int8) round(x[j]*id)  (product rounded to f32, then round half away
 *                                      from zero; the float->int8 cast saturates and
 *                                      maps NaN to 0, as Rust's `as i8` does)
 *       d is stored as f16, round to nearest even.
 *   matmul (k_quants::matmul): every activation row is quantized with from_float,
 *   then for each output y[m][n] = BlockQ8_0::vec_dot(K, W row n, x row m).
 *   talechime builds x86_64 without AVX target features (.cargo/config.toml has no
 *   rustflags; skills/candle-performance/references/windows-cpu.md:55-58 notes that
 *   candle's own cpu::avx is gated on target_feature=avx2 at compile time), so the
 *   shipped vec_dot is the scalar `vec_dot_unopt`:
 *       sumf = 0
 *       for b in 0..K/32:  isum = sum_j qw[j]*qx[j]             (exact int32)
 *                          sumf = sumf + (f32(isum) * dw) * dx   (f32, no FMA)
 *   This file follows that order exactly (built with -ffp-contract=off).
 *   aarch64 builds use candle's NEON vec_dot, which only reorders the f32 sum.
 *
 * Parity pinning
 * --------------
 * The quantize / dequantize / f16 rules are pinned bit-exactly against the
 * independent numpy implementation in the `gguf` Python package 0.19.0
 * (gguf.quants.Q8_0), which states bit-exactness with ggml-quants.c's reference
 * quantizer: see tests/golden/make_golden.py and tests/test_oracle_golden.py.
 * The matmul summation order is pinned against an independent numpy restatement
 * of the scalar loop (same fixtures).  candle itself cannot be run here (no Rust
 * toolchain, no candle source), so agreement with candle's binary is by restated
 * semantics, not by execution.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK8_0 32
#define Q8_0_BLOCK_BYTES 34

/* ---------- IEEE binary16 <-> binary32, written from the format definition ---------- */

uint16_t q8o_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) { /* inf / nan: keep a quiet-nan payload bit */
    if (ax == 0x7f800000u) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
  }
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 -> inf */
  if (ax < 0x38800000u) {                                    /* below 2^-14: subnormal */
    if (ax < 0x33000000u) return (uint16_t)sign;             /* <= 2^-25 -> 0 */
    const uint32_t e = ax >> 23;                             /* 102..112 */
    const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e;                         /* 14..24 */
    uint32_t q = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t r = ax - 0x38000000u; /* rebias exponent 127 -> 15 */
  r += 0x0fffu + ((r >> 13) & 1u);
  return (uint16_t)(sign | (r >> 13));
}

float q8o_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  const uint32_t m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else {
      float v = (float)m * 5.9604644775390625e-08f; /* m * 2^-24, exact */
      memcpy(&x, &v, 4);
      x |= sign;
    }
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

/* Rust `f32 as i8`: saturating, NaN -> 0. */
static int8_t sat_i8(float v) {
  if (v != v) return 0;
  if (v >= 127.0f) return 127;
  if (v <= -128.0f) return -128;
  return (int8_t)v;
}

/* Rust f32::max: returns the non-NaN operand when one is NaN. */
static float rust_fmax(float a, float b) {
  if (a != a) return b;
  if (b != b) return a;
  return a > b ? a : b;
}

/* One Q8_0 block from 32 floats; writes d (as f16 bits) and qs. */
static void quantize_block(const float* x, uint16_t* d_out, int8_t* qs) {
  float amax = 0.0f;
  for (int j = 0; j < QK8_0; ++j) amax = rust_fmax(amax, fabsf(x[j]));
  const float d = amax / 127.0f;
  const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
  *d_out = q8o_f32_to_f16(d);
  for (int j = 0; j < QK8_0; ++j) {
    const float p = x[j] * id;
    qs[j] = sat_i8(roundf(p));
  }
}

/* Quantize k floats into GGUF-layout Q8_0 blocks (k % 32 == 0). */
int q8o_quantize_row(const float* x, int64_t k, uint8_t* blocks) {
  if (k < 0 || k % QK8_0) return 1;
  for (int64_t b = 0; b < k / QK8_0; ++b) {
    uint16_t d;
    int8_t qs[QK8_0];
    quantize_block(x + b * QK8_0, &d, qs);
    uint8_t* o = blocks + b * Q8_0_BLOCK_BYTES;
    o[0] = (uint8_t)(d & 0xff);
    o[1] = (uint8_t)(d >> 8);
    memcpy(o + 2, qs, QK8_0);
  }
  return 0;
}

/* Quantize rows into separate planes: qs [m][k] int8 and d [m][k/32] f16 bits. */
int q8o_quantize_planes(const float* x, int64_t m, int64_t k, int8_t* qs, uint16_t* d) {
  if (m < 0 || k < 0 || k % QK8_0) return 1;
  const int64_t nb = k / QK8_0;
  for (int64_t r = 0; r < m; ++r)
    for (int64_t b = 0; b < nb; ++b)
      quantize_block(x + r * k + b * QK8_0, d + r * nb + b, qs + r * k + b * QK8_0);
  return 0;
}

/* Dequantize GGUF-layout Q8_0 blocks to k floats. */
int q8o_dequantize_row(const uint8_t* blocks, int64_t k, float* y) {
  if (k < 0 || k % QK8_0) return 1;
  for (int64_t b = 0; b < k / QK8_0; ++b) {
    const uint8_t* o = blocks + b * Q8_0_BLOCK_BYTES;
    const float d = q8o_f16_to_f32((uint16_t)(o[0] | (o[1] << 8)));
    for (int j = 0; j < QK8_0; ++j) y[b * QK8_0 + j] = (float)(int8_t)o[2 + j] * d;
  }
  return 0;
}

/* ---------- matmul: y[m][n] = vec_dot_unopt(W row n, Q8_0(x row m)) ---------- */

typedef struct {
  const uint8_t* w;  /* N rows of K/32 GGUF blocks */
  const int8_t* qx;  /* [M][K] */
  const float* dx;   /* [M][K/32] (f32 widened f16) */
  float* y;          /* [M][N] */
  int64_t m, n, k, n0, n1;
} mm_job;

static void* mm_worker(void* arg) {
  const mm_job* j = (const mm_job*)arg;
  const int64_t nb = j->k / QK8_0;
  for (int64_t col = j->n0; col < j->n1; ++col) {
    const uint8_t* wrow = j->w + col * nb * Q8_0_BLOCK_BYTES;
    for (int64_t r = 0; r < j->m; ++r) {
      const int8_t* xr = j->qx + r * j->k;
      const float* dxr = j->dx + r * nb;
      float sumf = 0.0f;
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = wrow + b * Q8_0_BLOCK_BYTES;
        const float dw = q8o_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        const int8_t* qw = (const int8_t*)(blk + 2);
        const int8_t* qx = xr + b * QK8_0;
        int32_t isum = 0;
        for (int t = 0; t < QK8_0; ++t) isum += (int32_t)qw[t] * (int32_t)qx[t];
        const float term = ((float)isum * dw) * dxr[b];
        sumf = sumf + term;
      }
      j->y[r * j->n + col] = sumf;
    }
  }
  return NULL;
}

/*
 * x: f32 [m][k] row-major; w: n rows of k/32 GGUF Q8_0 blocks; y: f32 [m][n].
 * threads <= 1 runs on the calling thread; otherwise columns are split across
 * `threads` pthreads (candle splits columns across its rayon pool the same way;
 * the per-output arithmetic does not depend on the split).
 * Returns 0 on success, 1 on bad shape, 2 on allocation failure.
 */
int q8o_matmul(const float* x, int64_t m, int64_t k, const uint8_t* w, int64_t n, float* y,
               int threads) {
  if (m < 0 || n < 0 || k <= 0 || k % QK8_0) return 1;
  if (m == 0 || n == 0) return 0;
  const int64_t nb = k / QK8_0;
  int8_t* qx = (int8_t*)malloc((size_t)(m * k));
  uint16_t* dh = (uint16_t*)malloc((size_t)(m * nb) * sizeof(uint16_t));
  float* dx = (float*)malloc((size_t)(m * nb) * sizeof(float));
  if (!qx || !dh || !dx) {
    free(qx); free(dh); free(dx);
    return 2;
  }
  q8o_quantize_planes(x, m, k, qx, dh);
  for (int64_t i = 0; i < m * nb; ++i) dx[i] = q8o_f16_to_f32(dh[i]);
  if (threads < 1) threads = 1;
  if (threads > n) threads = (int)n;
  mm_job* jobs = (mm_job*)calloc((size_t)threads, sizeof(mm_job));
  pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  if (!jobs || !tids) {
    free(qx); free(dh); free(dx); free(jobs); free(tids);
    return 2;
  }
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (mm_job){w, qx, dx, y, m, n, k, n * t / threads, n * (t + 1) / threads};
  }
  for (int t = 1; t < threads; ++t) pthread_create(&tids[t], NULL, mm_worker, &jobs[t]);
  mm_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tids[t], NULL);
  free(qx); free(dh); free(dx); free(jobs); free(tids);
  return 0;
}

/*
 * SwiGLU of the VoxCPM MLP (crates/voxcpm/src/transformer.rs:147-150:
 * `l.down.forward(&(l.gate.forward(&h)?.silu()? * l.up.forward(&h)?)?)`).
 * candle-core's f32 silu unary op is v / (1 + exp(-v)), each operation rounded to f32
 * (exp from the platform libm, as Rust's f32::exp), then the product with up.
 * gu[m][2*inter]: gate columns [0, inter), up columns [inter, 2*inter).
 */
int q8o_swiglu(const float* gu, int64_t m, int64_t inter, float* h) {
  if (m < 0 || inter <= 0) return 1;
  for (int64_t r = 0; r < m; ++r) {
    const float* g = gu + r * 2 * inter;
    const float* u = g + inter;
    for (int64_t i = 0; i < inter; ++i) {
      const float e = expf(-g[i]);
      const float s = g[i] / (1.0f + e);
      h[r * inter + i] = s * u[i];
    }
  }
  return 0;
}
