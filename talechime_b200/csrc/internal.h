// Host-side declarations shared by the translation units of libq8lin.so.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <string>

struct q8lin_workspace {
  int device = -1;
  void* ptr = nullptr;
  size_t bytes = 0;
};

struct q8lin_weight {
  int device = -1;
  int64_t n = 0;           // out features (rows)
  int64_t k = 0;           // in features
  int64_t row_stride = 0;  // bytes per repacked row
  uint8_t* packed = nullptr;
  size_t bytes = 0;
  const q8lin_workspace* ws = nullptr;  // bound by q8lin_weight_bind_workspace; not owned
};

namespace q8lin {

// Makes `device` current for the scope and restores the caller's device.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device);
  ~DeviceGuard();
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
  bool ok() const { return ok_; }

 private:
  int prev_ = 0;
  bool ok_ = false;
  bool switched_ = false;
};
// Q8LIN_OK if `device` exists and is a compute-capability 10.0 GPU.
int check_device(int device);
bool aligned16(const void* p);
// Opt-in of the dynamic shared memory of kernel `fn`, once per (device, size); `configured`
// is the caller's per-device record (128 entries).  With max_carveout the carveout is set
// to the maximum (two CTAs of the streaming GEMV share an SM).  Thread-safe.
cudaError_t ensure_smem(const void* fn, int* configured, int device, size_t smem, bool max_carveout);

// Error plumbing (thread-local message).
int fail(int status, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

// Kernel launchers (return cudaError_t of the launch).
cudaError_t launch_repack(const uint8_t* gguf, uint8_t* packed, int64_t n, int64_t k,
                          int64_t row_stride, cudaStream_t s);
cudaError_t launch_unpack(const uint8_t* packed, uint8_t* gguf, int64_t n, int64_t k,
                          int64_t row_stride, cudaStream_t s);
cudaError_t launch_dequantize(const uint8_t* packed, float* out, int64_t n, int64_t k,
                              int64_t row_stride, cudaStream_t s);
cudaError_t launch_quantize_rows(const float* x, int64_t m, int64_t k, int8_t* qs,
                                 uint16_t* d_f16, float* d_f32, cudaStream_t s);

// Optional prologue / epilogue of the M = 1 streaming GEMV (decode step fusions):
// prologue kRmsNorm: x -> x / sqrt(sum(x^2)/K + eps) * norm_w before quantization;
// prologue kSwiGLU: x holds gate|up [2K] -> silu(gate) * up; epilogue: y = residual + W.x
// (residual may alias y).
enum GemvPrologue : int { kPrologueNone = 0, kPrologueRmsNorm = 1, kPrologueSwiGLU = 2 };
struct GemvFusion {
  int prologue = kPrologueNone;
  const float* norm_w = nullptr;
  float eps = 0.0f;
  const float* residual = nullptr;
  // Sum of the output over `ar_world` GPUs (tensor-parallel down projection), fused into
  // the GEMV: every CTA stores each of its rows into every rank's staging buffer as one
  // 64-bit word (epoch << 32 | f32 bits, peer stores over NVLink), then each thread waits
  // for its rows' words of every rank to carry this call's epoch and adds them in rank
  // order.  ar_stage: device array of `ar_world` pointers (this rank's own buffer at index
  // ar_rank); stage[r] holds [2][ar_world][N] u64 (calls alternate halves by epoch
  // parity).  ar_epoch is a per-call counter starting at 1, so the buffers never need
  // resetting; a rank can be at most one call ahead of a peer's reads (its next sum waits
  // for that peer's next words), which the two halves cover.  ar_flags: not read (kept
  // for the C ABI).
  unsigned long long* const* ar_stage = nullptr;
  unsigned* const* ar_flags = nullptr;
  int ar_rank = 0;
  int ar_world = 1;
  unsigned ar_epoch = 0;
};
// The fused forms need the streaming kernel: M = 1 and K <= this bound.
constexpr int kFusedMaxK = 8192;
// CTAs covered by the cross-GPU flag arrays (the streaming kernel runs one per SM).
constexpr int kAllreduceMaxCtas = 1024;
cudaError_t launch_gemv_fused(const q8lin_weight& w, const float* x, float* y, const GemvFusion& f, cudaStream_t s);

// Decode GEMV for 1 <= m <= kGemvMaxM.
constexpr int kGemvMaxM = 16;
size_t gemv_smem_bytes(int m, int64_t k);
// 2 <= M <= kMrowMaxM streaming GEMV on dp4a (gemv_mrow.cu).
constexpr int kMrowMaxM = 16;
bool mrow_applies(int64_t m, int64_t k);
cudaError_t launch_gemv_mrow(const q8lin_weight& w, const float* x, float* y, int m, cudaStream_t s);
cudaError_t read_mrow_fault(unsigned int* flags, bool clear);  // bit 1
bool stream_applies(int64_t k);  // M = 1 streaming kernel (gemv.cu) serves this K
cudaError_t launch_gemv(const q8lin_weight& w, const float* x, float* y, int m,
                        cudaStream_t s);

// Batched path for m > kGemvMaxM over pre-quantized activations.
cudaError_t launch_gemm(const q8lin_weight& w, const int8_t* qx, const float* dx, float* y,
                        int64_t m, cudaStream_t s);

// Tensor-core batched path (gemm_tc.cu): quantize x to f16 integers + transposed
// scales in `workspace`, then the tcgen05 matmul.
size_t gemm_tc_workspace_bytes(int64_t m, int64_t k);
cudaError_t launch_gemm_tc(const q8lin_weight& w, const float* x, void* workspace, float* y, int64_t m,
                           cudaStream_t s);
cudaError_t read_tc_fault(unsigned int* flags, bool clear);

// Small-batch int8 tensor-core path (gemm_skinny.cu), for m up to kSkinnyMaxM: quantize
// x to int8 + transposed scales in `workspace`, then the kind::i8 matmul (split-K with
// partial sums in the workspace).  Fault word bit 2.
constexpr int kSkinnyMaxM = 32;
// x [M][K] f32 -> int8 [M][K] and scales dxT[K/32][Mp] (rows M .. Mp - 1 of dxT zero)
cudaError_t launch_quantize_rows_i8t(const float* x, int M, int Mp, int K, int8_t* qx, float* dxT, cudaStream_t s);
// small batches on mma.sync int8 tensor cores (gemm_mma.cu): activations quantized once
// into the workspace, then the weights streamed in 16-row x 256-value units
constexpr int kMmaMaxM = 16;
constexpr size_t kMmaMaxSmem = 220 * 1024;  // rings + staged activations of one CTA
constexpr int64_t kMmaInKernelMaxValues = 32768;  // M*K the kernel quantizes itself ...
constexpr int64_t kMmaInKernelMinN = 8192;        // ... for weights of at least this many rows
bool mma_applies(int64_t m, int64_t k);
size_t gemm_mma_workspace_bytes(int64_t m, int64_t k);
cudaError_t launch_gemm_mma(const q8lin_weight& w, const float* x, void* workspace, float* y, int64_t m,
                            cudaStream_t s);
size_t gemm_skinny_workspace_bytes(int64_t m, int64_t k);
cudaError_t launch_gemm_skinny(const q8lin_weight& w, const float* x, void* workspace, float* y, int64_t m,
                               cudaStream_t s);
cudaError_t read_skinny_fault(unsigned int* flags, bool clear);
// M = 1 streaming GEMV (gemv.cu): bit 1 of the fault word.
cudaError_t read_gemv_fault(unsigned int* flags, bool clear);

// SwiGLU between the MLP projections (mlp.cu): h[m][i] = silu(gu[m][i]) * gu[m][inter + i].
cudaError_t launch_swiglu(const float* gu, int64_t m, int64_t inter, float* h, cudaStream_t s);

// Decode-step kernels (decoder.cu).  Batch 1; pos and tokens are device ints.
cudaError_t launch_embed_rows(const q8lin_weight& w, const int* tokens, int n, float* out, cudaStream_t s);
cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int64_t m, int64_t n, float* y,
                           cudaStream_t s);
cudaError_t launch_rope_kv(const float* qkv, const int* pos, const float* cos_t, const float* sin_t, float* kc,
                           float* vc, int hq, int hkv, int d, int max_t, float* q_out, cudaStream_t s);
size_t attention_workspace_bytes(int hq, int max_t);
cudaError_t launch_attention_decode(const float* q, const float* kc, const float* vc, const int* pos, int hq,
                                    int hkv, int max_t, void* ws, float* out, cudaStream_t s);
cudaError_t launch_rope_attention(const float* qkv, const int* pos, const float* cos_t, const float* sin_t, float* kc,
                                  float* vc, int hq, int hkv, int max_t, float* out, int device, cudaStream_t s,
                                  bool pos_ready);
cudaError_t read_attention_fault(unsigned int* flags, bool clear);  // bit 3
cudaError_t launch_add(float* x, const float* y, int64_t n, cudaStream_t s);

// Prefill kernels (prefill.cu): `batch` sequences of t rows at positions pos0 .. pos0+t-1
// (host values, checked by the caller: pos0 >= 0, pos0 + t <= max_t); caches
// [batch][hkv][max_t][d].
cudaError_t launch_rope_kv_rows(const float* qkv, int batch, int t, int pos0, const float* cos_t, const float* sin_t,
                                float* kc, float* vc, int hq, int hkv, int d, int max_t, float* q_out, cudaStream_t s);
// x[m][n] += y; h = rms_norm(x) * w (one kernel where n % 4 == 0, n <= 8192 and the rows
// are 16-byte aligned; else the add and rmsnorm kernels).
cudaError_t launch_add_rmsnorm(float* x, const float* y, const float* w, float eps, int64_t m, int64_t n, float* h,
                               cudaStream_t s);
cudaError_t launch_attention_prefill(const float* q, const float* kc, const float* vc, int batch, int t, int pos0,
                                     int hq, int hkv, int max_t, float* out, int device, cudaStream_t s);

// Persistent decode-step kernel (step.cu).
constexpr int kStepMaxK = 8192;
enum StepOpKind { kStepOpGemv = 0, kStepOpAttention = 1, kStepOpEmbed = 2, kStepOpArgmax = 3 };
enum StepPrologue { kStepPrologueNone = 0, kStepPrologueRmsNorm = 1, kStepPrologueSwiGLU = 2 };
enum StepEpilogue { kStepEpilogueNone = 0, kStepEpilogueSwiGLU = 1 };
struct StepOp {
  int kind, prologue, epilogue, n, k;  // GEMV / EMBED: weight rows n, columns k
  int64_t S;                           // packed row stride
  const uint8_t* W;
  const float* x;         // GEMV input; ATTENTION: the qkv projection
  float* y;               // GEMV / EMBED / ATTENTION output
  const float* residual;  // GEMV: y = residual + W x
  const float* norm_w;    // GEMV rms_norm prologue weight
  float eps;
  int argmax;             // GEMV: per-CTA row maxima for the ARGMAX operation
  int rpc;                // GEMV rows per ring chunk
  int hq, hkv, max_t;     // ATTENTION
  float scale;
  float* kc;
  float* vc;
  const float* cos_t;
  const float* sin_t;
  float* attn_part;       // ATTENTION: [hq][splits][132] partials (workspace)
  unsigned* head_cnt;     // ATTENTION: [hq] arrival counters (zero between launches)
};
size_t step_smem_bytes();
int step_rows_per_chunk(int64_t k);  // 0 if a row does not fit a ring slot
int step_splits();
cudaError_t step_max_grid(int device, int* grid);
cudaError_t launch_decode_step(const StepOp* ops, int nops, int* pos, int* token, unsigned* done, float* am_gv,
                               int* am_gi, int grid, int device, cudaStream_t s);
cudaError_t read_step_fault(unsigned int* flags, bool clear);  // bit 4
size_t argmax_workspace_bytes();
cudaError_t launch_argmax(const float* logits, int n, void* ws, int* token, int* pos, cudaStream_t s);

int sm_count(int device);

// Time limit of the kernels' spin waits in nanoseconds (q8lin_set_wait_limit_ns), read
// when a kernel is launched (or captured) and passed to it as an argument.
uint64_t wait_limit_ns();
extern std::atomic<uint64_t> g_wait_limit_ns;

// Programmatic dependent launch on/off (env Q8LIN_PDL=0 turns it off; read once).
bool pdl_enabled();

}  // namespace q8lin
