/*
 * q8lin.h -- C ABI of the B200 (sm_100a) Q8_0 quantized linear.
 *
 * Drop-in for the Q8_0 projection path of talechime's VoxCPM BaseLM:
 *   Weights::linear keeps a Q8_0 GGUF tensor as QMatMul::QTensor(Arc<QTensor>)
 *     (crates/voxcpm/src/weights.rs:98-117, Q8_0 test at :103-104)
 *   Linear::forward flattens x to [rows, in] and calls QMatMul::forward
 *     (crates/voxcpm/src/weights.rs:213-229; the call itself at :221)
 *   callers: Transformer::forward q/k/v/o/gate/up/down
 *     (crates/voxcpm/src/transformer.rs:119-121,146,148-150).
 * The arithmetic it replaces is candle-core 0.11.0's QMatMul over GgmlDType::Q8_0
 * (third-party; Cargo.toml:20,94-98).
 *
 * Conventions
 *   - Every function returns an int status (Q8LIN_OK == 0) and never aborts;
 *     q8lin_last_error() returns the calling thread's message for the last failure.
 *   - Streams are cudaStream_t passed as void* (NULL = legacy default stream).
 *   - x / y / workspace are device pointers on the weight's device, 16-byte aligned.
 *   - q8lin_forward* never synchronize the host and never allocate: the paths that
 *     need scratch (M > 4 outside the small-batch kernel's range) read it from the
 *     workspace bound to the weight (q8lin_workspace_create at load time, then
 *     q8lin_weight_bind_workspace) or from the caller (q8lin_forward_ws), so every
 *     forward entry point may be captured in a CUDA graph.
 *   - Kernel spin waits are bounded in time (q8lin_set_wait_limit_ns); a wait that runs
 *     out sets a bit of the device fault word (q8lin_fault_status).
 */
#ifndef Q8LIN_H
#define Q8LIN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q8LIN_VERSION 3
#define Q8LIN_QK 32          /* values per Q8_0 block */
#define Q8LIN_BLOCK_BYTES 34 /* GGUF block: f16 d + int8 qs[32] */

typedef struct q8lin_weight q8lin_weight; /* one Q8_0 projection resident on one GPU */
typedef struct q8lin_workspace q8lin_workspace; /* device scratch of the batched paths */
typedef void* q8lin_stream_t;             /* cudaStream_t */

enum q8lin_status {
  Q8LIN_OK = 0,
  Q8LIN_ERR_INVALID_ARGUMENT = 1, /* null handle/pointer, negative size */
  Q8LIN_ERR_SHAPE = 2,            /* K % 32 != 0, K mismatch, size beyond limits */
  Q8LIN_ERR_ALIGNMENT = 3,        /* device pointer not 16-byte aligned */
  Q8LIN_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed */
  Q8LIN_ERR_NCCL = 5,             /* a collective failed (tensor-parallel entry points) */
  Q8LIN_ERR_OUT_OF_MEMORY = 6,
  Q8LIN_ERR_DEVICE = 7,           /* not a compute-capability 10.0 GPU, or wrong device */
  Q8LIN_ERR_WORKSPACE = 8,        /* caller workspace smaller than q8lin_workspace_size */
  Q8LIN_ERR_FORMAT = 9,           /* malformed GGUF file, or a value/tensor of the wrong type */
  Q8LIN_ERR_IO = 10,              /* a file could not be opened or mapped */
  Q8LIN_ERR_NOT_FOUND = 11        /* GGUF metadata key or tensor name not present */
};

/* Library version (Q8LIN_VERSION). */
int q8lin_version(void);
/* Message of the calling thread's last failing call ("" if none). */
const char* q8lin_last_error(void);
/* Static name of a status code. */
const char* q8lin_status_string(int status);

/*
 * Upload and repack one Q8_0 GGUF tensor.
 * Replaces: Content::tensor(file, name, device) -> QTensor and the
 *   QMatMul::QTensor(Arc::new(q)) construction (crates/voxcpm/src/weights.rs:100-104).
 * gguf_blocks: N rows x K/32 blocks of 34 bytes, the tensor's bytes as stored in the
 *   GGUF file (ggml ne = [K, N]); host or device memory (detected).
 * Repacks on `device` into per-row [int8 qs[K] | f16 d[K/32] | pad to 16 B] rows.
 * Synchronizes `stream` before returning (load time, not the hot path).
 */
int q8lin_weight_create(const void* gguf_blocks, int64_t n, int64_t k, int device,
                        q8lin_stream_t stream, q8lin_weight** out);
/* Free a weight (NULL is a no-op). */
int q8lin_weight_destroy(q8lin_weight* w);
/* Logical shape: n = out features, k = in features (candle shape (n, k)). */
int q8lin_weight_shape(const q8lin_weight* w, int64_t* n, int64_t* k, int* device);
/* Bytes the repacked weight holds in HBM. */
int q8lin_weight_device_bytes(const q8lin_weight* w, size_t* bytes);
/*
 * Dequantize to f32 [N][K] (device memory).
 * Replaces: QTensor::dequantize (crates/voxcpm/src/weights.rs:79-80,106).
 */
int q8lin_weight_dequantize(const q8lin_weight* w, float* out, q8lin_stream_t stream);
/* Write the weight back in GGUF block layout (device memory, N*K/32*34 bytes). */
int q8lin_weight_export_gguf(const q8lin_weight* w, void* out_blocks, q8lin_stream_t stream);

/* Workspace bytes q8lin_forward_ws needs for M rows: 0 where a GEMV kernel serves M
 * (M <= 4, and the dp4a small-batch kernel's range, see q8lin_dispatch_path); on the
 * mma.sync small-batch path (12 <= M <= 16 where it applies) the int8 activations
 * [M][K] and transposed f32 scales; on the int8 tensor-core path (M <= 32) the same plus
 * the split-K partial sums; for larger M the activations as f16 integers [M][K],
 * transposed f32 scales and one wave of split-K partial tiles.  Regions are 256-byte
 * aligned. */
size_t q8lin_workspace_size(const q8lin_weight* w, int64_t m);

/*
 * The kernel q8lin_forward runs for M rows of an N x K Q8_0 weight (host only, no GPU
 * needed; -1 for invalid sizes).  The choice follows crossovers measured on B200 in
 * CUDA graphs.  No counterpart in the reference (candle picks its own CUDA kernels by
 * M); it makes the dispatch inspectable and testable.
 */
enum q8lin_path {
  Q8LIN_PATH_STREAM_GEMV = 0, /* M = 1: bulk-copy ring, one CTA per SM */
  Q8LIN_PATH_GEMV = 1,        /* M <= 4: register-streaming GEMV */
  Q8LIN_PATH_SMALL_BATCH = 2, /* 2 <= M <= 16 where it wins: dp4a against every row */
  Q8LIN_PATH_INT8_TC = 3,     /* M <= 32: int8 tensor cores, weights on the 128-row side */
  Q8LIN_PATH_F16_TC = 4,      /* M > 32: f16 tensor cores with per-block rescale */
  Q8LIN_PATH_SMALL_BATCH_TC = 5 /* 2 <= M <= 16: mma.sync int8, activations quantized once */
};
int q8lin_dispatch_path(int64_t m, int64_t k, int64_t n);

/*
 * Workspace of the batched paths, allocated once (load time) and bound to the weights
 * that use it, so that q8lin_forward itself allocates nothing -- the reference's capture
 * rule: only buffers allocated before capture survive a replay
 * (crates/voxcpm/src/cuda_graph/replay.rs:46-80).
 * q8lin_workspace_bytes(max_m, max_k): bytes covering every M <= max_m and K <= max_k
 *   (0 if no path needs scratch there).
 * q8lin_workspace_create allocates it on `device` (cudaMalloc: call it at load time).
 * q8lin_weight_bind_workspace(w, ws): q8lin_forward(w, ...) reads ws from then on (NULL
 *   unbinds).  One workspace may be bound to every weight of a model: calls issued on one
 *   stream are ordered, calls on different streams that share it race.  Weights do not
 *   own it: unbind or destroy the weights before destroying the workspace.
 */
size_t q8lin_workspace_bytes(int64_t max_m, int64_t max_k);
int q8lin_workspace_create(int device, int64_t max_m, int64_t max_k, q8lin_workspace** out);
int q8lin_workspace_destroy(q8lin_workspace* ws);
int q8lin_workspace_capacity(const q8lin_workspace* ws, size_t* bytes);
int q8lin_weight_bind_workspace(q8lin_weight* w, q8lin_workspace* ws);

/*
 * y[M][N] = x[M][K] . W^T with candle's CPU Q8_0 semantics: every x row is
 * quantized to Q8_0 blocks (d = amax/127, q = round-half-away(x * (1/d)), d kept
 * as f16), then y = sum over blocks of f32(isum) * f32(dw) * f32(dx) in f32.
 * Replaces: QMatMul::forward for QMatMul::QTensor/Q8_0, called at
 *   crates/voxcpm/src/weights.rs:221 (shape rules as candle's: 2-D [M, K], K == in).
 * x, y: f32 device memory, row-major, contiguous.  M == 0 is a no-op.
 * Where the path needs scratch (q8lin_workspace_size > 0) it uses the workspace bound to
 * the weight and returns Q8LIN_ERR_WORKSPACE when none is bound or it is too small.
 */
int q8lin_forward(const q8lin_weight* w, const float* x, float* y, int64_t m,
                  q8lin_stream_t stream);
/* As q8lin_forward with a caller-provided workspace (256-byte aligned). */
int q8lin_forward_ws(const q8lin_weight* w, const float* x, float* y, int64_t m,
                     void* workspace, size_t workspace_bytes, q8lin_stream_t stream);

/*
 * No counterpart in the reference.  The same y = x . W^T for callers that must not
 * allocate device memory during a call -- a real-time audio producer cannot stall
 * on cudaMalloc's device synchronisation, and an embedder whose allocator owns all
 * device memory may not be allowed to allocate around it.  The activation scratch
 * is a fixed device array inside the library (9 MiB per GPU that loads it, held
 * until exit), so this call allocates nothing.  Limit: M*K <= Q8LIN_NOALLOC_MAX_VALUES;
 * larger inputs return Q8LIN_ERR_SHAPE.  The first call on a device looks up the
 * array's device address, so make it before any stream capture.  All calls on a
 * device share the array: calls that overlap on the GPU race (calls issued on one
 * stream are ordered).
 */
#define Q8LIN_NOALLOC_MAX_VALUES 8388608
int q8lin_forward_noalloc(const q8lin_weight* w, const float* x, float* y, int64_t m,
                          q8lin_stream_t stream);

/*
 * Time limit of every spin wait inside the kernels, in nanoseconds (default 1 s); it
 * applies to launches issued -- or captured into a CUDA graph -- after the call.  A wait
 * that runs out sets its bit of the fault word, and the kernel stops, writes NaN where it
 * could not compute and returns.  Waits for a kernel's own bulk copies before it exits
 * keep a fixed 2 s bound.  No counterpart in the reference (candle's kernels do not
 * spin); the library's failure-detection hook together with q8lin_fault_status.
 */
int q8lin_set_wait_limit_ns(uint64_t ns);
uint64_t q8lin_wait_limit_ns(void);

/*
 * Device-side fault word of `device` (bit 0: a tensor-core kernel's bounded wait ran
 * out, bit 1: a streaming GEMV's (M = 1, or the small-batch dp4a kernel), bit 2: the
 * small-batch int8 tensor-core kernel's, bit 3: the fused attention's, bit 4: the
 * persistent decode step's; the kernel returned early and its output is invalid).
 * Reads it with a device synchronisation; `clear` resets it.  No counterpart in the reference (candle's
 * kernels have no bounded waits); this is the library's failure-detection hook.
 */
int q8lin_fault_status(int device, uint32_t* flags, int clear);

/*
 * Quantize f32 activations x[M][K] to Q8_0 planes on the device: qs int8 [M][K]
 * and d as f16 bits [M][K/32].  The quantizer every forward path uses (candle's
 * BlockQ8_0::from_float applied to the lhs rows of its CPU matmul).
 */
int q8lin_quantize_rows(const float* x, int64_t m, int64_t k, int8_t* qs, uint16_t* d_f16,
                        q8lin_stream_t stream);

/*
 * SwiGLU between the gate/up and down projections of the MLP: gu is the f32 output
 * [M][2*inter] of one fused gate+up linear (gate columns first, then up), h[M][inter] =
 * silu(gate) * up with candle's f32 silu v / (1 + exp(-v)).  Replaces the
 * `l.gate.forward(&h)?.silu()? * l.up.forward(&h)?` step of
 * crates/voxcpm/src/transformer.rs:147-150 (two linears, silu, mul) when the gate and
 * up weights are stored as one fused weight, as the tensor-parallel shards are.
 * gu and h are device pointers (4-byte aligned; 16-byte aligned rows take the
 * vectorized kernel).  Capture-safe.
 */
int q8lin_swiglu(const float* gu, int64_t m, int64_t inter, float* h, q8lin_stream_t stream);

/*
 * Decode-step building blocks around the linears (batch 1, f32, device pointers).  The
 * position `pos` and tokens are device int32 values, so a captured CUDA graph of one
 * step replays for every token: q8lin_argmax writes the next token and advances pos.
 * Replace the per-layer tensor ops of crates/voxcpm/src/transformer.rs:107-155 and
 * attention.rs:28-98 (rms_norm, rotate, KV-cache cat, grouped attention, residual add)
 * and the greedy pick of the decode loop.
 */
/* The decode-step fusions around one projection (M = 1, K <= 8192), in one kernel:
 *   prologue 0: y = W . x;  1: y = W . rms_norm(x, norm_weight, eps)  (x[K]);
 *   2: y = W . (silu(x[0..K)) * x[K..2K))  (gate|up of the fused MLP projection);
 *   then, if residual != NULL, y = residual + y (residual may alias y).
 * Replaces norm -> linear and linear -> residual add pairs of
 * crates/voxcpm/src/transformer.rs:117-118,146-150 with one launch each. */
int q8lin_forward_fused(const q8lin_weight* w, const float* x, float* y, int64_t m, int32_t prologue,
                        const float* norm_weight, float eps, const float* residual, q8lin_stream_t stream);
/* Dequantized rows tokens[0..n) of a Q8_0 embedding weight [vocab][hidden] -> out[n][hidden]. */
int q8lin_embed_rows(const q8lin_weight* w, const int32_t* tokens, int64_t n, float* out, q8lin_stream_t stream);
/* y[m][n] = x / sqrt(sum(x^2)/n + eps) * weight (candle_nn::ops::rms_norm). */
int q8lin_rmsnorm(const float* x, const float* weight, int64_t m, int64_t n, float eps, float* y,
                  q8lin_stream_t stream);
/* qkv[(hq + 2 hkv) * d] of the token at *pos: rotated q -> q_out[hq][d], rotated k and v
 * -> k_cache / v_cache [hkv][max_t][d] at row *pos.  cos_t / sin_t: [max_t][d/2]. */
int q8lin_rope_kv(const float* qkv, const int32_t* pos, const float* cos_t, const float* sin_t, float* k_cache,
                  float* v_cache, int32_t hq, int32_t hkv, int32_t d, int32_t max_t, float* q_out,
                  q8lin_stream_t stream);
size_t q8lin_attention_workspace_size(int32_t hq, int32_t max_t);
/* out[hq][d] = softmax(q k^T / sqrt(d)) v over cache rows [0, *pos], kv head = q head /
 * (hq / hkv); d = 128.  The workspace must be zero-filled once before first use. */
int q8lin_attention_decode(const float* q, const float* k_cache, const float* v_cache, const int32_t* pos,
                           int32_t hq, int32_t hkv, int32_t d, int32_t max_t, void* workspace, size_t workspace_bytes,
                           float* out, q8lin_stream_t stream);
/* RoPE + KV append + attention in one launch: rotates q and the current k of qkv at *pos,
 * appends k and v to the caches at row *pos and writes out[hq][d] = softmax(q K^T /
 * sqrt(d)) V over rows [0, *pos]; d = 128.  One cluster of 8 CTAs per q head; no
 * workspace. */
int q8lin_rope_attention_decode(const float* qkv, const int32_t* pos, const float* cos_t, const float* sin_t,
                                float* k_cache, float* v_cache, int32_t hq, int32_t hkv, int32_t d, int32_t max_t,
                                float* out, q8lin_stream_t stream);
/* Q8LIN_ATTN_POS_READY: *pos and the cache rows below it were written before the launch
 * preceding this one on the stream began (true inside a decode step that starts with an
 * embedding launch after the previous step's argmax); the kernel then reads them and
 * starts copying K/V before its dependency wait. */
#define Q8LIN_ATTN_POS_READY 1u
int q8lin_rope_attention_decode_ex(const float* qkv, const int32_t* pos, const float* cos_t, const float* sin_t,
                                   float* k_cache, float* v_cache, int32_t hq, int32_t hkv, int32_t d, int32_t max_t,
                                   float* out, uint32_t flags, q8lin_stream_t stream);
/* x[0..n) += y[0..n). */
int q8lin_add(float* x, const float* y, int64_t n, q8lin_stream_t stream);
/* x[m][n] += y[m][n], then h[m][n] = x / sqrt(sum(x^2)/n + eps) * weight: the residual add
 * and the rms_norm after it (crates/voxcpm/src/transformer.rs:146-147, and :116-117 of
 * the next layer) in one pass over the rows; x and h must not overlap. */
int q8lin_add_rmsnorm(float* x, const float* y, const float* weight, int64_t m, int64_t n, float eps, float* h,
                      q8lin_stream_t stream);

/*
 * Prefill building blocks: `batch` sequences, each with t new rows at positions
 * pos0 .. pos0 + t - 1 (pos0 a host value), run as one batched forward -- the prompt
 * pass `self.base.forward(&input, ...)` with M = context of crates/voxcpm/src/
 * model.rs:492-495 through transformer.rs:107-155 (offset = pos0).  The linears,
 * norms, SwiGLU and residual adds of that pass are q8lin_forward / q8lin_rmsnorm /
 * q8lin_swiglu / q8lin_add at M = batch * t.  Row r = s * t + i of sequence s, new row i.
 * Both return Q8LIN_ERR_SHAPE when pos0 < 0 or pos0 + t > max_t (the reference's
 * "Transformer context limit exceeded", transformer.rs:110-113).
 *
 * qkv[batch * t][(hq + 2 hkv) * d]: rotated q -> q_out[batch * t][hq][d]; rotated k and
 * v -> k_cache / v_cache [batch][hkv][max_t][d] at rows pos0 + i (rotate(),
 * transformer.rs:159-170; the cat-growth of :131-139 preallocated).
 */
int q8lin_rope_kv_rows(const float* qkv, int32_t batch, int64_t t, int32_t pos0, const float* cos_t,
                       const float* sin_t, float* k_cache, float* v_cache, int32_t hq, int32_t hkv, int32_t d,
                       int32_t max_t, float* q_out, q8lin_stream_t stream);
/* Causal grouped attention of the new rows: out[batch * t][hq][d] = softmax(q K^T /
 * sqrt(d)) V over cache rows [0, pos0 + i] of the row's sequence (attention.rs:28-98,
 * causal mask :84-95), kv head = q head / (hq / hkv); d = 128.  The cache rows
 * [0, pos0 + t) must be written (q8lin_rope_kv_rows for the new ones).  q, the caches
 * and out 16-byte aligned.  No workspace. */
int q8lin_attention_prefill(const float* q, const float* k_cache, const float* v_cache, int32_t batch, int64_t t,
                            int32_t pos0, int32_t hq, int32_t hkv, int32_t d, int32_t max_t, float* out,
                            q8lin_stream_t stream);
size_t q8lin_argmax_workspace_size(void);
/* *token = argmax(logits[0..n)) (lowest index on ties); if pos != NULL, *pos += 1.  The
 * workspace must be zero-filled once before first use. */
int q8lin_argmax(const float* logits, int64_t n, void* workspace, size_t workspace_bytes, int32_t* token, int32_t* pos,
                 q8lin_stream_t stream);

/*
 * Tensor-parallel down projection with the cross-GPU sum fused into the GEMV (M = 1,
 * K <= 8192): y = [residual +] sum over the `world` ranks of W_rank . x_rank, each rank's
 * rows pushed into every rank's staging buffer over NVLink (peer stores) and added in rank
 * order (deterministic; bit-identical to a two-rank NCCL sum).  Replaces the partial
 * down projection + all-reduce of the tensor-parallel MLP (crates/voxcpm/src/transformer.rs
 * :147-150 split over GPUs).  Buffers: one staging buffer of
 * q8lin_allreduce_stage_bytes(N, world) per rank, allocated with q8lin_peer_alloc (zeroed;
 * its IPC handle, Q8LIN_IPC_HANDLE_BYTES bytes, is exchanged out of band and opened on the
 * other ranks with q8lin_peer_open).  Every staged value travels with the call's epoch in
 * one 64-bit word, so a rank knows a peer's row has arrived when it reads that epoch: no
 * fence and no flag.  stage_n: the N the staging buffers were sized for (a weight with
 * more rows is rejected).  stage_ptrs: DEVICE array of `world` pointers, entry r = rank
 * r's buffer as mapped on this GPU.  flag_ptrs: not read since version 3 (may be NULL;
 * q8lin_allreduce_flag_bytes is kept for callers of version 2).  epoch: the call count,
 * 1, 2, ... (every rank passes the same value; all ranks must make every call).  A rank
 * that never arrives makes the others time out (fault word bit 1, NaN rows) instead of
 * hanging.
 */
#define Q8LIN_IPC_HANDLE_BYTES 64
int q8lin_peer_alloc(int device, size_t bytes, void** ptr, void* ipc_handle);
int q8lin_peer_open(int device, const void* ipc_handle, void** ptr);
int q8lin_peer_close(int device, void* ptr);
int q8lin_peer_free(int device, void* ptr);
size_t q8lin_allreduce_stage_bytes(int64_t n, int32_t world);
size_t q8lin_allreduce_flag_bytes(int32_t world);
int q8lin_forward_allreduce(const q8lin_weight* w, const float* x, float* y, int64_t m, void* const* stage_ptrs,
                            void* const* flag_ptrs, int64_t stage_n, int32_t rank, int32_t world, uint32_t epoch,
                            const float* residual, q8lin_stream_t stream);

/*
 * Tensor-parallel Q8_0 SwiGLU MLP over `world` GPUs of one node: the VoxCPM MLP
 * down(silu(gate(h)) * up(h)) (crates/voxcpm/src/transformer.rs:147-150, three
 * Linear::forward calls, weights.rs:213-229) split with one exchange step -- gate and up
 * by output rows (rank r keeps rows [I*r/P, I*(r+1)/P) of each, fused as one [gate; up]
 * weight), SwiGLU local, down by Q8_0 block columns (I/P a multiple of 32), the partial
 * outputs summed with ncclAllReduce on the caller's communicator.
 * q8lin_mlp_tp_create: gate, up are the FULL [inter][hidden] Q8_0 GGUF tensors and down
 *   the full [hidden][inter] one (host or device memory); the rank keeps its shards.
 *   nccl_comm: an ncclComm_t of `world` ranks in which this process is `rank` (checked with
 *   ncclCommCount / ncclCommUserRank; may be NULL when world == 1); NCCL is the
 *   libnccl.so.2 the process has loaded (the one that made the communicator).  All scratch
 *   for up to max_m activation rows is allocated here.
 *   Q8LIN_TP_FUSED_DECODE (world > 1, hidden and inter/world <= 8192): create also
 *   allocates staging and flag buffers; the caller gathers every rank's
 *   q8lin_mlp_tp_peer_handle (Q8LIN_TP_HANDLE_BYTES each, in rank order) over its own
 *   transport and passes them to q8lin_mlp_tp_connect_peers on every rank (IPC mappings:
 *   the ranks share one node).  From then on one activation row runs the down projection
 *   and the cross-GPU sum as one kernel per rank over NVLink peer memory (see
 *   q8lin_forward_allreduce); before, M = 1 takes the NCCL path.
 * q8lin_mlp_tp_forward: y[M][hidden] = the whole MLP of x[M][hidden] (x replicated on
 *   every rank, y too).  Every rank calls it with the same M in the same order.  Allocates
 *   nothing.  Q8LIN_ERR_NCCL when the all-reduce fails; on the fused path a rank that never
 *   arrives makes the others time out (fault word bit 1, their output rows NaN).
 * Teardown with the fused path: every rank calls q8lin_mlp_tp_close_peers (it waits for
 *   its own work and unmaps the peers' buffers), the ranks meet at a host barrier, then
 *   each calls q8lin_mlp_tp_destroy -- so no rank frees a buffer a peer still maps.  No
 *   entry point here runs a collective except forward's all-reduce, so a rank that never
 *   arrives cannot hang the others in create or teardown.
 * q8lin_mlp_tp_shard: the shard plan alone (host only, no GPU): rows [row0, row0 + rows)
 *   of gate and up, block columns [blk0, blk0 + blks) of down.
 */
typedef struct q8lin_mlp_tp q8lin_mlp_tp;
#define Q8LIN_TP_FUSED_DECODE 1u
#define Q8LIN_TP_HANDLE_BYTES (2 * Q8LIN_IPC_HANDLE_BYTES)
int q8lin_mlp_tp_create(const void* gate_blocks, const void* up_blocks, const void* down_blocks, int64_t hidden,
                        int64_t inter, int32_t rank, int32_t world, void* nccl_comm, int device, int64_t max_m,
                        uint32_t flags, q8lin_stream_t stream, q8lin_mlp_tp** out);
int q8lin_mlp_tp_peer_handle(const q8lin_mlp_tp* mlp, void* out);
int q8lin_mlp_tp_connect_peers(q8lin_mlp_tp* mlp, const void* all_handles);
int q8lin_mlp_tp_forward(q8lin_mlp_tp* mlp, const float* x, float* y, int64_t m, q8lin_stream_t stream);
int q8lin_mlp_tp_close_peers(q8lin_mlp_tp* mlp);
int q8lin_mlp_tp_destroy(q8lin_mlp_tp* mlp);
int q8lin_mlp_tp_info(const q8lin_mlp_tp* mlp, int64_t* inter_local, int32_t* fused);
int q8lin_mlp_tp_shard(int64_t hidden, int64_t inter, int32_t rank, int32_t world, int64_t* row0, int64_t* rows,
                       int64_t* blk0, int64_t* blks);
/* 1 if libnccl.so.2 could be resolved (already loaded, or loadable), else 0. */
int q8lin_nccl_available(void);

/*
 * Persistent decode step: a program of operations run by ONE cooperative launch (one
 * CTA per SM).  The weights of every GEMV stream through each SM's shared-memory ring
 * ahead of the data; operation i starts when every CTA has finished operation i - 1.
 * Semantics per operation equal the multi-launch entry points:
 *   GEMV       y = [residual +] W . prologue(x), M = 1 (q8lin_forward_fused), K <= 8192;
 *              epilogue Q8LIN_EPILOGUE_SWIGLU: W holds [gate | up] rows (N = 2I) and
 *              y[i] = silu(gate_i) * up_i for i < I (K <= 2048, no residual);
 *              argmax != 0 records row maxima for a following ARGMAX op;
 *   ATTENTION  q8lin_rope_attention_decode on x = qkv at *pos into y [hq * head_dim];
 *   EMBED      y[0..K) = dequantized row *token of the weight (q8lin_embed_rows);
 *   ARGMAX     *token = argmax of the preceding GEMV's output, *pos += 1 (q8lin_argmax).
 * Pointers stay owned by the caller and must outlive the step.  q8lin_step_run is
 * stream-ordered, allocates nothing and may be captured in a CUDA graph; a step object
 * serves one stream at a time.  Fault word bit 4: a bounded wait of the step timed out.
 */
typedef struct q8lin_step q8lin_step;

enum q8lin_op_kind { Q8LIN_OP_GEMV = 0, Q8LIN_OP_ATTENTION = 1, Q8LIN_OP_EMBED = 2, Q8LIN_OP_ARGMAX = 3 };
#define Q8LIN_PROLOGUE_NONE 0
#define Q8LIN_PROLOGUE_RMSNORM 1
#define Q8LIN_PROLOGUE_SWIGLU 2
#define Q8LIN_EPILOGUE_NONE 0
#define Q8LIN_EPILOGUE_SWIGLU 1

typedef struct q8lin_op {
  int32_t kind;                /* q8lin_op_kind */
  int32_t prologue;            /* GEMV: Q8LIN_PROLOGUE_* */
  int32_t epilogue;            /* GEMV: Q8LIN_EPILOGUE_* */
  int32_t argmax;              /* GEMV: feed the following ARGMAX op */
  const q8lin_weight* weight;  /* GEMV, EMBED */
  const float* x;              /* GEMV input (2K values for the SwiGLU prologue); ATTENTION: qkv */
  float* y;                    /* GEMV output; EMBED output [K]; ATTENTION output */
  const float* residual;       /* GEMV: added to y (may alias y) */
  const float* norm_weight;    /* GEMV RMSNORM: [K] */
  float* k_cache;              /* ATTENTION: [hkv][max_t][head_dim] */
  float* v_cache;
  const float* cos_t;          /* ATTENTION: [max_t][head_dim / 2] */
  const float* sin_t;
  float eps;                   /* GEMV RMSNORM */
  int32_t hq, hkv, head_dim, max_t;
} q8lin_op;

int q8lin_step_create(const q8lin_op* ops, int32_t nops, int32_t* pos, int32_t* token, int device, q8lin_step** out);
int q8lin_step_run(q8lin_step* step, q8lin_stream_t stream);
int q8lin_step_destroy(q8lin_step* step);

/*
 * GGUF reader (versions 2 and 3): replaces candle's gguf_file::Content as used by
 * Weights::open / ::linear / ::value (crates/voxcpm/src/weights.rs:31-41, :96-115,
 * :117-137).  The file is mapped read-only; names and string values returned point into
 * the handle and stay valid until q8lin_gguf_close.  Tensor dims are GGUF `ne` order
 * (ne[0] contiguous; a [N out, K in] linear has ne = {K, N}); unused dims are 1.
 */
typedef struct q8lin_gguf q8lin_gguf;

enum q8lin_ggml_type {
  Q8LIN_GGML_F32 = 0,
  Q8LIN_GGML_F16 = 1,
  Q8LIN_GGML_Q8_0 = 8,
  Q8LIN_GGML_BF16 = 30
};

/* GGUF metadata value types (published numbering). */
enum q8lin_gguf_value_type {
  Q8LIN_GGUF_U8 = 0, Q8LIN_GGUF_I8 = 1, Q8LIN_GGUF_U16 = 2, Q8LIN_GGUF_I16 = 3,
  Q8LIN_GGUF_U32 = 4, Q8LIN_GGUF_I32 = 5, Q8LIN_GGUF_F32 = 6, Q8LIN_GGUF_BOOL = 7,
  Q8LIN_GGUF_STRING = 8, Q8LIN_GGUF_ARRAY = 9, Q8LIN_GGUF_U64 = 10, Q8LIN_GGUF_I64 = 11,
  Q8LIN_GGUF_F64 = 12
};

int q8lin_gguf_open(const char* path, q8lin_gguf** out);
int q8lin_gguf_close(q8lin_gguf* g);
int q8lin_gguf_version(const q8lin_gguf* g, uint32_t* version);
int64_t q8lin_gguf_tensor_count(const q8lin_gguf* g);   /* -1 for a null handle */
int64_t q8lin_gguf_metadata_count(const q8lin_gguf* g); /* -1 for a null handle */
/* Index of a tensor by name; Q8LIN_ERR_NOT_FOUND if absent. */
int q8lin_gguf_find_tensor(const q8lin_gguf* g, const char* name, int64_t* index);
/* Any output pointer may be NULL.  dims receives 4 values.  nbytes is 0 for a ggml type
 * the reader cannot size (its bytes cannot be read). */
int q8lin_gguf_tensor_info(const q8lin_gguf* g, int64_t index, const char** name, uint32_t* ggml_type,
                           uint32_t* n_dims, int64_t* dims, uint64_t* nbytes);
/* Host pointer to a tensor's bytes inside the mapping. */
int q8lin_gguf_tensor_data(const q8lin_gguf* g, int64_t index, const void** data, uint64_t* nbytes);
int q8lin_gguf_metadata_type(const q8lin_gguf* g, const char* key, uint32_t* value_type);
/* Typed getters: _u32 accepts a U32 value only (like Value::to_u32); _i64 any integer or
 * bool; _f64 any number; Q8LIN_ERR_NOT_FOUND if the key is absent, Q8LIN_ERR_FORMAT if
 * the type does not match. */
int q8lin_gguf_metadata_u32(const q8lin_gguf* g, const char* key, uint32_t* value);
int q8lin_gguf_metadata_i64(const q8lin_gguf* g, const char* key, int64_t* value);
int q8lin_gguf_metadata_f64(const q8lin_gguf* g, const char* key, double* value);
/* String bytes (not NUL-terminated) and their length. */
int q8lin_gguf_metadata_string(const q8lin_gguf* g, const char* key, const char** data, uint64_t* len);
/* Array element type and count; data / nbytes (may be NULL) give the raw element bytes
 * (for string or nested arrays, their serialized form). */
int q8lin_gguf_metadata_array(const q8lin_gguf* g, const char* key, uint32_t* elem_type, uint64_t* count,
                              const void** data, uint64_t* nbytes);
/* q8lin_weight_create from a Q8_0 matrix tensor of the file (Weights::linear's
 * QMatMul::QTensor branch, weights.rs:100-104); Q8LIN_ERR_FORMAT for other types. */
int q8lin_gguf_weight_create(const q8lin_gguf* g, const char* tensor_name, int device, q8lin_stream_t stream,
                             q8lin_weight** out);

#ifdef __cplusplus
}
#endif

#endif /* Q8LIN_H */
