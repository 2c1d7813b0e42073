/*
 * g4q.h -- C ABI of libg4q, the B200 (sm_100a) implementation of Helios/gemma4d's
 * quantized-linear hot path: every mlx::core::quantized_matmul / mlx::core::dequantize
 * call that native/gemma4_mlx makes for the Gemma-style decoder, in MLX's affine format
 * (4-bit, group_size 64 along K, eight nibbles per uint32 little-endian, bf16 scale and
 * bias per group, w = scale * q + bias).
 *
 * Conventions (mirroring the reference's narrow C ABI, native/gemma4_mlx/include/gemma4_mlx.h):
 *   - Every call returns G4qStatus; the message of the last failure on the calling thread is
 *     kept in a thread-local buffer read with g4q_get_last_error (runtime.cc:46, 115-133,
 *     816-823). No C++ exception crosses this boundary.
 *   - Handles are opaque, allocated by the library, tagged with a 64-bit magic and freed
 *     with the matching g4q_*_free (runtime.cc:41-45, 900-912).
 *   - Device pointers are plain pointers on the current CUDA device; `stream` is a
 *     cudaStream_t passed as void* (NULL = legacy default stream). All compute calls are
 *     asynchronous on that stream. Uploads accept host or device source pointers.
 *   - Element types: bf16 values travel as uint16_t bit patterns; packed weights as uint32_t.
 *   - A handle or a stream is not safe for concurrent use by two host threads (the
 *     reference's single scheduler thread owns a target: crates/gemma4d-server/src/http.rs:421-470).
 *   - Compute calls on one device share library scratch: the stream-K GEMV's partial sums and
 *     arrival counters, the prefill GEMM's row scales and split-K partials. Calls that overlap on
 *     the GPU race on it, even on different streams or handles, so issue a device's compute calls
 *     on one stream or order them with events (as the reference's single scheduler thread issues
 *     its matmuls one after another). Decode plans, LoRA handles and the allreduce communicator own
 *     their scratch; the LM head's lives in its weight handle.
 *   - That scratch is never freed while the process runs: it grows at g4q_weight_create (GEMV
 *     slots) or at the first GEMM launch outside a stream capture that needs more (split-K
 *     partials), and a grown buffer replaces the old one without freeing it. A CUDA graph captured
 *     with any compute call therefore stays valid when larger weights are created later.
 */
#ifndef G4Q_H
#define G4Q_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4Q_ABI_VERSION 1u

/* Same numbering as Gemma4Status (native/gemma4_mlx/include/gemma4_mlx.h:12-21). */
typedef enum G4qStatus {
    G4Q_OK = 0,
    G4Q_ERR_INVALID_ARGUMENT = 1,
    G4Q_ERR_UNSUPPORTED_CONFIG = 2,
    G4Q_ERR_MODEL_LOAD = 3,
    G4Q_ERR_RUNTIME = 4,
    G4Q_ERR_MEMORY_GUARD = 5
} G4qStatus;

/* Rounding chain of the bf16 `scale * q + bias` (MLX's cannot be observed here). */
typedef enum G4qChain {
    G4Q_CHAIN_R1 = 1, /* bf16(scale*q + bias), one rounding */
    G4Q_CHAIN_R2 = 2  /* bf16(bf16(scale*q) + bias), one rounding per bf16 op (default) */
} G4qChain;

/* g4q_qmm_ex / g4q_lm_head_argmax flags */
#define G4Q_QMM_RMS_SCALE 0x1u /* y[m,:] *= 1/sqrt(mean(x[m,:]^2) + eps) (RMSNorm folded as an output scale) */
#define G4Q_QMM_OUT_F32 0x2u   /* y is fp32 instead of bf16 */

typedef struct G4qVersionInfo {
    uint32_t abi_version;
    const char* backend_name;
    const char* backend_version;
} G4qVersionInfo;

typedef struct G4qWeightInfo {
    int64_t rows;          /* N (output features) */
    int64_t cols;          /* K (input features) */
    int32_t bits;
    int32_t group_size;
    uint64_t device_bytes; /* packed + scales/biases in the kernel layout */
    int32_t device;
    int32_t fast_path_ok;  /* 1 when every scale is finite with |s| < 2^120 (qmm/GEMM requirement) */
    int32_t error_flags;   /* bit 1: g4q_dequantize saw a row id outside [0, rows) (that row was zeroed) */
} G4qWeightInfo;

typedef struct G4qWeight G4qWeight;

/* Replaces gemma4_runtime_version (gemma4_mlx.h:198; runtime.cc:798-808). */
G4qStatus g4q_runtime_version(G4qVersionInfo* out);
/* Replaces gemma4_get_last_error (gemma4_mlx.h:199; runtime.cc:816-823). */
G4qStatus g4q_get_last_error(char* buffer, size_t buffer_len);

/* ---- weights: the loader repack -------------------------------------------------------
 * Replaces the tensor residency of NativeTextModel::load (native_model.cc:3506-3590) for the
 * `{prefix}.weight/.scales/.biases` triple consumed by quantized_linear (native_model.cc:349-362).
 * g4q_weight_create allocates an empty N x K handle. bits 4 / group 64 (N % 16 == 0,
 * K % 64 == 0) is repacked into the kernel layout and runs every entry point below. The 8-bit
 * group-64 override the reference's manifest allows per module (model_manifest.cc:146-152), and
 * groups 32 / 128 at 4 or 8 bits as mlx::core accepts them (any N, K % group == 0), keep MLX's
 * layout on the device and run g4q_qmm/_ex, g4q_dequantize and export on generic CUDA-core
 * kernels; the fused LM head and the decode plan return G4Q_ERR_UNSUPPORTED_CONFIG for them. Any
 * other bits/group is G4Q_ERR_UNSUPPORTED_CONFIG.
 * g4q_weight_load copies the window [src_row0, src_row0+n_rows) x [src_k0, src_k0+K) of an
 * MLX-layout matrix (packed uint32 [src_rows, src_cols*bits/32], scales/biases bf16
 * [src_rows, src_cols/group], host or device memory) into rows [dst_row0, dst_row0+n_rows) of the
 * handle (4-bit g64: rows in multiples of 16). One call per matrix uploads it whole; windows give
 * the tensor-parallel column split (rows) and row split (K, group aligned), and several loads into
 * one handle concatenate projections that share an input (q|k|v, gate|up). Dequantised values
 * are preserved exactly (g4q_weight_export inverts the repack). */
G4qStatus g4q_weight_create(int64_t rows, int64_t cols, int32_t bits, int32_t group_size, G4qWeight** out);
G4qStatus g4q_weight_load(G4qWeight* w, int64_t dst_row0, const uint32_t* packed, const uint16_t* scales,
                          const uint16_t* biases, int64_t src_rows, int64_t src_cols, int64_t src_row0,
                          int64_t src_k0, int64_t n_rows, void* stream);
G4qStatus g4q_weight_free(G4qWeight* w);
G4qStatus g4q_weight_info(const G4qWeight* w, G4qWeightInfo* out);
/* Inverse repack into MLX layout (device pointers: packed [rows, cols*bits/32], scales/biases
 * [rows, cols/group]). */
G4qStatus g4q_weight_export(const G4qWeight* w, uint32_t* packed, uint16_t* scales, uint16_t* biases,
                            void* stream);

/* ---- repacked-weight cache ------------------------------------------------------------------
 * A versioned file of a handle's kernel-layout buffers, so a later load skips the repack (the
 * reference re-reads and re-evaluates the MLX safetensors at every NativeTextModel::load,
 * native_model.cc:3506-3590). File: a 64-byte header (magic "G4QWCACH", format version 1, kernel
 * layout 1, rows, cols, bits 4, group 64, the two payload sizes, an FNV-1a 64-bit checksum of the
 * payload), then the packed words and the scale|bias words, little-endian. 4-bit group-64 handles
 * only (G4Q_ERR_UNSUPPORTED_CONFIG otherwise). g4q_weight_open checks the header, the file size
 * and the checksum on the host before it touches the GPU (G4Q_ERR_MODEL_LOAD on any mismatch),
 * then creates a handle on the current device and uploads the buffers as they are. */
G4qStatus g4q_weight_save(const G4qWeight* w, const char* path);
G4qStatus g4q_weight_open(const char* path, G4qWeight** out);

/* ---- dequantize --------------------------------------------------------------------------
 * Replaces mlx::core::dequantize(..., "affine") -> bf16: the embedding gather of
 * quantized_embedding (native_model.cc:364-376: take rows, then dequantize) when row_ids is
 * non-NULL (out = bf16 [n_ids, cols]), or the whole matrix when row_ids is NULL
 * (out = bf16 [rows, cols]). Bit-exact with the chain selected. */
G4qStatus g4q_dequantize(const G4qWeight* w, const int32_t* row_ids, int64_t n_ids, uint16_t* out,
                         int32_t chain, void* stream);
/* Same op straight from MLX-layout device arrays (bits 4 or 8, group 32/64/128), as
 * mx.dequantize(w, scales, biases, group_size, bits, mode="affine") is called in
 * scripts/xr54_dequant_assistant.py:117-125. out = bf16 [rows, cols]. */
G4qStatus g4q_dequantize_mlx(const uint32_t* packed, const uint16_t* scales, const uint16_t* biases,
                             int64_t rows, int64_t cols, int32_t bits, int32_t group_size, int32_t chain,
                             uint16_t* out, void* stream);

/* ---- quantized matmul ----------------------------------------------------------------------
 * Replaces mlx::core::quantized_matmul(x, W, scales, biases, transpose=true, 64, 4, "affine")
 * followed by the bf16 cast of quantized_linear (native_model.cc:349-362; call sites :802,
 * :813, :821, :892, :934, :939, :949 and their decode/verify twins :993-1128, :1158-1281):
 * y[m, n] = sum_k x[m, k] * deq(W)[n, k], fp32 accumulation, bf16 out. x: bf16 [M, ldx],
 * y: bf16 [M, ldy], device memory, row strides in elements (multiples of 8). M <= 16 runs the
 * decode GEMV; larger M runs the tcgen05 dequant-GEMM. */
G4qStatus g4q_qmm(const G4qWeight* w, const uint16_t* x, int64_t M, int64_t ldx, uint16_t* y, int64_t ldy,
                  void* stream);
/* As g4q_qmm with G4Q_QMM_* flags: RMS_SCALE multiplies each output row by
 * 1/sqrt(mean(x[m,:]^2) + eps) (the RMSNorm of the input folded into the epilogue), OUT_F32
 * writes fp32 y (ldy in fp32 elements). */
G4qStatus g4q_qmm_ex(const G4qWeight* w, const uint16_t* x, int64_t M, int64_t ldx, void* y, int64_t ldy,
                     uint32_t flags, float eps, void* stream);

/* Which kernel g4q_qmm / g4q_qmm_ex runs for this weight at M rows, without launching anything (no
 * reference counterpart: MLX picks its kernels internally). kernel: G4Q_PATH_GEMV_STREAMK (the
 * stream-K decode GEMV, M <= 8), G4Q_PATH_GEMV_CLUSTER (cluster split-K GEMV for the other M <= 16
 * shapes), G4Q_PATH_GEMM (the tcgen05 dequant-GEMM, M > 16) or G4Q_PATH_GENERIC (8-bit / group
 * 32, 128 weights). splits: the GEMM's k-block split count (1 = every CTA owns whole tiles; a split
 * launch inside a stream capture whose split scratch is too small runs unsplit), 0 otherwise. */
#define G4Q_PATH_GEMV_STREAMK 1
#define G4Q_PATH_GEMV_CLUSTER 2
#define G4Q_PATH_GEMM 3
#define G4Q_PATH_GENERIC 4
G4qStatus g4q_qmm_path(const G4qWeight* w, int64_t M, int32_t* kernel, int32_t* splits);

/* Replaces the pair model_dtype(fast::rms_norm(h, weight, eps)) -> quantized_linear of
 * layer_forward (native_model.cc:910-913 -> q/k/v, 929-932 -> gate/up; the decode twins
 * :993-1018, :1318-1321): y = qmm(bf16(weight * bf16(x * inv))) with inv = 1/sqrt(mean(x^2) + eps)
 * per row. At M <= 8 on a 4-bit group-64 weight the norm is fused into the stream-K GEMV's x
 * staging (one launch, x read twice from L2, no normalized copy in HBM); xn may be NULL there, and
 * when given it also receives the normalized rows. Otherwise xn (bf16 [M, ldxn], 16-byte aligned)
 * is required: the normalized rows are written there first and the matmul reads them. weight:
 * bf16 [cols], 16-byte aligned. */
G4qStatus g4q_qmm_norm(const G4qWeight* w, const uint16_t* x, int64_t M, int64_t ldx, const uint16_t* weight,
                       float eps, uint16_t* xn, int64_t ldxn, uint16_t* y, int64_t ldy, void* stream);

/* Replaces gate = quantized_linear(h, gate_proj), up = quantized_linear(h, up_proj),
 * act = geglu(gate, up) of layer_forward (native_model.cc:934-945; decode twin :1318-1321):
 * act = bf16 [M, rows/2] (row stride ld_act) of the GeGLU of the two bf16 matmul outputs. w is a
 * PAIRED gate|up weight: rows [64j, 64j+32) hold gate rows [32j, 32j+32) and rows [64j+32, 64j+64)
 * the same up rows (load each 32-row slice with g4q_weight_load; I = rows/2 must be a multiple of
 * 32). flags: 0 or G4Q_QMM_RMS_SCALE. At M <= 8 the GeGLU runs in the stream-K GEMV's epilogue and
 * at M > 16 in the tcgen05 GEMM's epilogue (or its split-K reduction): one launch, gate and up never
 * reach HBM, and y may be NULL. For 9 <= M <= 16 y (bf16 [M, rows], contiguous) is required and
 * receives the paired matmul output before the GeGLU pass. Bit-identical either way to g4q_qmm
 * followed by g4q_geglu on the pairs. norm_weight (bf16 [cols], or NULL):
 * x is first normalized as by g4q_qmm_norm (pre_feedforward_layernorm, :929-932), so the norm,
 * both projections and the GeGLU are one launch; only on the fused path (M <= 8, flags 0): other
 * calls with a norm weight are rejected, normalize with g4q_rms_norm first there. */
G4qStatus g4q_qmm_geglu(const G4qWeight* w, const uint16_t* x, int64_t M, int64_t ldx, const uint16_t* norm_weight,
                        uint32_t flags, float eps, uint16_t* y, uint16_t* act, int64_t ld_act, void* stream);

/* ---- tied LM head with fused softcap + greedy argmax ----------------------------------------
 * Replaces target_logits_for_hidden (native_model.cc:1782-1795: quantized_matmul against
 * embed_tokens, bf16, tanh(l/30)*30 in bf16) and the greedy argmax of its callers (:3825,
 * :3934; first index wins ties) in one pass over the 262144 x 3840 table. softcap <= 0 skips
 * the softcap. Per row m of x (M <= 16): tokens[m] = row_offset + argmax, values[m] = the
 * softcapped logit (as float), keys[m] = order-preserving 64-bit key
 * ((ordered float bits) << 32 | (0xFFFFFFFF - token)) for combining vocabulary shards with
 * a max. Any of tokens/values/keys/logits may be NULL; logits (bf16 [M, ld_logits]) receives
 * the pre-softcap bf16 logits when given. Uses a small scratch owned by the handle: calls on
 * one handle must not overlap on the GPU. */
G4qStatus g4q_lm_head_argmax(const G4qWeight* w, const uint16_t* x, int64_t M, int64_t ldx, float softcap,
                             uint32_t flags, float eps, int64_t row_offset, uint16_t* logits,
                             int64_t ld_logits, int32_t* tokens, float* values, uint64_t* keys,
                             void* stream);

/* ---- allocation-free LM head ---------------------------------------------------------------------
 * No counterpart in the reference. Same result as g4q_lm_head_argmax (same kernel), for callers
 * that cannot allocate device memory when they call it: code inside a CUDA stream capture, where
 * cudaMalloc is not allowed, and host runtimes that own every device byte through a pre-sized
 * arena and forbid driver allocations once serving starts. It allocates nothing and needs no
 * weight handle: the caller passes the weight in kernel layout v1 in memory it owns (packed:
 * (cols/64) x (rows/16) blocks of 128 uint32, block (g, r) at word (g*rows/16 + r)*128; sb:
 * (cols/64) x rows words scale | bias << 16 -- the layout g4q_weight_load builds, documented with
 * the oracle's g4o_repack), plus x and the outputs. Its scratch (16 argmax keys, a ticket
 * counter and an error word, 144 bytes) is a static array inside the library: every GPU that loads
 * libg4q holds it until the process exits, so M is limited to 16 rows (larger M is rejected with
 * G4Q_ERR_INVALID_ARGUMENT). Each call clears the keys and the ticket on `stream` before its
 * kernel. All calls on one device share that scratch, so calls that overlap on the GPU race:
 * serialise them. The first call on a device looks up the scratch's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before any stream capture.
 * Precondition, as for a handle (G4qWeightInfo.fast_path_ok): every scale finite with
 * |scale| < 2^120. A handle's scales are scanned at load time; caller-owned memory is not, so the
 * kernel checks the scales it reads, and a violation records code 50 in the error word that
 * g4q_device_error reports (tokens, values, keys and logits of that call are then invalid). */
G4qStatus g4q_lm_head_argmax_noalloc(const uint32_t* packed, const uint32_t* sb, int64_t rows, int64_t cols,
                                     const uint16_t* x, int64_t M, int64_t ldx, float softcap, uint32_t flags,
                                     float eps, int64_t row_offset, uint16_t* logits, int64_t ld_logits,
                                     int32_t* tokens, float* values, uint64_t* keys, void* stream);

/* ---- LoRA delta on a quantized linear's output -------------------------------------------------
 * One adapter module as the reference builds it in NativeLoraAdapter::load
 * (native/gemma4_mlx/src/native_model.cc:3296-3432): lora_A [rank, cols] and lora_B [rows, rank]
 * converted to fp32 (:3419-3420), scale = alpha / rank (:3378). Validation as there: rank > 0,
 * alpha finite and > 0. lora_a / lora_b: fp32, row-major, host or device memory (copied; lora_B is
 * stored transposed). cols % 8 == 0, rank <= 256. max_tokens (1..65536) sizes the handle's fp32
 * scratch for the low-rank activations; g4q_lora_apply processes larger M in chunks of it, so it
 * allocates nothing. */
typedef struct G4qLora G4qLora;
G4qStatus g4q_lora_create(int64_t rows, int64_t cols, int32_t rank, float alpha, const float* lora_a,
                          const float* lora_b, int32_t max_tokens, G4qLora** out);
/* Replaces add_lora_delta_if_active (native_model.cc:316-328), the tail of quantized_linear
 * (:349-362): in place on y (bf16 [M, ldy], the quantized matmul's bf16 output for the same x),
 *   y = bf16(y + bf16(fp32(fp32(x) @ lora_A^T @ lora_B^T) * bf16(alpha / rank)))
 * with fp32 accumulation. x: bf16 [M, ldx], 16-byte aligned, ldx % 8 == 0. Asynchronous on
 * `stream`; calls on one handle share its scratch, so serialise them. */
G4qStatus g4q_lora_apply(const G4qLora* lora, const uint16_t* x, int64_t M, int64_t ldx, uint16_t* y, int64_t ldy,
                         void* stream);
G4qStatus g4q_lora_free(G4qLora* lora);

/* ---- the MLP's elementwise neighbours ------------------------------------------------------------
 * Replaces geglu (native/gemma4_mlx/src/native_model.cc:378-386; called at :945): per element,
 * bf16 0.5*g*(1 + tanh(sqrt(2/pi)*(g + 0.044715*g^3))) * up with the constants rounded to bf16 and
 * every one of the nine ops rounded to bf16, as the reference's bf16 MLX ops do, in one launch.
 * gate / up / out: bf16 [M, I] with row strides ld_* (elements); I, the strides and the pointers
 * 16-byte multiples (I % 8 == 0). gate and up may be the two halves of one gate|up matmul output. */
G4qStatus g4q_geglu(const uint16_t* gate, int64_t ld_gate, const uint16_t* up, int64_t ld_up, int64_t M, int64_t I,
                    uint16_t* out, int64_t ld_out, void* stream);
/* Replaces model_dtype(fast::rms_norm(x, weight, eps)) (native_model.cc:910-913, 920-923,
 * 929-932, 954-957; values norm without weight :844): per row, inv = 1/sqrt(mean(x^2) + eps) in
 * fp32, out = bf16(weight * bf16(x * inv)). weight: bf16 [K] or NULL. x / out: bf16 [M, ld],
 * K % 8 == 0, 16-byte aligned rows. out may equal x (in place). */
G4qStatus g4q_rms_norm(const uint16_t* x, int64_t ldx, const uint16_t* weight, int64_t M, int64_t K, float eps,
                       uint16_t* out, int64_t ld_out, void* stream);

/* The tail of each sub-block of layer_forward in one pass: out = bf16(bf16(residual + norm) * scale)
 * with norm = model_dtype(fast::rms_norm(x, weight, eps)) as g4q_rms_norm computes it
 * (native_model.cc:954-968: post_feedforward_layernorm, the MLP residual add, layer_scalar; :920-926:
 * post_attention_layernorm and the attention residual add, layer_scalar NULL). layer_scalar: one bf16
 * value in device memory (the checkpoint's `.layer_scalar`), or NULL. residual / out: bf16 [M, ld],
 * 16-byte aligned rows; out may equal x or residual. */
G4qStatus g4q_rms_norm_residual(const uint16_t* x, int64_t ldx, const uint16_t* weight, int64_t M, int64_t K,
                                float eps, const uint16_t* residual, int64_t ld_res, const uint16_t* layer_scalar,
                                uint16_t* out, int64_t ld_out, void* stream);

/* ---- decode plan: every quantized matmul of one decode step in one persistent kernel ----------
 * Replaces the per-token chain of quantized_linear calls of the decode drivers
 * (native_model.cc:1843-1911 decode_last_logits -> 48 x target_layer_decode_forward :1284-1328 ->
 * target_logits_for_hidden :1782-1795 -> argmax :3825). Phase i computes
 * y_i = x_i . deq(W_i)^T (RMS_SCALE / OUT_F32 as for g4q_qmm_ex); x_i may be the output of phase
 * i-1 (the kernel waits for phase i-1 to finish on every SM before staging x_i). The last phase may
 * carry G4Q_PHASE_ARGMAX: its y is not stored; instead each row's bf16 logits go through the
 * softcap and a first-index argmax, reported as in g4q_lm_head_argmax. Pointers are fixed at plan
 * creation (device memory); g4q_decode_plan_run launches one cooperative grid on `stream` and
 * allocates nothing, so it can be captured in a CUDA graph. max_tokens (the M of every step: 1, or
 * the MTP-verify widths 2, 4 and 8 of decode_block_logits, native_model.cc:1954-2026) fixes the plan's
 * tokens per step; x and y are then [M, ld] row-major, and run takes exactly that M (logits, when
 * given, [M, ld_logits]; tokens / values / keys hold M entries). Runs of one plan must not overlap on
 * the GPU. */
#define G4Q_PHASE_ARGMAX 0x4u
/* Row-parallel phase of a tensor-parallel plan (o_proj, down_proj split along K): every rank's
 * partial sums are added across ranks inside the kernel (the allreduce after o/down). */
#define G4Q_PHASE_ALLREDUCE 0x8u
/* The phase's weight is a paired gate|up weight (see g4q_qmm_geglu): its output y is
 * geglu(gate, up), bf16 [M, rows/2], with the same roundings as the matmul followed by g4q_geglu. */
#define G4Q_PHASE_GEGLU 0x10u

typedef struct G4qDecodePhase {
    const G4qWeight* weight;
    const uint16_t* x; /* bf16 [M, ldx] */
    int64_t ldx;
    void* y;           /* bf16 or fp32 [M, ldy]; unused by the argmax phase */
    int64_t ldy;
    uint32_t flags;
} G4qDecodePhase;

typedef struct G4qDecodePlan G4qDecodePlan;

G4qStatus g4q_decode_plan_create(const G4qDecodePhase* phases, int32_t n_phases, int32_t max_tokens,
                                 G4qDecodePlan** out);

/* Elementwise work a phase applies to its staged x before its matmul: the neighbours of the linears
 * in layer_forward (native_model.cc:899-970) -- a sub-block's post-norm, residual add and
 * layer_scalar (:920-926, :954-968, as g4q_rms_norm_residual computes them) and the next sub-block's
 * input norm (:910-913, :929-932, as g4q_rms_norm computes it). With v the staged values (the
 * previous phase's output, or the plan's input for phase 0), per token:
 *   if post_norm_weight: v = bf16(post_norm_weight * bf16(v * inv(v)))
 *   residual 1: the residual stream starts as v;  residual 2: v = bf16(residual + v), then, with a
 *               layer_scalar, v = bf16(v * layer_scalar); either way v is the new residual stream
 *               (kept by the plan; also copied to residual_out [M, ld_residual_out] when given)
 *   if norm_weight: v = bf16(norm_weight * bf16(v * inv(v)))
 * with inv(v) = 1/sqrt(mean(v^2) + eps) in fp32. Weights are bf16 [K], the layer scalar one bf16
 * value, all in device memory. A phase with a prologue takes no G4Q_QMM_RMS_SCALE and must read all
 * of the previous phase's output (or be phase 0). */
typedef struct G4qPhasePrologue {
    const uint16_t* post_norm_weight;
    int32_t residual;             /* 0 none, 1 start the residual stream, 2 add to it */
    const uint16_t* layer_scalar;
    const uint16_t* norm_weight;
    uint16_t* residual_out;
    int64_t ld_residual_out;
    float eps;
} G4qPhasePrologue;

/* As g4q_decode_plan_create_tp (rank 0 of 1 for a single GPU) with a prologue per phase: prologues
 * is NULL or an array of n_phases entries (all-zero entries for phases without one). */
G4qStatus g4q_decode_plan_create_ex(const G4qDecodePhase* phases, const G4qPhasePrologue* prologues,
                                    int32_t n_phases, int32_t max_tokens, int32_t rank, int32_t n_ranks,
                                    G4qDecodePlan** out);
G4qStatus g4q_decode_plan_run(G4qDecodePlan* plan, int64_t M, float eps, float softcap, int64_t row_offset,
                              int32_t* tokens, float* values, uint64_t* keys, uint16_t* logits, int64_t ld_logits,
                              void* stream);
G4qStatus g4q_decode_plan_free(G4qDecodePlan* plan);
/* Per-phase timeline of a plan's runs, a profiling aid (no reference counterpart; the reference
 * profiles its own phases separately, gemma4_mlx.h:141). *words receives the size of a trace in
 * 64-bit words: grid CTAs x phases x (3 + 16) globaltimer stamps (ns), per CTA and phase: entry,
 * x's producers done, x staged with its RMS scale, then the end of each of the 16 warps' units.
 * With a device buffer of at least that many words set, later runs launch the tracing build of the
 * kernel and overwrite the buffer; NULL switches back to the regular build. */
G4qStatus g4q_decode_plan_trace(G4qDecodePlan* plan, uint64_t* buffer, int64_t* words);

/* ---- tensor-parallel decode plans (one process per GPU) ---------------------------------------
 * Replaces the per-rank linears plus the NCCL allreduce after o_proj / down_proj and the vocab-shard
 * argmax combine of a tensor-parallel decode step (the reference runs one device; its column/row
 * split is the MLX sharding of the same linears). Each rank builds the plan of its shards with
 * g4q_decode_plan_create_tp(rank, n_ranks); phases with G4Q_PHASE_ALLREDUCE write their partial
 * sums into the slot buffers of every rank over NVLink and every rank sums them in the same order,
 * so all ranks see bit-identical activations. The LM-head argmax keys are exchanged the same way at
 * the end of each step (tokens/values/keys are the global result on every rank). Wiring: every rank
 * exports its buffers (g4q_decode_plan_buffers -> g4q_ipc_handle), the handles are exchanged by
 * the host (e.g. an allgather over the process group), each rank opens its peers' handles
 * (g4q_ipc_open) and passes the pointers indexed by rank to g4q_decode_plan_set_peers (the own
 * rank's entries are ignored). All ranks must run the same number of steps. */
G4qStatus g4q_decode_plan_create_tp(const G4qDecodePhase* phases, int32_t n_phases, int32_t max_tokens,
                                    int32_t rank, int32_t n_ranks, G4qDecodePlan** out);
G4qStatus g4q_decode_plan_buffers(G4qDecodePlan* plan, void** slots, uint64_t* slot_bytes, void** xkeys,
                                  uint64_t* xkey_bytes);
G4qStatus g4q_decode_plan_set_peers(G4qDecodePlan* plan, void* const* slots, void* const* xkeys);

/* CUDA IPC of device allocations between the processes of one node (no reference counterpart:
 * the reference runs one process per model). */
#define G4Q_IPC_HANDLE_BYTES 64
G4qStatus g4q_ipc_handle(const void* device_ptr, uint8_t* handle);
G4qStatus g4q_ipc_open(const uint8_t* handle, void** device_ptr);
G4qStatus g4q_ipc_close(void* device_ptr);

/* ---- tensor-parallel allreduce -----------------------------------------------------------------
 * The TP communicator of the boundary: allreduce(sum) of a bf16 or fp32 vector across the ranks of
 * one node, for the sum after o_proj / down_proj when the linears run sharded outside a decode plan
 * (prefill chunks, verify blocks). No reference counterpart: the reference runs one process per
 * model; this replaces the collective of the Megatron split of the same linears. Over NVLink peer
 * memory (CUDA IPC); no library kernel touches peer memory: one shot (every rank pushes its vector
 * to every rank) up to 256 KB, two shots (reduce-scatter + all-gather, chunked) above. Sums are fp32
 * in rank order, so every rank gets the same bits; every wait is bounded (code 40 in the device
 * error word). Wiring as for the TP decode plan: g4q_comm_create on every rank, export
 * g4q_comm_buffer with g4q_ipc_handle, exchange the handles on the host, g4q_ipc_open the peers'
 * and pass them indexed by rank to g4q_comm_set_peers. Collective: every rank calls g4q_allreduce
 * the same number of times with the same count and dtype; calls on one communicator are serialised
 * on `stream`. data: device pointer, 16-byte aligned, count * element size a multiple of 16,
 * count <= max_elems. */
typedef struct G4qComm G4qComm;
#define G4Q_DTYPE_BF16 0
#define G4Q_DTYPE_F32 1
G4qStatus g4q_comm_create(int32_t rank, int32_t n_ranks, int64_t max_elems, G4qComm** out);
G4qStatus g4q_comm_buffer(const G4qComm* comm, void** buffer, uint64_t* bytes);
G4qStatus g4q_comm_set_peers(G4qComm* comm, void* const* peer_buffers);
G4qStatus g4q_allreduce(G4qComm* comm, void* data, int64_t count, int32_t dtype, void* stream);
G4qStatus g4q_comm_free(G4qComm* comm);

/* ---- device-side failure detection ----------------------------------------------------------
 * Every wait inside a libg4q kernel is bounded; a wait that gives up records a nonzero code in a
 * per-device error word and the kernel runs to its end (its results are then invalid). This
 * reads the word for the current device (synchronising it) and optionally clears it; it also
 * reports (and clears) code 50 of g4q_lm_head_argmax_noalloc, and allocates nothing. No
 * reference counterpart: the reference's MLX graph has no device-side waits. */
G4qStatus g4q_device_error(int32_t* code, int32_t reset);

/* ---- seeded synthetic data (no reference counterpart: benchmark / test inputs) ---------------
 * Counter-based splitmix64 generator identical to the CPU oracle's: MLX-layout packed
 * (q ~ U{0..15}), scale = bf16(U(0.002, 0.02)), bias = bf16(-8*scale + 1e-3*N(0,1)); and
 * bf16 ~ N(0,1) activations. Device pointers. */
G4qStatus g4q_synth_matrix(uint64_t seed, int64_t rows, int64_t cols, int32_t bits, int32_t group_size,
                           uint32_t* packed, uint16_t* scales, uint16_t* biases, void* stream);
G4qStatus g4q_synth_normal_bf16(uint64_t seed, int64_t count, uint16_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* G4Q_H */
