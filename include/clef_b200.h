/*
 * clef_b200.h — C ABI of the B200-native prefill backend for clef-rs.
 *
 * One shared library, libclef_b200.so, exports every symbol declared here.
 * The ABI carries plain pointers, sizes and a cudaStream_t (passed as void*),
 * never a framework type. It replaces, one function per operator, the Candle
 * CustomOp objects that the reference engine dispatches on its device path,
 * plus an engine handle that replaces the reference's backbone prefill loop.
 *
 * Conventions shared by every entry point
 *   - Return value: CLEF_OK (0) or a nonzero clef_status. Shapes, dtypes and
 *     byte ranges are validated BEFORE anything is launched or allocated, as the
 *     reference's dispatch wrappers do (crates/core/src/models/metal.rs:280-290,
 *     :303-307, :507-527). The message of the last failure on the calling host
 *     thread is returned by clef_last_error().
 *   - Operator entry points (clef_rmsnorm ... clef_attention_gqa) take DEVICE
 *     pointers, are stream-ordered on `stream` (NULL = the legacy default
 *     stream), never synchronise the host and never allocate: callers pass
 *     outputs and, where a *_workspace_size query exists, a workspace.
 *   - Engine entry points take HOST pointers for ids and results; the engine
 *     owns its device memory and synchronises once per call, like
 *     DirectEngine::decide (crates/core/src/runtime.rs:715).
 *   - Threading: one owner thread per device and per engine handle
 *     (crates/core/src/runtime.rs:1062-1075). Handles are not shared.
 *   - Element types: F32 = IEEE float, BF16 = bfloat16 bit pattern (uint16_t).
 *   - Weight matrices follow the reference layout W[out, in] (row-major, the
 *     reduction dimension contiguous), i.e. y = x W^T.
 */
#ifndef CLEF_B200_H
#define CLEF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum clef_status {
  CLEF_OK = 0,
  CLEF_ERR_INVALID = 1,      /* bad shape, dtype, pointer or range          */
  CLEF_ERR_CUDA = 2,         /* a CUDA runtime/driver call failed           */
  CLEF_ERR_UNSUPPORTED = 3,  /* dimensions this build does not implement    */
  CLEF_ERR_NOMEM = 4,        /* device or host allocation failed            */
  CLEF_ERR_CANCELLED = 5,    /* clef_engine_cancel() was observed           */
  CLEF_ERR_DEVICE_TIMEOUT = 6 /* a bounded device-side wait gave up        */
} clef_status;

typedef enum clef_dtype { CLEF_F32 = 0, CLEF_BF16 = 1 } clef_dtype;

/* Message for the last failing call on this host thread ("" when none). */
const char* clef_last_error(void);
/* Library version string. */
const char* clef_version(void);

/* ------------------------------------------------------------------------ */
/* Model geometry. Mirrors TextConfig (crates/core/src/models/qwen.rs:42-58). */
/* ------------------------------------------------------------------------ */
#define CLEF_MAX_LAYERS 128

typedef struct clef_config {
  int32_t hidden_size;              /* 2560 at the benchmark geometry       */
  int32_t intermediate_size;        /* 9216                                  */
  int32_t num_hidden_layers;        /* 32                                    */
  int32_t vocab_size;               /* 248320                                */
  int32_t num_attention_heads;      /* 16                                    */
  int32_t num_key_value_heads;      /* 4                                     */
  int32_t head_dim;                 /* 256                                   */
  int32_t linear_num_key_heads;     /* 16                                    */
  int32_t linear_num_value_heads;   /* 32                                    */
  int32_t linear_key_head_dim;      /* 128                                   */
  int32_t linear_value_head_dim;    /* 128                                   */
  int32_t linear_conv_kernel_dim;   /* 4 (the only supported value)          */
  int32_t rotary_dim;               /* head_dim * partial_rotary_factor      */
  int32_t head_outputs;             /* schema-head logits (7), 0 = no head   */
  float rms_norm_eps;               /* 1e-6                                  */
  double rope_theta;                /* 1e7                                   */
  /* layer_types[i]: 1 = full_attention, 0 = linear_attention (DeltaNet).    */
  uint8_t layer_types[CLEF_MAX_LAYERS];
} clef_config;

/* Validates a configuration against what the kernels implement. */
int clef_config_validate(const clef_config* cfg);

/* ------------------------------------------------------------------------ */
/* Operators (device pointers, stream-ordered, caller-allocated outputs).    */
/* ------------------------------------------------------------------------ */

/* Offset-free RMSNorm: out = x * rsqrt(mean(x^2) + eps) * weight, per row.
 * `weight` already holds (1 + w) for offset norms, exactly as Norms::load
 * precomputes it. x is F32 [rows, width]; out is F32 or BF16 [rows, width].
 * Replaces RmsKernel (crates/core/src/models/pointwise.rs:42-100) and
 * ops::rms_inner (crates/core/src/models/ops.rs:24-32). */
int clef_rmsnorm(const float* x, const float* weight, int64_t rows, int32_t width,
                 float eps, int32_t out_dtype, void* out, void* stream);

/* Four-tap causal depthwise convolution, taps accumulated oldest to newest.
 * x F32 [T, width] with row stride ldx; history F32 [history_rows, width]
 * (0..3 rows that precede x[0]; missing rows are zero); weight F32 [width, 4];
 * out F32 [T, width]. Replaces ConvKernel (pointwise.rs:133-192) and
 * causal_convolution (crates/core/src/models/qwen.rs:765-796). */
int clef_conv4(const float* x, int64_t ldx, const float* history, int32_t history_rows,
               const float* weight, int64_t T, int32_t width, float* out, void* stream);

/* Gated-DeltaNet prologue for one sequence: conv4 over the q|k|v columns of
 * the fused projection, SiLU, L2 normalisation of q and k (eps 1e-6 inside the
 * square root), q scaling by 1/sqrt(dk), and the decay / beta gates
 *   g = -exp(A_log) * softplus(a + dt_bias),  beta = sigmoid(b).
 * proj F32 [T, ldp]: columns [0, 2*Hk*dk + Hv*dv) are q|k|v, column a_col+h is
 * a_h and b_col+h is b_h. Outputs: q, k F32 [T, Hk, dk]; v F32 [T, Hv, dv];
 * g, beta F32 [T, Hv]. Replaces ConvKernel + DeltaPrepareKernel
 * (pointwise.rs:133-281; pointwise.metal:46-114) and the gate lines of
 * Delta::forward (qwen.rs:616-627). */
int clef_delta_prologue(const float* proj, int64_t ldp, int32_t a_col, int32_t b_col,
                        const float* history, int32_t history_rows,
                        const float* conv_weight, const float* dt_bias, const float* a_log,
                        int64_t T, int32_t Hk, int32_t Hv, int32_t dk, int32_t dv,
                        float* q, float* k, float* v, float* g, float* beta, void* stream);

/* Workspace bytes needed by clef_delta_scan for `nseq` sequences totalling
 * `total_tokens` tokens with Hk key heads and Hv value heads (0 for
 * unsupported dimensions). The workspace holds the chunk tables and, per
 * 64-token chunk, the split K/Q tiles (64 KB per key head) and the solved
 * T diag(beta), P tiles and decay vectors (33 KB per value head). */
size_t clef_delta_scan_workspace_size(int64_t total_tokens, int32_t nseq, int32_t Hk, int32_t Hv,
                                      int32_t dk, int32_t dv);

/* Chunked (C = 64) gated-DeltaNet scan over one or more packed sequences.
 * q, k F32 [T, Hk, dk] already L2-normalised (q also scaled by 1/sqrt(dk));
 * v F32 [T, Hv, dv]; g (log decay, <= 0) and beta F32 [T, Hv]; v-head h reads
 * k-head h / (Hv / Hk). For each token, per head, the result equals the
 * reference recurrence S <- S e^g; d = (v - S^T k) beta; S <- S + k d^T;
 * o = S^T q (delta_recurrence_prefill, qwen.rs:826-882; clef_delta,
 * delta.metal:18-131).
 * cu_seqlens: HOST int64 [nseq + 1] token offsets (NULL = one sequence of T).
 * init_state: F32 [nseq or 1, Hv, dk, dv] initial states, NULL = zeros;
 *   init_shared = 1 makes every sequence start from the same state.
 * capture: if > 0 (nseq must be 1), the state after token `capture` is
 *   written to capture_state [Hv, dk, dv] (CachedDelta, metal.rs:340-413).
 * final_state: F32 [nseq, Hv, dk, dv] or NULL.
 * out: F32 [T, Hv, dv]. Dimensions: dk = 128, dv = 128, Hv % Hk == 0. */
int clef_delta_scan(const float* q, const float* k, const float* v, const float* g,
                    const float* beta, int64_t T, int32_t Hk, int32_t Hv, int32_t dk,
                    int32_t dv, const int64_t* cu_seqlens, int32_t nseq,
                    const float* init_state, int32_t init_shared, int64_t capture,
                    float* capture_state, float* final_state, float* out,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of clef_delta_scan (no counterpart in the
 * reference). Some callers cannot call cudaMalloc or pass a workspace: hosts
 * whose allocator owns all device memory behind an op signature with no
 * room for an extra buffer, and latency-critical loops that must not hit
 * cudaMalloc's implicit synchronisation. Same arguments and results as
 * clef_delta_scan minus the workspace; the per-sequence offsets go into a
 * fixed device array inside this library (at most 4096 sequences per call;
 * more is rejected with CLEF_ERR_UNSUPPORTED). It allocates nothing. The
 * first call on each device resolves the array's device address and should
 * come before any stream capture. cu_seqlens is read by a copy ordered on
 * `stream` (asynchronous when the buffer is page-locked): keep it unchanged
 * until the stream has reached the call. All calls on a device share the
 * array: calls whose work overlaps on the GPU race, so serialise them on one
 * stream. */
int clef_delta_scan_noalloc(const float* q, const float* k, const float* v, const float* g,
                            const float* beta, int64_t T, int32_t Hk, int32_t Hv, int32_t dk,
                            int32_t dv, const int64_t* cu_seqlens, int32_t nseq,
                            const float* init_state, int32_t init_shared, int64_t capture,
                            float* capture_state, float* final_state, float* out, void* stream);

/* DeltaKernel and CachedDelta in the reference's packed layout
 * (crates/core/src/models/metal.rs:79-413, delta.metal:18-131): `packed` F32
 * [T, H, 2 dk + dv + 2] holds per token and head q | k | v | decay | beta,
 * with q and k already normalised (and q scaled) by the caller and decay =
 * e^g. Output `out` F32: o [T, H, dv], followed by the state after token
 * `capture` [H, dk, dv] when capture > 0 (CachedDelta's flat output, so `out`
 * holds T H dv + H dk dv floats then). initial_state: F32 [H, dk, dv] to
 * resume from, or NULL for zeros. Dimensions as the reference's `dimensions`
 * check (metal.rs:280-290): 1 <= T <= 4096, 1 <= H <= 32, dk a power of two
 * up to 128, 1 <= dv <= 128, 0 <= capture <= T; anything else is
 * CLEF_ERR_INVALID before any launch. Per-token F32 recurrence; a capture
 * followed by a resume reproduces the uninterrupted run bit for bit.
 * Stream-ordered, no workspace. */
int clef_delta_packed(const float* packed, int64_t T, int32_t H, int32_t dk, int32_t dv,
                      const float* initial_state, int64_t capture, float* out, void* stream);

/* DeltaPrepareKernel (crates/core/src/models/pointwise.rs:195-279,
 * pointwise.metal:69-114): from the post-conv rows `mixed` F32 [T, ldm]
 * (q | k | v = Hk*128 | Hk*128 | Hv*128 columns), the log-decay g and beta
 * F32 [T, Hv], writes the packed input of clef_delta_packed with dk = dv = 128:
 * out F32 [T, Hv, 386] = q / sqrt(|q|^2 + 1e-6) / sqrt(128) | k / sqrt(|k|^2 +
 * 1e-6) | v | e^g | beta, q and k of value head h taken from key head
 * h / (Hv / Hk). 1 <= T <= 4096 as in the reference. */
int clef_delta_prepare_packed(const float* mixed, int64_t ldm, const float* g, const float* beta, int64_t T,
                              int32_t Hk, int32_t Hv, float* out, void* stream);

/* GEMM epilogues for clef_gemm_bf16. */
typedef enum clef_epilogue {
  CLEF_EPI_STORE_BF16 = 0,  /* out BF16 [M, ldo] = X W^T                    */
  CLEF_EPI_STORE_F32 = 1,   /* out F32  [M, ldo] = X W^T                    */
  CLEF_EPI_ADD_F32 = 2      /* out F32  [M, ldo] += X W^T (residual stream) */
} clef_epilogue;

/* Y[M, N] = X[M, K] * W[N, K]^T, BF16 operands, F32 accumulation on the
 * tcgen05 tensor cores. K % 64 == 0, N % 16 == 0, ldo >= N. Replaces
 * GemmKernel / TileKernel (crates/core/src/models/neural.rs:151-280) and the
 * candle_nn::Linear call of Projection::forward_inner (projection.rs:82-95). */
int clef_gemm_bf16(const uint16_t* X, const uint16_t* W, int64_t M, int32_t N, int32_t K,
                   int32_t epilogue, void* out, int64_t ldo, void* stream);

/* Same product with the activation carried as a split BF16 pair: X2 BF16
 * [M, 2K] holds hi = bf16(x) in columns [0, K) and lo = bf16(x - hi) in
 * [K, 2K); the result is (hi + lo) W^T, i.e. x W^T to about 2^-17 of x, at
 * twice the tensor-core work (no counterpart in the reference; the F32-class
 * projection of the engine's CLEF_PRECISION_SPLIT). */
int clef_gemm_bf16_split(const uint16_t* X2, const uint16_t* W, int64_t M, int32_t N, int32_t K,
                         int32_t epilogue, void* out, int64_t ldo, void* stream);

/* Fused SwiGLU projection: out BF16 [M, N] = silu(X Wg^T) * (X Wu^T), with
 * Wg, Wu BF16 [N, K]. Replaces the gated TileKernel path and
 * Projection::gated_forward (projection.rs:67-81; neural.metal:99-125). */
int clef_gemm_swiglu(const uint16_t* X, const uint16_t* Wg, const uint16_t* Wu, int64_t M,
                     int32_t N, int32_t K, uint16_t* out, void* stream);

/* Causal grouped-query attention with the lower-right mask (query i of Tq
 * sees keys j <= i + Tk - Tq), scale 1/sqrt(d), online softmax in F32 on the
 * tcgen05 tensor cores (BF16 q, k, v and probabilities, F32 accumulation).
 * q BF16 [Hq, Tq, d], k, v BF16 [Hkv, Tk, d], out F32 [Hq, Tq, d].
 * Query head h reads kv head h / (Hq / Hkv). d = 256, Tq <= Tk. The
 * workspace (256-byte aligned, clef_attention_gqa_workspace_size bytes)
 * holds the token-major q/k and transposed v the kernel reads.
 * Replaces AttentionKernel (metal.rs:415-633) and ops::attention
 * (ops.rs:62-143). */
size_t clef_attention_gqa_workspace_size(int32_t Hq, int32_t Hkv, int64_t Tq, int64_t Tk);
int clef_attention_gqa(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t Hq,
                       int32_t Hkv, int64_t Tq, int64_t Tk, int32_t d, float* out,
                       void* workspace, size_t workspace_bytes, void* stream);

/* The same attention on the tcgen05 tensor cores, in the engine's layouts:
 * q BF16 [Tq, Hq, 256] and k BF16 [Tk, Hkv, 256] token-major; V given
 * transposed, vt BF16 [Hkv * 256, vt_pitch] (row = kv head * 256 + feature,
 * column = key); out F32 [Tq, Hq, 256]. Keys [0, Tk - Tq) act as a shared
 * prefix; Tk - Tq and vt_pitch must be multiples of 8. */
int clef_attention_gqa_vt(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int32_t Hq,
                          int32_t Hkv, int64_t Tq, int64_t Tk, int32_t d, int64_t vt_pitch,
                          float* out, void* stream);

/* Contiguous copy of a strided view (up to 4 dims, element size 2 or 4).
 * Replaces CompactCopy (metal.rs:26-77). */
int clef_compact_copy(const void* src, int32_t ndim, const int64_t* dims,
                      const int64_t* strides, int32_t elem_size, void* dst, void* stream);

/* ------------------------------------------------------------------------ */
/* Engine: the hybrid backbone prefill plus the schema head.                 */
/* Replaces Backbone::{load, forward, prefill} (qwen.rs:193-426).            */
/* ------------------------------------------------------------------------ */
typedef struct clef_engine clef_engine;
typedef struct clef_prefix clef_prefix;

/* Creates an engine on CUDA device `device` for the given geometry. */
int clef_engine_create(const clef_config* cfg, int32_t device, clef_engine** out);

/* Loads one tensor by its checkpoint name (the Qwen3.5 names the reference's
 * Weights::take uses, e.g. "model.language_model.layers.0.linear_attn.in_proj_qkv.weight";
 * the schema head is "clef.head.weight" [head_outputs, hidden]). Host F32
 * data; projections and embeddings are stored as BF16 on the device, norms,
 * convolution, gates and the head as F32. `count` must match the shape. */
int clef_engine_set_weight(clef_engine* e, const char* name, const float* host, size_t count);

/* Fills every tensor not yet loaded with seeded synthetic values generated on
 * the device (normal(0, std) for matrices and norm offsets, A_log ~ U(0, ln 16),
 * dt_bias ~ N(0, 0.1)). Deterministic in (seed, tensor name, element). */
int clef_engine_init_random(clef_engine* e, uint64_t seed, float std);

/* Copies a loaded tensor back to host F32 (BF16 values widened exactly). */
int clef_engine_get_weight(clef_engine* e, const char* name, float* host, size_t count);

/* Number of elements of a named tensor (0 if the name is unknown). */
size_t clef_engine_weight_count(const clef_engine* e, const char* name);

/* Checks that every tensor is present and builds the fused device layouts. */
int clef_engine_finalize(clef_engine* e);

/* Prefill of `nseq` independent sequences packed back to back.
 * ids: host int32 [offsets[nseq]]; offsets: host int64 [nseq + 1].
 * initial: prefix state every sequence continues from (NULL = none); the
 *   positions of each sequence then start at the prefix length.
 * capture: 0 = none; otherwise nseq must be 1 and the state at token
 *   `capture` (1 <= capture <= T) is returned in *captured.
 * logits: host F32 [nseq, head_outputs] read at each sequence's last token
 *   (may be NULL). hidden: host F32 [total_tokens, hidden] final-normed
 *   hidden states (may be NULL). */
int clef_engine_prefill(clef_engine* e, const int32_t* ids, const int64_t* offsets,
                        int32_t nseq, const clef_prefix* initial, int64_t capture,
                        clef_prefix** captured, float* logits, float* hidden);

/* Stream-ordered prefill with device-resident ids (int32, packed as in
 * clef_engine_prefill) and device logits [nseq, head_outputs]; `offsets` is a
 * host array. Issues the work on `stream` (NULL = the engine's stream) and
 * returns without synchronising: the caller reads the logits after its own
 * stream synchronisation. Same computation as clef_engine_prefill. */
int clef_engine_prefill_device(clef_engine* e, const int32_t* ids_device, const int64_t* offsets,
                               int32_t nseq, const clef_prefix* initial, float* logits_device,
                               void* stream);

/* Arithmetic of the projection GEMMs (no counterpart in the reference, whose
 * device profiles pick one model dtype). CLEF_PRECISION_BF16 (the default):
 * BF16 operands and BF16 in-projection / attention-projection outputs, the
 * fastest path. CLEF_PRECISION_SPLIT: every activation operand of a GEMM is
 * carried as two BF16 halves (hi = bf16(x), lo = bf16(x - hi)) against the
 * same BF16 weights, and the projection outputs are F32, so the projections
 * reproduce F32 arithmetic on the BF16 weights to about 2^-17 relative, at
 * twice the tensor-core work; the attention's q, k, v and probabilities stay
 * BF16. Used to qualify decisions against the reference's F32 CPU path.
 * Takes effect from the next prefill; waits for the engine's pending work. */
typedef enum clef_precision { CLEF_PRECISION_BF16 = 0, CLEF_PRECISION_SPLIT = 1 } clef_precision;
int clef_engine_set_precision(clef_engine* e, int32_t precision);
int32_t clef_engine_precision(const clef_engine* e);

/* Caps the SMs that the engine's persistent kernels (projection GEMMs, scan
 * carry) occupy during its prefills, 0 = all (the default). Lets two engines,
 * or an engine and other work, share one GPU on separate streams with their
 * persistent kernels on disjoint SM sets instead of queueing behind each
 * other. Results do not depend on it (the same tiles and sequences, spread
 * over fewer CTAs). No counterpart in the reference. */
int clef_engine_set_sm_limit(clef_engine* e, int32_t sms);

/* Number of kernels the engine has issued in prefill calls so far. */
int64_t clef_engine_launches(const clef_engine* e);

/* Requests cooperative cancellation; checked between layers
 * (Control::check, crates/core/src/models/mod.rs:44-59). */
int clef_engine_cancel(clef_engine* e, int32_t cancel);

/* Per-stage device milliseconds accumulated (CUDA events) since profiling was
 * last enabled, written into `ms` [n] in the order: embed, norm, gemm,
 * delta_prologue, delta_scan, delta_epilogue, attention_prologue, attention,
 * head. Synchronises the device if stream-ordered prefills are pending.
 * Returns the count written. */
int clef_engine_stage_times(clef_engine* e, float* ms, int32_t n);
int clef_engine_set_profiling(clef_engine* e, int32_t enabled);

int clef_engine_destroy(clef_engine* e);

/* Prefix state: {Linear{recurrent S, conv history}, Full{K, V}} per layer and
 * the captured final-normed hidden rows (PrefixState, qwen.rs:153-190). */
int64_t clef_prefix_tokens(const clef_prefix* p);
uint64_t clef_prefix_bytes(const clef_prefix* p);
int clef_prefix_destroy(clef_prefix* p);

/* Moving a prefix state between devices (no counterpart in the reference,
 * which serves one device; a multi-GPU server computes a shared prefix once
 * and broadcasts it to the other GPUs instead of recomputing it on each).
 * A prefix is one device allocation of clef_prefix_span_bytes bytes whose
 * layout depends only on the engine configuration and the token count; its
 * first 256 bytes are a layout descriptor (layer kinds, widths, token count).
 * clef_prefix_export copies it to `dst` (device memory of the prefix's
 * device, `bytes` = the span), stream-ordered on `stream` (NULL = default
 * stream). clef_prefix_create makes an empty prefix of `tokens` tokens for
 * engine `e`; it cannot be used as an initial state until filled.
 * clef_prefix_import fills it from such a copy (for example after an NCCL
 * broadcast): it copies on `stream`, then waits for that stream and checks
 * the copied descriptor against the prefix's own, returning
 * CLEF_ERR_INVALID (and leaving the prefix unfilled) when the copy was made
 * for another layout or token count. */
uint64_t clef_prefix_span_bytes(const clef_prefix* p);
int clef_prefix_create(clef_engine* e, int64_t tokens, clef_prefix** out);
int clef_prefix_export(const clef_prefix* p, void* dst, uint64_t bytes, void* stream);
int clef_prefix_import(clef_prefix* p, const void* src, uint64_t bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Learned joint schema head (Head, crates/core/src/models/head.rs:26-274):   */
/* span means over the record's instruction and option spans, evidence       */
/* routing, decoder layers and the joint scorer, in F32.                     */
/* ------------------------------------------------------------------------ */
/* HeadConfig (head.rs:26-33). The released head is hidden 2560 or 4096,
 * width 1024, 2 routing layers, 4 decoder layers, 16 heads, feed-forward 4096
 * (HeadConfig::validate, head.rs:34-47); other sizes are accepted for tests. */
typedef struct clef_head_config {
  int32_t hidden_size;
  int32_t width;
  int32_t routing_layers;
  int32_t layers;
  int32_t heads;
  int32_t feedforward;
} clef_head_config;

/* One EncodedQuestion (encoding.rs): type kind 0..2, instruction token span
 * [start, end), and its options as entries [option_offset, option_offset +
 * option_count) of the option-span array (listed in question order). */
typedef struct clef_head_question {
  int32_t kind;
  int32_t instruction_start;
  int32_t instruction_end;
  int32_t option_offset;
  int32_t option_count;
} clef_head_question;

typedef struct clef_head clef_head;

/* Replaces Head::load (head.rs:91-145): create, load every tensor by its
 * checkpoint name (joint_head.safetensors names, e.g. "layers.0.norm1.weight",
 * host F32; scalars prior_logit_scale, joint_logit_scale, residual_gate have
 * count 1), then finalize. Weights stay F32 on the device. */
int clef_head_create(const clef_head_config* cfg, int32_t device, clef_head** out);
int clef_head_set_weight(clef_head* h, const char* name, const float* data, int64_t count);
int clef_head_finalize(clef_head* h);

/* Replaces Head::forward (head.rs:147-274) for one record.
 * hidden: device F32 [T, hidden_size] (the backbone's final hidden rows);
 * output_embeddings: device F32 [vocab, hidden_size]; ids: host int32 [T];
 * questions: host [nq]; option_spans: host int32 [2 * options] as
 * (start, end) pairs; logits: host F32 [options], question by question.
 * Runs on the head's own stream and returns after the logits are on the
 * host; a nonfinite logit is an error, as in the reference (head.rs:265-267).
 * T <= 49152; at most 64 options per question. */
int clef_head_forward(clef_head* h, const float* hidden, int64_t T, const float* output_embeddings,
                      int64_t vocab, const int32_t* ids, const clef_head_question* questions,
                      int32_t nq, const int32_t* option_spans, float* logits);
int clef_head_destroy(clef_head* h);

/* Diagnostic with no counterpart in the reference: runs the bounded-wait
 * failure path of the device kernels on purpose (an mbarrier nothing arrives
 * on, given up after limit_ms in [1, 2000]) and returns the status a stuck
 * wait produces, CLEF_ERR_DEVICE_TIMEOUT, with the context still usable.
 * Any other status means the failure path is broken. */
int clef_selftest_wait_timeout(int32_t limit_ms, void* stream);

/* ------------------------------------------------------------------------ */
/* Decisions from schema-head logits (answers, crates/core/src/types.rs:728-802). */
/* ------------------------------------------------------------------------ */
typedef struct clef_decision {
  float noul;          /* softmax(logits[0:2])[0] = P(true)                  */
  int32_t choice;      /* first strict maximum of softmax(logits[2:6])      */
  float confidence;    /* that maximum probability                          */
  float score;         /* raw score logit (a one-option softmax is 1.0)     */
} clef_decision;

int clef_decide(const float* logits, int32_t n, int32_t head_outputs, clef_decision* out);

#ifdef __cplusplus
}
#endif
#endif /* CLEF_B200_H */
