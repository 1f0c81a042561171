/*
 * ovf.h — C ABI of libovf_cuda.so, the B200 (sm_100a) implementation of
 * Overfit's quantized-projection inference path.
 *
 * Boundary rules
 *  - C linkage, plain pointers and sizes, no C++ or torch types.
 *  - Every entry point returns ovf_status (0 = OVF_OK, negative = error) and
 *    never throws or aborts; ovf_last_error() gives a message for the calling
 *    host thread.  Argument checks happen on the host before any launch.
 *  - Kernel-level entry points take DEVICE pointers and a cudaStream_t passed
 *    as void* (NULL = the legacy default stream); they are stream-ordered and
 *    do not synchronize.  As in the reference, the caller owns every buffer
 *    including the activation-quantization scratch; nothing allocates per call.
 *  - Session-level entry points take HOST pointers and return after the token
 *    is on the host, like the reference's synchronous session API.
 *
 * Each declaration cites the reference routine it replaces (paths relative to
 * Sources/Main/LanguageModels/ of DevOnBike/Overfit).  Weight bytes are the
 * verbatim GGUF blocks: Q4_K 144 B / 256 weights, Q6_K 210 B / 256 weights,
 * stored output-major (row o = the K-long contraction vector of output o).
 * Q8_0 weights are held de-interleaved like the reference's Q8Weight
 * (Runtime/Q8Weight.cs:21-60): int8 quants [n x k] plus fp32 scales
 * [n x k/32]; ovf_q8_0_deinterleave converts GGUF Q8_0 blocks to that form.
 */
#ifndef OVF_H
#define OVF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t ovf_status;
#define OVF_OK 0
#define OVF_EINVAL (-1)       /* bad argument (shape, alignment, null) — ArgumentException */
#define OVF_ENOMEM (-2)       /* device allocation failed */
#define OVF_ECUDA (-3)        /* CUDA runtime / launch error */
#define OVF_ENCCL (-4)        /* NCCL error */
#define OVF_ETIMEDOUT (-5)    /* a bounded device wait gave up (error word set by a kernel) */
#define OVF_ESTATE (-6)       /* invalid state, e.g. KV cache full — OverfitRuntimeException */
#define OVF_EUNSUPPORTED (-7) /* format/shape combination not supported */
#define OVF_EBUSY (-8)        /* the object is in use by another call */

/* ggml type ids (GGUF numbering, Loading/GgmlType.cs). */
#define OVF_TYPE_F32 0
#define OVF_TYPE_F16 1
#define OVF_TYPE_Q8_0 8
#define OVF_TYPE_Q4_K 12
#define OVF_TYPE_Q6_K 14

/* ---------------------------------------------------------------- misc */
const char *ovf_last_error(void);
int32_t ovf_version(void);
/* Reads and clears the device-side error word that bounded waits set. */
ovf_status ovf_device_error(int32_t device, int32_t *code_out);

/* ---------------------------------------------------- activation quantizers */
/* Runtime/Q4KDotKernel.cs:71 QuantizeActivationQ8K: per 256 elements an fp32
 * scale absmax/127, int8 quants round-half-even(x * 1/scale) clamped to
 * +-127 and 16 int16 group sums.  k % 256 == 0. */
ovf_status ovf_quantize_q8k(const float *x, int64_t k, int8_t *q, float *scales, int16_t *bsums,
                            void *stream);
/* Runtime/Q8DotKernel.cs:42 Quantize: per 32 elements an fp32 scale. k % 32 == 0. */
ovf_status ovf_quantize_q8_0(const float *x, int64_t k, int8_t *q, float *scales, void *stream);

/* ----------------------------------------------------------- projections */
/* Runtime/Q4KDotKernel.cs:485 ProjectParallel (and Q6KDotKernel.cs:314 for
 * type OVF_TYPE_Q6_K): y[o] = bias[o] + sum over super-blocks of the
 * Q4_K x Q8_K dot, accumulated in ascending super-block order.  x [k] is
 * quantized once into the caller's scratch (act_q [k], act_scales [k/256],
 * act_bsums [k/16]), exactly as the reference fills its scratch spans.
 * bias may be NULL.  k % 256 == 0; w 16-byte aligned. */
ovf_status ovf_kq_project(int32_t type, const float *x, const void *w, int64_t n, int64_t k,
                          const float *bias, float *y, int8_t *act_q, float *act_scales,
                          int16_t *act_bsums, void *stream);
/* Runtime/Q4KDotKernel.cs:445 ProjectPreQuantized (Q6KDotKernel.cs:274). */
ovf_status ovf_kq_project_prequantized(int32_t type, const void *w, int64_t n, int64_t k,
                                       const float *bias, float *y, const int8_t *act_q,
                                       const float *act_scales, const int16_t *act_bsums,
                                       void *stream);
/* Runtime/Q4KDotKernel.cs:563 ProjectGateUpParallel: both Q4_K halves from
 * one Q8_K quantize in one launch (no bias). */
ovf_status ovf_q4k_project_gate_up(const float *x, const void *gate_w, const void *up_w, int64_t n,
                                   int64_t k, float *gate_y, float *up_y, int8_t *act_q,
                                   float *act_scales, int16_t *act_bsums, void *stream);
/* Runtime/Q4KDotKernel.cs:663 ProjectBatched / :819 ProjectBatchedWeightStationary
 * (Q6KDotKernel.cs:403 ProjectBatched): rows x k activations, y [rows x n],
 * every row bit-identical to ovf_kq_project.  Scratch: act_q [rows*k],
 * act_scales [rows*k/256], act_bsums [rows*k/16]. */
ovf_status ovf_kq_project_batched(int32_t type, const float *x, int64_t rows, const void *w, int64_t n,
                                  int64_t k, const float *bias, float *y, int8_t *act_q,
                                  float *act_scales, int16_t *act_bsums, void *stream);
/* Runtime/Q4KDotKernel.cs:819 ProjectBatchedWeightStationary on the tensor
 * cores (tcgen05.mma, fp32 accumulators in TMEM): the same outputs as
 * ovf_kq_project_batched, bit for bit (the integer parts of every
 * super-block dot are exact in the fp32 accumulators; the reference's fp32
 * tail runs in the epilogue).  Q4_K weights, or Q6_K (Q6KDotKernel.cs:403
 * ProjectBatched) with k a multiple of 2048.  Scratch: the activation
 * quantization as for ovf_kq_project_batched plus `scratch` of
 * ovf_tc_scratch_bytes(rows, k) bytes (16-byte aligned) for the packed
 * operand tiles. */
int64_t ovf_tc_scratch_bytes(int64_t rows, int64_t k);
ovf_status ovf_kq_project_batched_tc(int32_t type, const float *x, int64_t rows, const void *w, int64_t n,
                                     int64_t k, const float *bias, float *y, int8_t *act_q, float *act_scales,
                                     int16_t *act_bsums, void *scratch, void *stream);
/* Runtime/Q8DotKernel.cs:352 ProjectBatched on the tensor cores (tcgen05.mma
 * kind::i8: every 32-element block dot is an exact int32 in TMEM, the
 * reference's fp32 tail runs in the epilogue): the same outputs as
 * ovf_q8_0_project_batched, bit for bit.  k a multiple of 64.  Scratch:
 * x_q [rows*k], x_scales [rows*k/32] as for ovf_q8_0_project_batched plus
 * `scratch` of ovf_tc_scratch_bytes(rows, k) bytes (16-byte aligned), which
 * also covers ovf_kq_project_batched_tc when k is a multiple of 256. */
ovf_status ovf_q8_0_project_batched_tc(const float *x, int64_t rows, const int8_t *wq, const float *wscales,
                                       int64_t n, int64_t k, const float *bias, float *y, int8_t *x_q,
                                       float *x_scales, void *scratch, void *stream);
/* Runtime/Q8DotKernel.cs:252 ProjectParallel over a de-interleaved Q8Weight:
 * y[o] = bias[o] + sum_b (wscale*xscale)*int8dot, ascending b.  Scratch
 * x_q [k], x_scales [k/32].  k % 32 == 0. */
ovf_status ovf_q8_0_project(const float *x, const int8_t *wq, const float *wscales, int64_t n,
                            int64_t k, const float *bias, float *y, int8_t *x_q, float *x_scales,
                            void *stream);
/* Runtime/Q8DotKernel.cs:352 ProjectBatched. */
ovf_status ovf_q8_0_project_batched(const float *x, int64_t rows, const int8_t *wq,
                                    const float *wscales, int64_t n, int64_t k, const float *bias,
                                    float *y, int8_t *x_q, float *x_scales, void *stream);

/* ---------------------------------------------------------- weight codecs */
/* Loading/GgmlQuant.cs:141 QuantizeQ4_K: fp32 [rows x k] -> Q4_K bytes. */
ovf_status ovf_quantize_q4k(const float *w, int64_t rows, int64_t k, void *out, void *stream);
/* Q6_K encoder for the decoder at Loading/GgmlDequant.cs:159 (the reference
 * has no Q6_K encoder): per 16 weights an int8 scale, per 256 an fp16 d,
 * 6-bit values q - 32 from a symmetric absmax fit. */
ovf_status ovf_quantize_q6k(const float *w, int64_t rows, int64_t k, void *out, void *stream);
/* GGUF Q8_0 encoder (fp16 scale + 32 int8) using Runtime/Q8DotKernel.cs:42 quants. */
ovf_status ovf_quantize_q8_0_gguf(const float *w, int64_t n, void *out, void *stream);
/* Loading/GgufReader.cs:198 LoadTensorQ8_0Raw: GGUF Q8_0 -> int8 + fp32 scales. */
ovf_status ovf_q8_0_deinterleave(const void *gguf, int64_t n, int8_t *q, float *scales,
                                 void *stream);
/* Runtime/Q4KWeight.cs:122 DecodeRow (and the Q6_K / Q8_0 / F32 analogues):
 * rows [row0, row0+nrows) of a [* x k] weight decoded to fp32. */
ovf_status ovf_dequant_rows(int32_t type, const void *w, const float *q8_scales, int64_t row0,
                            int64_t nrows, int64_t k, float *dst, void *stream);
/* Loading/GgufLlamaLoader.cs:977-995 + :1298-1336 (LoadOutputHeads ->
 * SplitOutput -> Q8Weight.QuantizeRows): a K-quant attn_output weight is
 * decoded to fp32 and re-quantized to Q8_0 with fp32 scales. */
ovf_status ovf_requant_q8_0(int32_t src_type, const void *w, int64_t rows, int64_t k, int8_t *q,
                            float *scales, void *stream);

/* ---------------------------------------------------------------- ops */
/* Runtime/CachedTransformerBlock.cs:525 RmsNormalize: y = (x*s)*gamma,
 * s = 1/sqrt(sum(x^2)/d + eps). gamma may be NULL. */
ovf_status ovf_rmsnorm(const float *x, const float *gamma, float *y, int64_t d, float eps,
                       void *stream);
/* MathF.Exp elementwise (the softmax and SiLU exponential of
 * Runtime/CachedAttentionKernel.cs:36 and Runtime/CachedFeedForwardBlock.cs:464):
 * the bits of the host C library's expf on an x86-64 host with FMA (glibc's
 * ARM optimized-routines expf), which is what MathF.Exp calls on Linux. */
ovf_status ovf_exp_f32(const float *x, float *y, int64_t n, void *stream);
/* Runtime/CachedFeedForwardBlock.cs:464-472 ApplySiLU then :309 Multiply:
 * h = (g * sigmoid(g)) * u with sigmoid(g) = 1 / (1 + exp(-g)). */
ovf_status ovf_swiglu(const float *gate, const float *up, float *h, int64_t n, void *stream);
/* Rope/RopeKernel.cs:46 Apply over n_vec vectors of head_dim, rotated at
 * the given cos/sin row (Rope/RopeTable.cs:109 layout [hd/2]). */
ovf_status ovf_rope_apply(float *v, int32_t n_vec, int32_t head_dim, const float *cos_row,
                          const float *sin_row, int32_t split_half, void *stream);
/* Runtime/CachedAttentionKernel.cs:36 ComputeSingleHead for every query head
 * (GQA: head h reads KV head h/(n_heads/n_kv_heads), CachedMultiHeadAttention.cs:897)
 * over fp16 caches (no reference counterpart), split along the sequence
 * (flash-decode) and merged with log-sum-exp: within tolerance of the
 * reference, not bit-identical.
 * q [n_heads x hd] fp32; k_cache/v_cache fp16 [n_kv_heads x max_ctx x hd];
 * positions [0, seq_len) are attended.  scratch must hold
 * ovf_attention_scratch_bytes(n_heads, n_kv_heads, hd) bytes and
 * counters n_kv_heads int32 zeros (they are left zero on return). */
int64_t ovf_attention_scratch_bytes(int32_t n_heads, int32_t n_kv_heads, int32_t head_dim);
/* Runtime/CachedAttentionKernel.cs:36 ComputeSingleHead for every query head
 * over F32 caches k_cache/v_cache [n_kv_heads x max_ctx x hd], positions
 * [0, seq_len): the reference's operation order, bit-identical results.
 * head_dim 32, 64, 128 or 256.  No scratch. */
ovf_status ovf_attention_single_head(const float *q, const float *k_cache, const float *v_cache, float *out,
                                     int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t max_ctx,
                                     int32_t seq_len, float scale, void *stream);
/* Runtime/CachedAttentionKernel.cs:36 ComputeSingleHead over fp16 caches
 * [n_kv_heads x max_ctx x hd] (IEEE binary16, no reference counterpart: the
 * F32 cache's values rounded to fp16): every value widens exactly to fp32 and
 * the arithmetic is ComputeSingleHead's, bit for bit. */
ovf_status ovf_attention_single_head_f16(const float *q, const void *k_cache, const void *v_cache, float *out,
                                         int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t max_ctx,
                                         int32_t seq_len, float scale, void *stream);
/* Runtime/CachedAttentionKernel.cs:139 ComputeSingleHeadQ8 for every query
 * head over a Q8 cache (Q8KvQuant per-vector int8 [n_kv_heads x max_ctx x hd]
 * + fp32 scales [n_kv_heads x max_ctx]), positions [0, seq_len): the
 * reference's operation order. */
ovf_status ovf_attention_single_head_q8(const float *q, const int8_t *k_cache, const float *k_scales,
                                        const int8_t *v_cache, const float *v_scales, float *out, int32_t n_heads,
                                        int32_t n_kv_heads, int32_t head_dim, int32_t max_ctx, int32_t seq_len,
                                        float scale, void *stream);
ovf_status ovf_attention_decode(const float *q, const void *k_cache, const void *v_cache, float *out,
                                int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                int32_t max_ctx, int32_t seq_len, float scale, void *scratch,
                                int32_t *counters, void *stream);

/* No counterpart in the reference (its attention allocates nothing on the
 * GPU because it has no GPU path).  Same computation as ovf_attention_decode
 * for callers that cannot call cudaMalloc (a host whose device memory is
 * owned by one sanctioned allocator, or an allocation-free hot path): the
 * scratch lives in a file-scope device array of 1 MiB (plus 1 KiB of
 * counters) that every GPU loading the library holds until exit.  Layouts
 * whose ovf_attention_scratch_bytes exceed 1 MiB, or with more than 256 KV
 * heads, return OVF_EINVAL.  The first call on each device looks up the
 * array's address (make it before any stream capture).  All calls on a
 * device share the array: calls that overlap on the GPU race. */
ovf_status ovf_attention_decode_noalloc(const float *q, const void *k_cache, const void *v_cache, float *out,
                                        int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t max_ctx,
                                        int32_t seq_len, float scale, void *stream);

/* ------------------------------------------------------------- sessions */
typedef struct ovf_model ovf_model;
typedef struct ovf_session ovf_session;

/* One weight as the GGUF loader hands it over: host pointer to the verbatim
 * tensor bytes (K-quant / Q8_0 GGUF blocks, or fp32), rows x cols with cols
 * the contraction length.  F32 vectors (norms, biases) use rows = 1. */
typedef struct {
    int32_t type;
    const void *data;
    int64_t rows, cols;
} ovf_tensor;

/* Config as GgufLlamaLoader.cs:93-229 reads it from GGUF metadata.  eps is
 * taken as given: the reference uses 1e-6 for every GGUF model
 * (Runtime/CachedLlamaInferenceEngine.cs:139). */
typedef struct {
    int32_t n_layers, d_model, n_heads, n_kv_heads, head_dim, d_ff, vocab;
    int32_t rope_split_half;   /* 1 for qwen2-style split-half, 0 for llama adjacent pairs */
    int32_t n_experts, n_experts_used, normalize_experts;
    float eps, rope_theta;
} ovf_model_config;

/* Tensor table order, per layer (stride OVF_TENSORS_PER_LAYER):
 *   attn_norm, wq, wk, wv, wo, bq, bk, bv, bo, ffn_norm, w_gate, w_up, w_down,
 *   router (MoE, input-major F32 [d_model x n_experts])
 * then (after all layers): token_embd, output_norm, output (lm head; may be
 * type -1 for tied embeddings).  Absent optional tensors have data == NULL.
 * MoE experts: w_gate/w_up/w_down hold n_experts matrices back to back.
 * The loader follows the reference's residency choices: K-quant and Q8_0
 * Q/K/V/FFN/lm-head stay in their format; a K-quant attn_output is
 * re-quantized to Q8_0 with fp32 scales; embeddings stay K-quant or become
 * fp32 (GgufLlamaLoader.cs:546-572). */
#define OVF_TENSORS_PER_LAYER 14
ovf_status ovf_model_create(int32_t device, const ovf_model_config *cfg, const ovf_tensor *tensors,
                            int32_t n_tensors, ovf_model **out);
ovf_status ovf_model_destroy(ovf_model *m);

/* Tensor parallelism over `world` GPUs (one process per GPU), the north
 * star's split of Llama-family models: rank r holds query heads
 * [r*H/world, (r+1)*H/world) with their KV heads (Q/K/V rows, attn_output
 * columns, its share of the KV cache), FFN rows [r*F/world, ...) of gate/up
 * and the same columns of down, and vocabulary rows of the LM head; the
 * embedding and norms are replicated.  Every rank passes the FULL tensor
 * table; the library uploads only its shard (shard-aware upload of the
 * loader's slices, GgufLlamaLoader.cs:45-531).  The per-head outputs
 * (CachedMultiHeadAttention.cs:221-298), the down projection's super-block
 * terms and the logits are exchanged over NVLink through peer memory, and
 * every rank adds them in the reference's order, so the results are
 * bit-identical to one GPU.  Requires n_kv_heads, d_ff/256 and vocab
 * divisible by world (world <= 8); no MoE.  After creation, exchange the
 * ranks' OVF_TP_HANDLE_BYTES handles (ovf_model_tp_export) between the
 * processes and call ovf_model_tp_connect with all of them in rank order.
 * Sessions then run in lockstep: every rank makes the same calls in the
 * same order (a rank that stops makes the others' next step fail with
 * OVF_ETIMEDOUT after about a second).  Prompts take the single-token loop;
 * batch decode and speculative verify return OVF_EUNSUPPORTED. */
#define OVF_TP_HANDLE_BYTES 64
ovf_status ovf_model_create_tp(int32_t device, const ovf_model_config *cfg, const ovf_tensor *tensors,
                               int32_t n_tensors, int32_t rank, int32_t world, ovf_model **out);
ovf_status ovf_model_tp_export(ovf_model *m, void *handle_out);
ovf_status ovf_model_tp_connect(ovf_model *m, const void *handles);
/* Device bytes of resident weights (for bandwidth accounting). */
int64_t ovf_model_weight_bytes(const ovf_model *m);

/* KV-cache element types (Runtime/KvCacheDType.cs:15).  OVF_KV_F32 is the
 * reference's default: attention then runs in the reference's exact
 * operation order (CachedAttentionKernel.ComputeSingleHead).  OVF_KV_Q8 is
 * the reference's Q8 cache (per-vector int8 + fp32 scale, Q8KvQuant), attended
 * in ComputeSingleHeadQ8's exact order.  OVF_KV_F16 has
 * no reference counterpart: half the KV traffic, flash-decode attention with
 * a log-sum-exp merge, results within tolerance of the F32 path only. */
#define OVF_KV_F32 0
#define OVF_KV_Q8 1
#define OVF_KV_F16 2

/* ISlmInferenceEngine.CreateSession (Contracts/ISlmInferenceEngine.cs:9):
 * F32 KV cache. */
ovf_status ovf_session_create(ovf_model *m, int32_t max_ctx, ovf_session **out);
/* CachedLlamaInferenceEngine.CreateSession(maxContextLength, kvCacheDType)
 * (Runtime/CachedLlamaInferenceEngine.cs:360). */
ovf_status ovf_session_create_kv(ovf_model *m, int32_t max_ctx, int32_t kv_dtype, ovf_session **out);
ovf_status ovf_session_destroy(ovf_session *s);
/* ISlmSession.Reset (Contracts/ISlmSession.cs:8). */
ovf_status ovf_session_reset(ovf_session *s);
int32_t ovf_session_position(const ovf_session *s);
/* CachedLlamaSession.DecodeToken (Runtime/CachedLlamaSession.cs:773): one
 * token through the stack; logits_host (vocab floats) may be NULL;
 * argmax_out (first index of the max, TokenSampler.ArgMax) may be NULL. */
ovf_status ovf_session_decode(ovf_session *s, int32_t token, float *logits_host, int32_t *argmax_out);
/* CachedLlamaSession.Prefill (Runtime/CachedLlamaSession.cs:167): logits
 * of the last token only.  Like the reference, n >= 16 tokens take the
 * batched path (PrefillBatchedQuant, :818-835), which leaves the session in
 * the state the single-token loop would, bit for bit. */
ovf_status ovf_session_prefill(ovf_session *s, const int32_t *tokens, int32_t n, float *logits_host,
                               int32_t *argmax_out);
/* Greedy generation (GenerateNextToken with temperature 0, repeated): feeds
 * argmax back on the device, n_steps tokens, returns them in tokens_out.
 * Requires a prior prefill/decode (the reference throws on an empty session). */
ovf_status ovf_session_generate_greedy(ovf_session *s, int32_t n_steps, int32_t *tokens_out);
/* The cudaStream_t (as void*) all of the session's device work is ordered
 * on, for callers that time it with events. */
void *ovf_session_stream(const ovf_session *s);
/* One DecodeToken in each of n (<= 64) distinct sessions of one model, run
 * as one batch: every weight tile is read once for all n tokens, and each
 * session ends in the state its own ovf_session_decode would leave (same
 * logits and argmax, bit for bit).  logits_host: [n x vocab] or NULL;
 * argmax_out: [n] or NULL.  The reference serves concurrent sessions one
 * DecodeToken call at a time (a session per client from
 * ISlmInferenceEngine.CreateSession, Contracts/ISlmInferenceEngine.cs:9-52).
 * One batch call per model at a time: a second concurrent call returns
 * OVF_EBUSY.  If a call fails after enqueuing work, its sessions return
 * OVF_ESTATE until ovf_session_reset. */
ovf_status ovf_session_decode_batch(ovf_session *const *sessions, int32_t n, const int32_t *tokens,
                                    float *logits_host, int32_t *argmax_out);

/* Session options.  OVF_OPT_PREFILL_SINGLE (value 0/1):
 * CachedLlamaSession.DisableBatchedPrefillForParity (:808) — prompts take
 * the single-token loop instead of the batched prefill (same results, bit
 * for bit; for parity checks). */
#define OVF_OPT_PREFILL_SINGLE 1
ovf_status ovf_session_set_option(ovf_session *s, int32_t option, int32_t value);

/* CachedLlamaSession.GenerateSpeculative's verify forward
 * (Runtime/CachedLlamaSession.cs:468-477, PrefillBatchedQuantAllRows +
 * ProjectLogitsBatched): n (1..64) tokens appended at positions pos.. in one
 * batched forward, every row projected to logits with one read of the LM
 * head.  Row j's logits are those a single-token decode of tokens[0..j]
 * would give, bit for bit; the last row's become the session's logits.
 * logits_host: [n x vocab] or NULL; argmax_out: [n] (first index of the
 * max, the greedy acceptance test) or NULL. */
ovf_status ovf_session_verify(ovf_session *s, const int32_t *tokens, int32_t n, float *logits_host,
                              int32_t *argmax_out);
/* KeyValueCache.TruncateTo (Runtime/KeyValueCache.cs:246) as
 * CachedLlamaSession.RollbackTo (:318) uses it: the position becomes length
 * (0 <= length <= position); rejected draft rows are dropped. */
ovf_status ovf_session_truncate(ovf_session *s, int32_t length);
/* Bytes of one side (keys or values) of a prefix snapshot at the current
 * position: n_layers * n_kv_heads * position * head_dim * element size. */
int64_t ovf_session_prefix_bytes(const ovf_session *s);
/* CachedLlamaSession.SavePrefix (:231) -> KeyValueCache.Snapshot
 * (Runtime/KeyValueCache.cs:264): the live rows packed
 * [layer][kv_head][position][head_dim] into host buffers of
 * ovf_session_prefix_bytes each, in the cache's element type (F32; fp16 for
 * an fp16 cache).  A Q8 cache returns OVF_EUNSUPPORTED, as the reference's
 * ThrowIfQuantized does. */
ovf_status ovf_session_save_prefix(const ovf_session *s, void *keys, void *values, int32_t *length_out);
/* CachedLlamaSession.RestorePrefix (:242) -> KeyValueCache.RestoreFrom
 * (Runtime/KeyValueCache.cs:296): the packed rows of a snapshot from a
 * session of the same model and cache type; the position becomes length and
 * the session holds no logits until the next prefill or decode. */
ovf_status ovf_session_restore_prefix(ovf_session *s, const void *keys, const void *values, int32_t length);

#ifdef __cplusplus
}
#endif
#endif
