/*
 * ovf_oracle.h — CPU restatement of Overfit's quantized-projection decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * product (overfit_b200/libovf_cuda.so) and the timed CPU baseline in bench.py.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may load it.
 * Nothing in the product path links or calls it.
 *
 * The reference (DevOnBike/Overfit) is C#/.NET 10 with no native parts, and no
 * .NET SDK exists in this image, so the reference itself cannot be compiled or
 * run here.  Every function below restates one reference routine and cites the
 * C# file:line it follows (paths relative to Sources/Main/LanguageModels/).
 * Parity pinning: the codecs are pinned against the reference's hand-built
 * known-answer tests (Tests/LanguageModels/Loading/GgmlDequantTests.cs) and its
 * property tests (Q4KDotKernelTests.cs, GgmlQuantTests.cs,
 * CachedAttentionKernelTests.cs), restated as fixtures in tests/golden/.
 *
 * Arithmetic contract (what "bit-exact" means here): compiled with
 * -ffp-contract=off and without -ffast-math so every float op is one IEEE
 * binary32 op in the reference's order (RyuJIT does not contract to FMA);
 * MathF.Round == rintf (round half to even); int->float conversions are
 * round-to-nearest-even; fp16<->fp32 via _Float16 (RNE).
 */
#ifndef OVF_ORACLE_H
#define OVF_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (same numbering as GGUF / Loading/GgmlType.cs) */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q6_K = 14 };

#define ORC_QK_K 256
#define ORC_Q4K_BYTES 144
#define ORC_Q6K_BYTES 210
#define ORC_Q8_0_BYTES 34

/* ---------------- block codecs ---------------- */
void orc_unpack_q4k_scales_mins(const uint8_t *packed12, uint8_t *scales8, uint8_t *mins8);
void orc_decode_q4k_block(const uint8_t *block144, float *dst256);
void orc_decode_q6k_block(const uint8_t *block210, float *dst256);
void orc_encode_q4k_block(const float *src256, uint8_t *block144);
void orc_quantize_q4k(const float *w, int64_t rows, int64_t k, uint8_t *out);
void orc_encode_q6k_block(const float *src256, uint8_t *block210);
void orc_quantize_q6k(const float *w, int64_t rows, int64_t k, uint8_t *out);
void orc_quantize_q8_0_gguf(const float *w, int64_t n, uint8_t *out);
void orc_q8_0_deinterleave(const uint8_t *gguf, int64_t n, int8_t *quants, float *scales);
void orc_requant_q8_0(int type, const void *data, int64_t rows, int64_t k, int8_t *q, float *scales);
void orc_dequant_rows(int type, const void *data, const float *q8_scales,
                      int64_t row0, int64_t nrows, int64_t k, float *dst);

/* ---------------- activation quantizers ---------------- */
void orc_quantize_q8k(const float *x, int64_t k, int8_t *q, float *scales, int16_t *bsums);
void orc_quantize_q8_0(const float *x, int64_t k, int8_t *q, float *scales);

/* ---------------- dots ---------------- */
float orc_q4k_dot(const uint8_t *blk, const int8_t *q8, float q8scale, const int16_t *bsums);
float orc_q6k_dot(const uint8_t *blk, const int8_t *q8, float q8scale, const int16_t *bsums);
float orc_q8_0_dot(const int8_t *wq, const float *ws, const int8_t *xq, const float *xs, int64_t len);

/* ---------------- projections (rows split over OpenMP threads) ---------------- */
void orc_kq_project_prequantized(int type, const uint8_t *w, int64_t n, int64_t k,
                                 const float *bias, float *y,
                                 const int8_t *q, const float *s, const int16_t *bsums);
void orc_kq_project(int type, const float *x, const uint8_t *w, int64_t n, int64_t k,
                    const float *bias, float *y, int8_t *q, float *s, int16_t *bsums);
void orc_kq_project_batched(int type, const float *x, int64_t rows, const uint8_t *w,
                            int64_t n, int64_t k, const float *bias, float *y);
void orc_q8_0_project(const float *x, const int8_t *wq, const float *ws, int64_t n, int64_t k,
                      const float *bias, float *y, int8_t *xq, float *xs);
void orc_q8_0_project_batched(const float *x, int64_t rows, const int8_t *wq, const float *ws,
                              int64_t n, int64_t k, const float *bias, float *y);
void orc_f32_project_input_major(const float *x, const float *w, int64_t k, int64_t n, float *y);

/* ---------------- small ops ---------------- */
void orc_rmsnorm(const float *x, const float *gamma, float *y, int64_t d, float eps);
void orc_rope_table(int max_seq, int head_dim, float theta, float *cos_t, float *sin_t);
void orc_rope_apply(float *v, int head_dim, const float *cos_p, const float *sin_p, int split_half);
void orc_attention_single_head(const float *q, const float *keys, const float *values,
                               float *out, float *scratch, int seq_len, int head_dim,
                               float scale);
void orc_silu_inplace(float *v, int64_t n);
int  orc_moe_select_topk(const float *logits, int n, int top_k, int *idx, float *w, int normalize);
int  orc_argmax(const float *v, int64_t n);

/* ---------------- whole-model decode ---------------- */
typedef struct {
    int type;              /* ORC_F32 / ORC_Q8_0 / ORC_Q4_K / ORC_Q6_K */
    const void *data;      /* K-quant: GGUF block bytes; Q8_0: int8 quants; F32: floats */
    const float *scales;   /* Q8_0 only: fp32 per-32 scales (de-interleaved form) */
    int64_t rows, cols;    /* output rows x contraction length */
} orc_weight;

typedef struct {
    const float *attn_norm;
    orc_weight wq, wk, wv, wo;         /* wo must be ORC_Q8_0 (per-head Q8_0, see .c) */
    const float *bq, *bk, *bv, *bo;    /* optional (NULL) */
    const float *ffn_norm;
    orc_weight w_gate, w_up, w_down;   /* dense SwiGLU */
    const float *router;               /* MoE: input-major [d_model x n_experts] F32 */
    const orc_weight *e_gate, *e_up, *e_down;  /* MoE: n_experts each */
} orc_layer;

typedef struct {
    int n_layers, d_model, n_heads, n_kv_heads, head_dim, d_ff, vocab, max_ctx;
    int rope_split_half, n_experts, n_experts_used, normalize_experts;
    float eps, theta;
    orc_weight embed;                  /* Q4_K / Q6_K / F32 rows [vocab x d_model] */
    const orc_layer *layers;
    const float *final_norm;
    orc_weight lm_head;                /* Q4_K / Q6_K / Q8_0 [vocab x d_model] */
} orc_model;

typedef struct orc_session orc_session;
orc_session *orc_session_create(const orc_model *m, int max_ctx);
void orc_session_destroy(orc_session *s);
void orc_session_reset(orc_session *s);
/* Test switch: store K/V rounded to fp16 (the GPU's cache format); the
 * reference's cache is F32 (Runtime/KeyValueCache.cs:593-602). */
void orc_session_set_kv_fp16(orc_session *s, int on);
void orc_session_set_kv_q8(orc_session *s, int on);
float orc_q8kv_quantize(const float *src, int n, int8_t *dst);
void orc_attention_single_head_q8(const float *q, const int8_t *kq, const float *ks, const int8_t *vq,
                                  const float *vs, float *out, float *scratch, int seq_len, int hd, float scale);
/* Test switch: exp rounded once from double precision (as on the GPU). */
int orc_session_fill_context(orc_session *s, int n, uint64_t seed);
void orc_expf_array(const float *x, float *y, int64_t n);
int  orc_session_position(const orc_session *s);
/* One token through the stack; writes logits[vocab] when logits != NULL. */
int  orc_session_decode(orc_session *s, int token, float *logits);
/* Decode a run of layers only (bounded CPU-baseline samples): returns hidden. */
int  orc_session_decode_layers(orc_session *s, int token, int n_layers_to_run, int with_logits,
                               float *logits);
int  orc_num_threads(void);
void orc_set_num_threads(int n);

/* deterministic synthetic data (splitmix64 + Box-Muller), for CPU-side samples */
void orc_fill_normal(float *dst, int64_t n, uint64_t seed, float mean, float stddev);

#ifdef __cplusplus
}
#endif
#endif
