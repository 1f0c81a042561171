// ovf_internal.cuh — launchers and device helpers shared between the
// translation units of libovf_cuda.so (not part of the public C ABI).
#pragma once

#include "ovf_common.cuh"
#include "ovf_gemv.cuh"

namespace ovf {

// ---- element decoders (shared by the codecs and the embedding lookup)
// Value of element e (0..255) of a Q4_K block, exactly as
// Loading/GgmlDequant.cs:95-141 computes it: (d*sc)*nib - dmin*m.
__device__ __forceinline__ float q4k_elem(const uint8_t *b, int e) {
    const float d = h2f_bits((uint16_t)(b[0] | (b[1] << 8)));
    const float dmin = h2f_bits((uint16_t)(b[2] | (b[3] << 8)));
    const int j = e / 32;  // sub-block
    const uint8_t *q = b + 4;
    int sc, m;
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
    const int p = j >> 1, i = e & 31;
    const uint8_t byte = b[16 + 32 * p + i];
    const int nib = (j & 1) ? (byte >> 4) : (byte & 0x0F);
    return fsub(fmul(fmul(d, (float)sc), (float)nib), fmul(dmin, (float)m));
}

// Loading/GgmlDequant.cs:159-209: (d*sc)*(q-32).
__device__ __forceinline__ float q6k_elem(const uint8_t *b, int e) {
    const float d = h2f_bits((uint16_t)(b[208] | (b[209] << 8)));
    const int h = e / 128, r = e % 128, k = r / 32, l = r % 32;
    const uint8_t qlb = b[64 * h + l + ((k & 1) ? 32 : 0)];
    const int low = (k >= 2) ? (qlb >> 4) : (qlb & 0x0F);
    const int hi = (b[128 + 32 * h + l] >> (2 * k)) & 3;
    const int q = low | (hi << 4);
    const int sc = (int)(int8_t)b[192 + 8 * h + l / 16 + 2 * k];
    return fmul(fmul(d, (float)sc), (float)(q - 32));
}

// ---- ovf_quant.cu
ovf_status launch_quantize_q8k(const float *x, int64_t k, int8_t *q, float *s, int16_t *b, cudaStream_t st);
ovf_status launch_quantize_q8_0(const float *x, int64_t k, int8_t *q, float *s, cudaStream_t st);
ovf_status launch_encode(int type, const float *w, int64_t rows, int64_t k, void *out, cudaStream_t st);
ovf_status launch_q8_0_deinterleave(const void *g, int64_t n, int8_t *q, float *s, cudaStream_t st);
ovf_status launch_dequant_rows(int type, const void *w, const float *q8s, int64_t row0, int64_t nrows, int64_t k,
                               float *dst, cudaStream_t st);
ovf_status launch_requant_q8_0(int type, const void *w, int64_t rows, int64_t k, int8_t *q, float *s,
                               cudaStream_t st);

// ---- ovf_batched.cu: weight-stationary projection of `rows` pre-quantized
// activation rows (Q8_K for K-quants, Q8_0 for Q8_0 weights).  `group` > 0
// (Q8_0 only): head-ordered sums of `group` blocks; `resid` [rows x n]:
// added after the bias.
ovf_status launch_batched_project(int type, const void *w, const float *ws, size_t w_bytes, const float *bias,
                                  const int8_t *aq, const float *as, const int16_t *ab, float *y, int64_t n,
                                  int64_t k, int64_t rows, cudaStream_t st, int group = 0,
                                  const float *resid = nullptr);

// ---- ovf_ops.cu
struct AttnParams {
    const float *q;           // [H*hd] query (raw when rope tables are given)
    const float *k_new;       // [KVH*hd] key of the current token (raw), or null
    const float *v_new;       // [KVH*hd] value of the current token, or null
    __half *kc, *vc;          // this layer's cache [KVH][max_ctx][hd] (fp16 kernels; the
                              // exact kernel reads these pointers as fp32 or int8)
    float *ks, *vs;           // Q8 cache: per-vector scales [KVH][max_ctx]
    float *out;               // [H*hd]
    const float *rope_cos;    // [max_ctx][hd/2] or null
    const float *rope_sin;
    const int *pos_dev;       // position of the current token on the device, or null
    float *partial;           // [H][n_splits][hd+2]
    int *counters;            // [KVH], zero on entry and on exit
    int split_half, H, KVH, hd, max_ctx, seq_len_host, n_splits, chunk_max, sc_floats;
    float scale;
    L2Prefetch pf;            // weights of later launches to pull into L2 during the chains
    TraceSlot *trace;         // OVF_TRACE timeline slot, or null
    int no_kv_prefetch;       // skip the early L2 prefetch of the cache rows
    int rows;                 // query rows in one launch (batched prefill; 0 or 1 = one): row r is at
                              // position seq_len_host - 1 + r, its q/out at r * H * hd; k_new must be
                              // null (the rows' keys and values are appended beforehand)
};
int attn_splits(int n_kv_heads);
int64_t attn_scratch_bytes(int H, int KVH, int hd);
ovf_status launch_attention(const AttnParams &p, cudaStream_t st, bool pdl);
// ovf_attn_cluster.cu: cluster-merged variant used by the decode session.
bool attn_cluster_supported(int G, int hd);
ovf_status launch_attention_cluster(const AttnParams &p, cudaStream_t st, bool pdl);
// ovf_attn_group.cu: F32 / fp16 caches, one cluster per KV head (exact order).
bool attn_group_supported(int H, int KVH, int hd, int kv_dtype, int seq_cap, int smem_optin_bytes);
ovf_status launch_attention_group(const AttnParams &p, int seq_cap, cudaStream_t st, bool pdl, int kv_dtype);
// ovf_tc.cu: Q4_K prefill projection on tcgen05 tensor cores (bit-identical).
int64_t tc_scratch_bytes(int64_t rows, int64_t k);
bool tc_project_supported(int type, int64_t n, int64_t k, int64_t rows);
// ovf_tc6.cu: the Q6_K projection of M rows on tcgen05 (k a multiple of 2048).
bool tc6_project_supported(int64_t n, int64_t k, int64_t rows);
ovf_status launch_tc6_project(const void *w, const float *bias, const int8_t *aq, const float *as, const int16_t *ab,
                              float *y, int64_t n, int64_t k, int64_t rows, void *scratch, cudaStream_t st,
                              const float *resid = nullptr);
// ovf_tc8.cu: the Q8_0 projection of M rows on tcgen05 (kind::i8).
bool tc8_project_supported(int64_t n, int64_t k, int64_t rows, int group);
int64_t tc8_scratch_bytes(int64_t rows, int64_t k);
ovf_status launch_tc8_project(const int8_t *wq, const float *ws, const float *bias, const int8_t *aq,
                              const float *as, float *y, int64_t n, int64_t k, int64_t rows, int group,
                              void *scratch, cudaStream_t st, const float *resid = nullptr);
ovf_status launch_tc_project(int type, const void *w, const float *bias, const int8_t *aq, const float *as,
                             const int16_t *ab, float *y, int64_t n, int64_t k, int64_t rows, void *scratch,
                             cudaStream_t st, const float *resid = nullptr);
// ovf_attn_rows.cu: a prefill chunk's causal attention, one thread per chain.
bool attn_rows_supported(int hd, int kv_dtype);
int64_t attn_rows_scratch_floats(int rows, int H, int max_ctx);
ovf_status launch_attention_rows(const AttnParams &p, int pos0, float *P, cudaStream_t st, int kv_dtype);
// ovf_attn_exact.cu: F32 / Q8 / fp16 caches in the reference's operation order (bit-exact on the cached values).
bool attn_exact_supported(int hd);
int attn_exact_max_seq(int hd);
ovf_status launch_attention_exact(const AttnParams &p, int seq_len_max, cudaStream_t st, bool pdl,
                                  int kv_dtype = OVF_KV_F32);
// RoPE + append of `rows` keys/values ([rows][KVH*hd] each) at positions
// pos0 .. pos0+rows-1 into the cache of `p` (kv_dtype: OVF_KV_*), exactly as
// the attention kernels append the token they decode.
ovf_status launch_kv_append_rows(const AttnParams &p, const float *k, const float *v, int rows, int pos0,
                                 int kv_dtype, cudaStream_t st);
ovf_status launch_rmsnorm(const float *x, const float *g, float *y, int64_t d, float eps, cudaStream_t st);
ovf_status launch_rmsnorm_rows(const float *x, const float *g, float *y, int rows, int d, float eps, float *scales,
                               cudaStream_t st);
ovf_status launch_embed_rows(const int32_t *tokens, int n, int type, const void *w, const float *q8s, int d,
                             float *out, cudaStream_t st);
ovf_status launch_set_step_pos(DevStep *step, int cur, int next, cudaStream_t st);
ovf_status launch_argmax_rows(const float *logits, int rows, int vocab, int32_t *out, cudaStream_t st);
ovf_status launch_batch_finish(DevStep *step, int cur, int next, const int32_t *token, int32_t *tokens_log,
                               cudaStream_t st);
ovf_status launch_rope(float *v, int n_vec, int hd, const float *c, const float *s, int split_half, cudaStream_t st);
ovf_status launch_embed(const DevStep *step, int type, const void *w, const float *q8s, int d, float *hidden,
                        DevStep *step_mut, float *norm_out, float eps, TraceSlot *trace, cudaStream_t st,
                        bool pdl, unsigned *epoch = nullptr);
// ovf_tp.cu: tensor-parallel exchange (flags in every rank's arena).
struct TpExchange {
    unsigned *flags_peer[8];  // every rank's flag table [slots][world]
    const unsigned *flags_own;
    const unsigned *epoch;    // this rank's step epoch (bumped by the embedding kernel)
    int world, rank, slot;
};
ovf_status launch_tp_sum_combine(const TpExchange &x, const float *recv, int n, const float *bias, const float *resid,
                                 float *out, float *norm_out, int D, float eps, cudaStream_t st, bool pdl);
ovf_status launch_tp_moe_combine(const TpExchange &x, const float *recv, const float *w, int K, const float *resid,
                                 float *out, float *norm_out, int D, float eps, cudaStream_t st, bool pdl);
ovf_status launch_tp_lm_finish(const TpExchange &x, const unsigned long long *keys, DevStep *step, int32_t *tokens_log,
                               cudaStream_t st, bool pdl);
// ovf_moe.cu: router, combine, row gather/scatter of the MoE FFN.
ovf_status launch_moe_route(const float *x, int ld_x, const float *gamma, const float *norm_scale, const float *R,
                            int rows, int D, int E, int K, int normalize, int32_t *sel, float *w, cudaStream_t st,
                            bool pdl);
ovf_status launch_moe_combine(const float *after, const float *y, const float *w, int K, int D, float *hidden,
                              float *norm_out, float eps, cudaStream_t st, bool pdl);
ovf_status launch_moe_combine_rows(const float *a, const float *slot, const float *w, int K, int rows, int D, float *out,
                                   cudaStream_t st);
ovf_status launch_gather_rows(const float *src, const int32_t *rows, int n, int width, float *dst, cudaStream_t st);
ovf_status launch_scatter_slots(const float *src, const int32_t *rows, const int32_t *slots, int n, int K, int width,
                                float *dst, cudaStream_t st);
ovf_status launch_take_error(int *dev_slot, cudaStream_t st);
ovf_status launch_exp(const float *x, float *y, int64_t n, cudaStream_t st);
ovf_status launch_silu_mul(const float *g, const float *u, float *h, int64_t n, cudaStream_t st, bool pdl);

}  // namespace ovf
