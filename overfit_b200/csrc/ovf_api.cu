// ovf_api.cu — the extern "C" surface of libovf_cuda.so (include/ovf.h):
// host-side argument validation, status codes, and the kernel-level entry
// points that mirror the reference's static kernel classes.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "ovf_internal.cuh"

namespace ovf {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

ovf_status cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return OVF_OK;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? OVF_ENOMEM : OVF_ECUDA;
}

}  // namespace ovf

using namespace ovf;

static inline cudaStream_t S(void *st) { return reinterpret_cast<cudaStream_t>(st); }

extern "C" {

const char *ovf_last_error(void) { return ovf::g_err; }

int32_t ovf_version(void) { return 10000; }

ovf_status ovf_device_error(int32_t device, int32_t *code_out) {
    OVF_CHECK_ARG(code_out, "ovf_device_error: code_out is null");
    int prev = 0;
    OVF_CUDA_TRY(cudaGetDevice(&prev));
    OVF_CUDA_TRY(cudaSetDevice(device));
    int code = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&code, g_dev_error, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_status(e, "ovf_device_error");
    *code_out = code;
    return OVF_OK;
}

// ------------------------------------------------------------ quantizers
ovf_status ovf_quantize_q8k(const float *x, int64_t k, int8_t *q, float *scales, int16_t *bsums, void *stream) {
    OVF_CHECK_ARG(k >= 0 && k % 256 == 0, "QuantizeActivationQ8K: length %lld must be a multiple of 256", (long long)k);
    OVF_CHECK_ARG(k == 0 || (x && q && scales && bsums), "QuantizeActivationQ8K: null buffer");
    return launch_quantize_q8k(x, k, q, scales, bsums, S(stream));
}

ovf_status ovf_quantize_q8_0(const float *x, int64_t k, int8_t *q, float *scales, void *stream) {
    OVF_CHECK_ARG(k >= 0 && k % 32 == 0, "Q8 Quantize: length %lld must be a multiple of 32", (long long)k);
    OVF_CHECK_ARG(k == 0 || (x && q && scales), "Q8 Quantize: null buffer");
    return launch_quantize_q8_0(x, k, q, scales, S(stream));
}

// ----------------------------------------------------------- projections
static ovf_status check_kq(int32_t type, const void *w, int64_t n, int64_t k) {
    OVF_CHECK_ARG(type == OVF_TYPE_Q4_K || type == OVF_TYPE_Q6_K, "projection: type %d is not a K-quant", type);
    OVF_CHECK_ARG(n >= 0 && n <= 0x7FFFFFFF, "projection: bad output size");
    OVF_CHECK_ARG(k > 0 && k % 256 == 0, "projection: inputSize %lld must be a multiple of 256", (long long)k);
    OVF_CHECK_ARG(k <= 32768, "projection: inputSize %lld too large (at most 32768)", (long long)k);
    OVF_CHECK_ARG(w && aligned16(w), "projection: weight must be non-null and 16-byte aligned");
    return OVF_OK;
}

ovf_status ovf_kq_project(int32_t type, const float *x, const void *w, int64_t n, int64_t k, const float *bias,
                          float *y, int8_t *act_q, float *act_scales, int16_t *act_bsums, void *stream) {
    ovf_status st = check_kq(type, w, n, k);
    if (st) return st;
    OVF_CHECK_ARG(x && y && act_q && act_scales && act_bsums, "ProjectParallel: null buffer");
    OVF_CHECK_ARG(aligned16(x), "ProjectParallel: input must be 16-byte aligned");
    // QuantizeActivationQ8K once into the caller's scratch (as the reference
    // fills it), then the projection of the pre-quantized activation, launched
    // so that its weight streaming overlaps the quantization
    st = launch_quantize_q8k(x, k, act_q, act_scales, act_bsums, S(stream));
    if (st || n == 0) return st;
    GemvParams p{};
    p.nseg = 1;
    p.seg[0] = GemvSeg{(const uint8_t *)w, nullptr, bias, y, type, (int)n, 0};
    p.K = (int)k;
    p.act_mode = ACT_PREQ_Q8K;
    p.aq = act_q;
    p.as = act_scales;
    p.ab = act_bsums;
    p.epi = EPI_STORE;
    return gemv_launch(p, S(stream), true);
}

ovf_status ovf_kq_project_prequantized(int32_t type, const void *w, int64_t n, int64_t k, const float *bias, float *y,
                                       const int8_t *act_q, const float *act_scales, const int16_t *act_bsums,
                                       void *stream) {
    ovf_status st = check_kq(type, w, n, k);
    if (st) return st;
    OVF_CHECK_ARG(y && act_q && act_scales && act_bsums, "ProjectPreQuantized: null buffer");
    if (n == 0) return OVF_OK;
    GemvParams p{};
    p.nseg = 1;
    p.seg[0] = GemvSeg{(const uint8_t *)w, nullptr, bias, y, type, (int)n, 0};
    p.K = (int)k;
    p.act_mode = ACT_PREQ_Q8K;
    p.aq = act_q;
    p.as = act_scales;
    p.ab = act_bsums;
    p.epi = EPI_STORE;
    return gemv_launch(p, S(stream), false);
}

ovf_status ovf_q4k_project_gate_up(const float *x, const void *gate_w, const void *up_w, int64_t n, int64_t k,
                                   float *gate_y, float *up_y, int8_t *act_q, float *act_scales, int16_t *act_bsums,
                                   void *stream) {
    ovf_status st = check_kq(OVF_TYPE_Q4_K, gate_w, n, k);
    if (st) return st;
    st = check_kq(OVF_TYPE_Q4_K, up_w, n, k);
    if (st) return st;
    OVF_CHECK_ARG(x && gate_y && up_y && act_q && act_scales && act_bsums, "ProjectGateUpParallel: null buffer");
    OVF_CHECK_ARG(aligned16(x), "ProjectGateUpParallel: input must be 16-byte aligned");
    if (n == 0) return launch_quantize_q8k(x, k, act_q, act_scales, act_bsums, S(stream));
    GemvParams p{};
    p.nseg = 2;
    p.seg[0] = GemvSeg{(const uint8_t *)gate_w, nullptr, nullptr, gate_y, OVF_TYPE_Q4_K, (int)n, 0};
    p.seg[1] = GemvSeg{(const uint8_t *)up_w, nullptr, nullptr, up_y, OVF_TYPE_Q4_K, (int)n, 0};
    p.K = (int)k;
    p.act_mode = ACT_F32;
    p.x = x;
    p.aq_out = act_q;
    p.as_out = act_scales;
    p.ab_out = act_bsums;
    p.epi = EPI_STORE;
    return gemv_launch(p, S(stream), false);
}

ovf_status ovf_kq_project_batched(int32_t type, const float *x, int64_t rows, const void *w, int64_t n, int64_t k,
                                  const float *bias, float *y, int8_t *act_q, float *act_scales, int16_t *act_bsums,
                                  void *stream) {
    ovf_status st = check_kq(type, w, n, k);
    if (st) return st;
    OVF_CHECK_ARG(rows > 0, "ProjectBatched: rows must be positive");
    OVF_CHECK_ARG(x && y && act_q && act_scales && act_bsums, "ProjectBatched: null buffer");
    OVF_CHECK_ARG(aligned16(x) && aligned16(act_q), "ProjectBatched: input and act_q must be 16-byte aligned");
    // One row: the streaming decode GEMV is the faster kernel for the same sums.
    if (rows == 1) return ovf_kq_project(type, x, w, n, k, bias, y, act_q, act_scales, act_bsums, stream);
    st = launch_quantize_q8k(x, rows * k, act_q, act_scales, act_bsums, S(stream));
    if (st) return st;
    const size_t wbytes = (size_t)n * (size_t)(k / 256) * (type == OVF_TYPE_Q4_K ? 144 : 210);
    return launch_batched_project(type, w, nullptr, wbytes, bias, act_q, act_scales, act_bsums, y, n, k, rows,
                                  S(stream));
}

int64_t ovf_tc_scratch_bytes(int64_t rows, int64_t k) {
    if (rows <= 0 || k <= 0 || k % 64) return 0;
    const int64_t q8 = tc8_scratch_bytes(rows, k);
    return k % 256 ? q8 : std::max(q8, tc_scratch_bytes(rows, k));
}

ovf_status ovf_kq_project_batched_tc(int32_t type, const float *x, int64_t rows, const void *w, int64_t n, int64_t k,
                                     const float *bias, float *y, int8_t *act_q, float *act_scales,
                                     int16_t *act_bsums, void *scratch, void *stream) {
    ovf_status st = check_kq(type, w, n, k);
    if (st) return st;
    OVF_CHECK_ARG(type == OVF_TYPE_Q4_K || (type == OVF_TYPE_Q6_K && k % 2048 == 0),
                  "ProjectBatched (tensor cores): Q4_K weights, or Q6_K with inputSize a multiple of 2048");
    OVF_CHECK_ARG(rows > 0 && rows <= (int64_t)65535 * 128, "ProjectBatched (tensor cores): rows must be in [1, 8388480]");
    OVF_CHECK_ARG(x && y && act_q && act_scales && act_bsums && scratch, "ProjectBatched (tensor cores): null buffer");
    if (n == 0) return OVF_OK;
    st = launch_quantize_q8k(x, rows * k, act_q, act_scales, act_bsums, S(stream));
    if (st) return st;
    if (type == OVF_TYPE_Q6_K)
        return launch_tc6_project(w, bias, act_q, act_scales, act_bsums, y, n, k, rows, scratch, S(stream));
    return launch_tc_project(type, w, bias, act_q, act_scales, act_bsums, y, n, k, rows, scratch, S(stream));
}

static ovf_status q8_project_impl(const float *x, const int8_t *wq, const float *ws, int64_t n, int64_t k,
                                  const float *bias, float *y, int8_t *xq, float *xs, cudaStream_t st) {
    OVF_CHECK_ARG(n >= 0 && n <= 0x7FFFFFFF, "Q8 ProjectParallel: bad output size");
    OVF_CHECK_ARG(k > 0 && k % 32 == 0 && k <= 32 * 512, "Q8 ProjectParallel: inputSize %lld must be a multiple of 32",
                  (long long)k);
    OVF_CHECK_ARG(x && wq && ws && y && xq && xs, "Q8 ProjectParallel: null buffer");
    OVF_CHECK_ARG(aligned16(x) && aligned16(wq) && aligned16(ws), "Q8 ProjectParallel: buffers must be 16-byte aligned");
    if (n == 0) return launch_quantize_q8_0(x, k, xq, xs, st);
    GemvParams p{};
    p.nseg = 1;
    p.seg[0] = GemvSeg{(const uint8_t *)wq, ws, bias, y, OVF_TYPE_Q8_0, (int)n, 0};
    p.K = (int)k;
    p.act_mode = ACT_F32;
    p.x = x;
    p.aq_out = xq;
    p.as_out = xs;
    p.epi = EPI_STORE;
    p.q8_group = 0;
    return gemv_launch(p, st, false);
}

ovf_status ovf_q8_0_project(const float *x, const int8_t *wq, const float *wscales, int64_t n, int64_t k,
                            const float *bias, float *y, int8_t *x_q, float *x_scales, void *stream) {
    return q8_project_impl(x, wq, wscales, n, k, bias, y, x_q, x_scales, S(stream));
}

ovf_status ovf_q8_0_project_batched(const float *x, int64_t rows, const int8_t *wq, const float *wscales, int64_t n,
                                    int64_t k, const float *bias, float *y, int8_t *x_q, float *x_scales, void *stream) {
    OVF_CHECK_ARG(rows > 0, "Q8 ProjectBatched: rows must be positive");
    OVF_CHECK_ARG(n >= 0 && n <= 0x7FFFFFFF, "Q8 ProjectBatched: bad output size");
    OVF_CHECK_ARG(k > 0 && k % 32 == 0 && k <= 32 * 512, "Q8 ProjectBatched: inputSize %lld must be a multiple of 32",
                  (long long)k);
    OVF_CHECK_ARG(x && wq && wscales && y && x_q && x_scales, "Q8 ProjectBatched: null buffer");
    OVF_CHECK_ARG(aligned16(x) && aligned16(wq) && aligned16(x_q), "Q8 ProjectBatched: buffers must be 16-byte aligned");
    ovf_status st = launch_quantize_q8_0(x, rows * k, x_q, x_scales, S(stream));
    if (st) return st;
    return launch_batched_project(OVF_TYPE_Q8_0, wq, wscales, (size_t)n * (size_t)k, bias, x_q, x_scales, nullptr, y,
                                  n, k, rows, S(stream));
}

ovf_status ovf_q8_0_project_batched_tc(const float *x, int64_t rows, const int8_t *wq, const float *wscales,
                                       int64_t n, int64_t k, const float *bias, float *y, int8_t *x_q,
                                       float *x_scales, void *scratch, void *stream) {
    OVF_CHECK_ARG(rows > 0 && rows <= (int64_t)65535 * 64, "Q8 ProjectBatched (tensor cores): rows must be in [1, 4194240]");
    OVF_CHECK_ARG(n >= 0 && n <= 0x7FFFFFFF, "Q8 ProjectBatched (tensor cores): bad output size");
    OVF_CHECK_ARG(k > 0 && k % 64 == 0, "Q8 ProjectBatched (tensor cores): inputSize %lld must be a multiple of 64",
                  (long long)k);
    OVF_CHECK_ARG(x && wq && wscales && y && x_q && x_scales && scratch, "Q8 ProjectBatched (tensor cores): null buffer");
    OVF_CHECK_ARG(aligned16(x) && aligned16(wq) && aligned16(x_q) && aligned16(scratch),
                  "Q8 ProjectBatched (tensor cores): buffers must be 16-byte aligned");
    if (n == 0) return OVF_OK;
    ovf_status st = launch_quantize_q8_0(x, rows * k, x_q, x_scales, S(stream));
    if (st) return st;
    return launch_tc8_project(wq, wscales, bias, x_q, x_scales, y, n, k, rows, 0, scratch, S(stream));
}

// --------------------------------------------------------------- codecs
ovf_status ovf_quantize_q4k(const float *w, int64_t rows, int64_t k, void *out, void *stream) {
    OVF_CHECK_ARG(rows >= 0 && k > 0 && k % 256 == 0, "QuantizeQ4_K: inputSize must be a multiple of 256");
    OVF_CHECK_ARG(rows == 0 || (w && out), "QuantizeQ4_K: null buffer");
    return launch_encode(OVF_TYPE_Q4_K, w, rows, k, out, S(stream));
}

ovf_status ovf_quantize_q6k(const float *w, int64_t rows, int64_t k, void *out, void *stream) {
    OVF_CHECK_ARG(rows >= 0 && k > 0 && k % 256 == 0, "Q6_K encode: inputSize must be a multiple of 256");
    OVF_CHECK_ARG(rows == 0 || (w && out), "Q6_K encode: null buffer");
    return launch_encode(OVF_TYPE_Q6_K, w, rows, k, out, S(stream));
}

ovf_status ovf_quantize_q8_0_gguf(const float *w, int64_t n, void *out, void *stream) {
    OVF_CHECK_ARG(n >= 0 && n % 32 == 0, "Q8_0 encode: element count must be a multiple of 32");
    OVF_CHECK_ARG(n == 0 || (w && out), "Q8_0 encode: null buffer");
    return launch_encode(OVF_TYPE_Q8_0, w, 1, n, out, S(stream));
}

ovf_status ovf_q8_0_deinterleave(const void *gguf, int64_t n, int8_t *q, float *scales, void *stream) {
    OVF_CHECK_ARG(n >= 0 && n % 32 == 0, "LoadTensorQ8_0Raw: element count %lld is not divisible by 32", (long long)n);
    OVF_CHECK_ARG(n == 0 || (gguf && q && scales), "LoadTensorQ8_0Raw: null buffer");
    return launch_q8_0_deinterleave(gguf, n, q, scales, S(stream));
}

ovf_status ovf_dequant_rows(int32_t type, const void *w, const float *q8_scales, int64_t row0, int64_t nrows,
                            int64_t k, float *dst, void *stream) {
    OVF_CHECK_ARG(type == OVF_TYPE_Q4_K || type == OVF_TYPE_Q6_K || type == OVF_TYPE_Q8_0 || type == OVF_TYPE_F32,
                  "DecodeRow: unsupported type %d", type);
    OVF_CHECK_ARG(row0 >= 0 && nrows >= 0 && k > 0, "DecodeRow: bad range");
    OVF_CHECK_ARG((type != OVF_TYPE_Q4_K && type != OVF_TYPE_Q6_K) || k % 256 == 0, "DecodeRow: k must be a multiple of 256");
    OVF_CHECK_ARG(type != OVF_TYPE_Q8_0 || (k % 32 == 0 && q8_scales), "DecodeRow: Q8_0 needs k%%32==0 and scales");
    OVF_CHECK_ARG(nrows == 0 || (w && dst), "DecodeRow: null buffer");
    return launch_dequant_rows(type, w, q8_scales, row0, nrows, k, dst, S(stream));
}

ovf_status ovf_requant_q8_0(int32_t src_type, const void *w, int64_t rows, int64_t k, int8_t *q, float *scales,
                            void *stream) {
    OVF_CHECK_ARG(src_type == OVF_TYPE_Q4_K || src_type == OVF_TYPE_Q6_K || src_type == OVF_TYPE_F32,
                  "requant: unsupported source type %d", src_type);
    OVF_CHECK_ARG(rows >= 0 && k > 0 && k % 32 == 0, "requant: k must be a multiple of 32");
    OVF_CHECK_ARG(src_type == OVF_TYPE_F32 || k % 256 == 0, "requant: K-quant k must be a multiple of 256");
    OVF_CHECK_ARG(rows == 0 || (w && q && scales), "requant: null buffer");
    return launch_requant_q8_0(src_type, w, rows, k, q, scales, S(stream));
}

// ------------------------------------------------------------------- ops
ovf_status ovf_rmsnorm(const float *x, const float *gamma, float *y, int64_t d, float eps, void *stream) {
    OVF_CHECK_ARG(d > 0 && x && y, "RmsNormalize: bad arguments");
    return launch_rmsnorm(x, gamma, y, d, eps, S(stream));
}

ovf_status ovf_exp_f32(const float *x, float *y, int64_t n, void *stream) {
    OVF_CHECK_ARG(n >= 0 && (n == 0 || (x && y)), "Exp: bad arguments");
    return launch_exp(x, y, n, S(stream));
}

ovf_status ovf_swiglu(const float *gate, const float *up, float *h, int64_t n, void *stream) {
    OVF_CHECK_ARG(n >= 0 && (n == 0 || (gate && up && h)), "ApplySiLU: bad arguments");
    if (n == 0) return OVF_OK;
    return launch_silu_mul(gate, up, h, n, S(stream), false);
}

ovf_status ovf_rope_apply(float *v, int32_t n_vec, int32_t head_dim, const float *cos_row, const float *sin_row,
                          int32_t split_half, void *stream) {
    OVF_CHECK_ARG(head_dim > 0 && head_dim % 2 == 0, "RopeKernel.Apply: headDimension must be positive and even");
    OVF_CHECK_ARG(n_vec >= 0 && (n_vec == 0 || (v && cos_row && sin_row)), "RopeKernel.Apply: null buffer");
    return launch_rope(v, n_vec, head_dim, cos_row, sin_row, split_half, S(stream));
}

int64_t ovf_attention_scratch_bytes(int32_t n_heads, int32_t n_kv_heads, int32_t head_dim) {
    if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0) return 0;
    return attn_scratch_bytes(n_heads, n_kv_heads, head_dim);
}

ovf_status ovf_attention_decode(const float *q, const void *k_cache, const void *v_cache, float *out, int32_t n_heads,
                                int32_t n_kv_heads, int32_t head_dim, int32_t max_ctx, int32_t seq_len, float scale,
                                void *scratch, int32_t *counters, void *stream) {
    OVF_CHECK_ARG(q && k_cache && v_cache && out && scratch && counters, "ComputeSingleHead: null buffer");
    OVF_CHECK_ARG(seq_len >= 1, "ComputeSingleHead: seq_len must be >= 1 (an empty sequence gives zeros on the host side)");
    AttnParams p{};
    p.q = q;
    p.kc = (__half *)k_cache;
    p.vc = (__half *)v_cache;
    p.out = out;
    p.partial = (float *)scratch;
    p.counters = counters;
    p.H = n_heads;
    p.KVH = n_kv_heads;
    p.hd = head_dim;
    p.max_ctx = max_ctx;
    p.seq_len_host = seq_len;
    p.scale = scale;
    return launch_attention(p, S(stream), false);
}

ovf_status ovf_attention_single_head(const float *q, const float *k_cache, const float *v_cache, float *out,
                                     int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t max_ctx,
                                     int32_t seq_len, float scale, void *stream) {
    OVF_CHECK_ARG(q && k_cache && v_cache && out, "ComputeSingleHead: null buffer");
    OVF_CHECK_ARG(seq_len >= 1 && seq_len <= max_ctx, "ComputeSingleHead: seq_len must be in [1, max_ctx]");
    AttnParams p{};
    p.q = q;
    p.kc = (__half *)k_cache;
    p.vc = (__half *)v_cache;
    p.out = out;
    p.H = n_heads;
    p.KVH = n_kv_heads;
    p.hd = head_dim;
    p.max_ctx = max_ctx;
    p.seq_len_host = seq_len;
    p.scale = scale;
    return launch_attention_exact(p, seq_len, S(stream), false);
}

ovf_status ovf_attention_single_head_f16(const float *q, const void *k_cache, const void *v_cache, float *out,
                                         int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t max_ctx,
                                         int32_t seq_len, float scale, void *stream) {
    OVF_CHECK_ARG(q && k_cache && v_cache && out, "ComputeSingleHead (fp16 cache): null buffer");
    OVF_CHECK_ARG(seq_len >= 1 && seq_len <= max_ctx, "ComputeSingleHead (fp16 cache): seq_len must be in [1, max_ctx]");
    AttnParams p{};
    p.q = q;
    p.kc = (__half *)k_cache;
    p.vc = (__half *)v_cache;
    p.out = out;
    p.H = n_heads;
    p.KVH = n_kv_heads;
    p.hd = head_dim;
    p.max_ctx = max_ctx;
    p.seq_len_host = seq_len;
    p.scale = scale;
    return launch_attention_exact(p, seq_len, S(stream), false, OVF_KV_F16);
}

ovf_status ovf_attention_single_head_q8(const float *q, const int8_t *k_cache, const float *k_scales,
                                        const int8_t *v_cache, const float *v_scales, float *out, int32_t n_heads,
                                        int32_t n_kv_heads, int32_t head_dim, int32_t max_ctx, int32_t seq_len,
                                        float scale, void *stream) {
    OVF_CHECK_ARG(q && k_cache && k_scales && v_cache && v_scales && out, "ComputeSingleHeadQ8: null buffer");
    OVF_CHECK_ARG(seq_len >= 1 && seq_len <= max_ctx, "ComputeSingleHeadQ8: seq_len must be in [1, max_ctx]");
    OVF_CHECK_ARG(head_dim % 32 == 0, "ComputeSingleHeadQ8: head_dim must be a multiple of 32");
    AttnParams p{};
    p.q = q;
    p.kc = (__half *)k_cache;
    p.vc = (__half *)v_cache;
    p.ks = const_cast<float *>(k_scales);
    p.vs = const_cast<float *>(v_scales);
    p.out = out;
    p.H = n_heads;
    p.KVH = n_kv_heads;
    p.hd = head_dim;
    p.max_ctx = max_ctx;
    p.seq_len_host = seq_len;
    p.scale = scale;
    return launch_attention_exact(p, seq_len, S(stream), false, OVF_KV_Q8);
}

}  // extern "C"
