// ovf_ops.cu — decode attention (flash-decode, GQA, fused RoPE + KV append),
// RMSNorm, RoPE, embedding lookup and SiLU*up for sm_100a.
#include "ovf_internal.cuh"

#include <algorithm>
#include <cstdlib>

namespace ovf {

// ---------------------------------------------------------------- attention
// One CTA per (sequence split, KV head).  The CTA rotates the queries of its
// KV group (RoPE at the current position, Rope/RopeKernel.cs:46-93), scores
// its slice of the fp16 cache (dot * 1/sqrt(hd), CachedAttentionKernel.cs:
// 65-82), keeps an unnormalised softmax partial (max, sum, sum p*v) and
// writes it to scratch.  The CTA whose slice holds the current position also
// rotates the new key and appends key/value to the cache.  The last CTA of a
// KV group (atomic ticket) merges the partials of its heads with a
// log-sum-exp rescale in fixed split order; an empty or non-finite sum gives
// zeros as in the reference (:88-92).
static constexpr int kAttnThreads = 128;

int attn_splits(int n_kv_heads) {
    static const int forced = [] {
        const char *e = getenv("OVF_ATTN_SPLITS");
        return e ? atoi(e) : 0;
    }();
    if (forced > 0) return std::min(64, forced);
    return std::max(1, std::min(64, 296 / std::max(1, n_kv_heads)));
}

int64_t attn_scratch_bytes(int H, int KVH, int hd) {
    return (int64_t)H * attn_splits(KVH) * (hd + 2) * (int64_t)sizeof(float);
}

__device__ __forceinline__ void rope_rotate(float *v, int hd, const float *c, const float *s, int split_half,
                                            int tid, int nthreads) {
    const int half = hd / 2;
    for (int i = tid; i < half; i += nthreads) {
        if (split_half) {
            const float x0 = v[i], x1 = v[i + half];
            v[i] = fsub(fmul(x0, c[i]), fmul(x1, s[i]));
            v[i + half] = fadd(fmul(x0, s[i]), fmul(x1, c[i]));
        } else {
            const float x0 = v[2 * i], x1 = v[2 * i + 1];
            v[2 * i] = fsub(fmul(x0, c[i]), fmul(x1, s[i]));
            v[2 * i + 1] = fadd(fmul(x0, s[i]), fmul(x1, c[i]));
        }
    }
}

// GT > 0: the query heads per KV head are a compile-time constant (the
// per-head accumulators stay in registers); GT == 0: runtime count (<= 16).
template <int GT, int HD>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float asmem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = kAttnThreads / 32;
    const int split = blockIdx.x, g = blockIdx.y;
    const int G = GT > 0 ? GT : p.H / p.KVH, hd = p.hd;
    constexpr int GM = GT > 0 ? GT : 16;
    float *qs = asmem;                       // [G][hd]
    float *knew = qs + G * hd;               // [hd]
    float *vnew = knew + hd;                 // [hd]
    float *sc = vnew + hd;                   // [G][chunk_max]
    float *mh = sc + p.sc_floats;            // [G] max, [G] sum
    __shared__ int s_last;

    pdl_wait();
    const int pos = p.pos_dev ? *p.pos_dev : p.seq_len_host - 1;
    const int seq = pos + 1;
    const int chunk = (seq + p.n_splits - 1) / p.n_splits;
    const int t0 = split * chunk;
    const int t1 = min(seq, t0 + chunk);
    const int nt = max(0, t1 - t0);
    const size_t cache_head = (size_t)g * p.max_ctx * hd;

    for (int i = tid; i < G * hd; i += kAttnThreads) qs[i] = p.q[(size_t)(g * G) * hd + i];
    const bool owns_new = p.k_new != nullptr && pos >= t0 && pos < t1;
    if (owns_new)
        for (int i = tid; i < hd; i += kAttnThreads) {
            knew[i] = p.k_new[(size_t)g * hd + i];
            vnew[i] = p.v_new[(size_t)g * hd + i];
        }
    __syncthreads();
    pdl_launch_dependents();
    if (p.rope_cos) {
        const float *c = p.rope_cos + (size_t)pos * (hd / 2), *s = p.rope_sin + (size_t)pos * (hd / 2);
        for (int h = 0; h < G; ++h) rope_rotate(qs + h * hd, hd, c, s, p.split_half, tid, kAttnThreads);
        if (owns_new) rope_rotate(knew, hd, c, s, p.split_half, tid, kAttnThreads);
        __syncthreads();
    }
    if (owns_new) {
        // Append the current token; the cache keeps K rotated (CachedSingleHeadAttention.cs:264-281).
        for (int i = tid; i < hd; i += kAttnThreads) {
            const __half kh = __float2half_rn(knew[i]), vh = __float2half_rn(vnew[i]);
            p.kc[cache_head + (size_t)pos * hd + i] = kh;
            p.vc[cache_head + (size_t)pos * hd + i] = vh;
            knew[i] = __half2float(kh);
            vnew[i] = __half2float(vh);
        }
        __syncthreads();
    }

    // Scores: four threads per key, each a quarter of the head dimension read
    // with independent 16-byte loads issued together; partial dots for all
    // query heads of the group are folded with two shuffles.
    {
        constexpr int HDQ = HD > 0 ? HD / 4 : 64;  // dims per thread (compile-time bound)
        const int hq = hd / 4;
        const int kq = tid & 3, kslot = tid >> 2;  // 32 keys per pass
        for (int tb = 0; tb < nt; tb += kAttnThreads / 4) {
            const int t = tb + kslot;
            const bool ok = t < nt;
            const int pt = t0 + (ok ? t : 0);
            float kv[HDQ];
            if (ok && owns_new && pt == pos) {
#pragma unroll
                for (int i = 0; i < HDQ; ++i)
                    if (i < hq) kv[i] = knew[kq * hq + i];
            } else {
                const uint4 *kr = reinterpret_cast<const uint4 *>(p.kc + cache_head + (size_t)pt * hd + kq * hq);
                uint4 w[HDQ / 8];
#pragma unroll
                for (int i = 0; i < HDQ / 8; ++i)
                    if (i < hq / 8) w[i] = kr[i];
#pragma unroll
                for (int i = 0; i < HDQ / 8; ++i) {
                    const __half2 *h2 = reinterpret_cast<const __half2 *>(&w[i]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __half22float2(h2[j]);
                        kv[8 * i + 2 * j] = f.x;
                        kv[8 * i + 2 * j + 1] = f.y;
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < GM; ++h) {
                if (h < G) {
                    const float *qh = qs + h * hd + kq * hq;
                    float acc = 0.0f;
#pragma unroll
                    for (int i = 0; i < HDQ; ++i)
                        if (i < hq) acc = fadd(acc, fmul(qh[i], kv[i]));
                    acc = fadd(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 1));
                    acc = fadd(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 2));
                    if (ok && kq == 0) sc[h * p.chunk_max + t] = fmul(acc, p.scale);
                }
            }
        }
    }
    __syncthreads();
    // Per head: max, exp, sum (warp per head).
    for (int h = warp; h < G; h += nw) {
        float m = -INFINITY;
        for (int t = lane; t < nt; t += 32) m = fmaxf(m, sc[h * p.chunk_max + t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        float l = 0.0f;
        for (int t = lane; t < nt; t += 32) {
            const float e = expf(fsub(sc[h * p.chunk_max + t], m));
            sc[h * p.chunk_max + t] = e;
            l = fadd(l, e);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l = fadd(l, __shfl_xor_sync(0xFFFFFFFFu, l, o));
        if (lane == 0) {
            mh[h] = m;
            mh[G + h] = l;
        }
    }
    __syncthreads();
    // Weighted values: a thread per (dimension pair, quarter of the keys);
    // loads of consecutive keys are independent, so four are kept in flight.
    {
        const int npair = hd / 2;
        const int part = tid / npair, nparts = kAttnThreads / npair;  // hd=128: 64 pairs x 2 parts
        const int d2 = tid % npair;
        float o0[GM], o1[GM];
#pragma unroll
        for (int h = 0; h < GM; ++h) o0[h] = o1[h] = 0.0f;
        if (part < nparts) {
            // eight keys' values loaded before any is used (independent loads)
            for (int tb = part; tb < nt; tb += 8 * nparts) {
                float2 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int t = tb + u * nparts;
                    const int pt = t0 + t;
                    if (t >= nt) v[u] = make_float2(0.0f, 0.0f);
                    else if (owns_new && pt == pos) v[u] = make_float2(vnew[2 * d2], vnew[2 * d2 + 1]);
                    else v[u] = __half22float2(reinterpret_cast<const __half2 *>(p.vc + cache_head + (size_t)pt * hd)[d2]);
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int t = tb + u * nparts;
                    if (t < nt) {
#pragma unroll
                        for (int h = 0; h < GM; ++h) {
                            if (h < G) {
                                const float pr = sc[h * p.chunk_max + t];
                                o0[h] = fadd(o0[h], fmul(pr, v[u].x));
                                o1[h] = fadd(o1[h], fmul(pr, v[u].y));
                            }
                        }
                    }
                }
            }
        }
        // Partials of part 0..nparts-1 are written side by side and summed by part 0.
        float *tmp = sc;  // scores are no longer needed
        __syncthreads();
        if (part > 0 && part < nparts)
            for (int h = 0; h < G; ++h) {
                tmp[((part - 1) * G + h) * hd + 2 * d2] = o0[h];
                tmp[((part - 1) * G + h) * hd + 2 * d2 + 1] = o1[h];
            }
        __syncthreads();
        if (part == 0) {
            for (int q = 1; q < nparts; ++q)
                for (int h = 0; h < G; ++h) {
                    o0[h] = fadd(o0[h], tmp[((q - 1) * G + h) * hd + 2 * d2]);
                    o1[h] = fadd(o1[h], tmp[((q - 1) * G + h) * hd + 2 * d2 + 1]);
                }
            for (int h = 0; h < G; ++h) {
                float *dst = p.partial + ((size_t)(g * G + h) * p.n_splits + split) * (hd + 2);
                dst[2 * d2] = o0[h];
                dst[2 * d2 + 1] = o1[h];
            }
        }
    }
    if (tid < G) {
        float *pp = p.partial + ((size_t)(g * G + tid) * p.n_splits + split) * (hd + 2) + hd;
        pp[0] = mh[tid];
        pp[1] = mh[G + tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int ticket = atomicAdd(&p.counters[g], 1);
        s_last = (ticket == p.n_splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Merge: every split's (max, sum) of every head in one parallel pass, the
    // rescale weights exp(m_s - M) in another, then each dimension loads all
    // of its splits at once (independent loads) and sums them in split order.
    {
        const int ns = p.n_splits;
        float *mm = sc;              // [G][ns] split maxima (-inf when empty)
        float *ll = mm + G * ns;     // [G][ns] split sums
        float *ww = ll + G * ns;     // [G][ns] weights
        float *hm = ww + G * ns;     // [G] M, [G] 1/L (0 when the sum is not usable)
        for (int i = tid; i < G * ns; i += kAttnThreads) {
            const int h = i / ns, s2 = i - h * ns;
            const float *pp = p.partial + ((size_t)(g * G + h) * ns + s2) * (hd + 2) + hd;
            const float ls = __ldcg(pp + 1), ms = __ldcg(pp);
            mm[i] = ls > 0.0f ? ms : -INFINITY;
            ll[i] = ls;
        }
        __syncthreads();
        if (tid < G) {
            float M = -INFINITY;
            for (int s2 = 0; s2 < ns; ++s2) M = fmaxf(M, mm[tid * ns + s2]);
            hm[tid] = M;
        }
        __syncthreads();
        for (int i = tid; i < G * ns; i += kAttnThreads)
            ww[i] = ll[i] > 0.0f ? expf(fsub(mm[i], hm[i / ns])) : 0.0f;
        __syncthreads();
        if (tid < G) {
            float L = 0.0f;
            for (int s2 = 0; s2 < ns; ++s2) L = fadd(L, fmul(ll[tid * ns + s2], ww[tid * ns + s2]));
            hm[G + tid] = (L > 0.0f && isfinite(L)) ? fdiv(1.0f, L) : 0.0f;
        }
        __syncthreads();
        for (int h = 0; h < G; ++h) {
            const float *base = p.partial + (size_t)(g * G + h) * ns * (hd + 2);
            const float inv = hm[G + h];
            for (int d = tid; d < hd; d += kAttnThreads) {
                float v[64];
#pragma unroll
                for (int s2 = 0; s2 < 64; ++s2)
                    v[s2] = s2 < ns ? __ldcg(base + (size_t)s2 * (hd + 2) + d) : 0.0f;
                float acc = 0.0f;
#pragma unroll
                for (int s2 = 0; s2 < 64; ++s2)
                    if (s2 < ns) acc = fadd(acc, fmul(ww[h * ns + s2], v[s2]));
                p.out[(size_t)(g * G + h) * hd + d] = inv > 0.0f ? fmul(acc, inv) : 0.0f;
            }
        }
    }
    if (tid == 0) p.counters[g] = 0;
}

ovf_status launch_attention(const AttnParams &p0, cudaStream_t st, bool pdl) {
    AttnParams p = p0;
    OVF_CHECK_ARG(p.H > 0 && p.KVH > 0 && p.H % p.KVH == 0, "attention: n_heads must be a multiple of n_kv_heads");
    OVF_CHECK_ARG(p.H / p.KVH <= 16, "attention: at most 16 query heads per KV head");
    OVF_CHECK_ARG(p.hd >= 32 && p.hd <= 256 && p.hd % 32 == 0, "attention: head_dim must be 32..256, multiple of 32");
    OVF_CHECK_ARG(p.max_ctx > 0, "attention: max_ctx must be positive");
    if (!p.pos_dev) OVF_CHECK_ARG(p.seq_len_host >= 1 && p.seq_len_host <= p.max_ctx, "attention: seq_len out of range");
    p.n_splits = attn_splits(p.KVH);
    const int span = p.pos_dev ? p.max_ctx : p.seq_len_host;
    p.chunk_max = (span + p.n_splits - 1) / p.n_splits;
    const int G = p.H / p.KVH;
    const int nparts = kAttnThreads / (p.hd / 2);
    const size_t scratch_f = std::max({(size_t)G * p.chunk_max, (size_t)(nparts - 1) * G * p.hd,
                                       (size_t)3 * G * p.n_splits + 2 * G});
    p.sc_floats = (int)scratch_f;
    const size_t smem = sizeof(float) * ((size_t)G * p.hd + 2 * p.hd + scratch_f + 2 * G);
    OVF_CHECK_ARG(smem <= 48 * 1024, "attention: context too long for one split's score buffer");
    cudaError_t e;
    const dim3 grid(p.n_splits, p.KVH), block(kAttnThreads);
#define OVF_ATTN(gt, hdv) e = launch_pdl(attention_kernel<gt, hdv>, grid, block, smem, st, pdl, p)
    if (p.hd == 128 && G == 4) OVF_ATTN(4, 128);
    else if (p.hd == 128 && G == 8) OVF_ATTN(8, 128);
    else if (p.hd == 128 && G == 1) OVF_ATTN(1, 128);
    else if (p.hd == 64 && G == 7) OVF_ATTN(7, 64);
    else if (p.hd == 64 && G == 4) OVF_ATTN(4, 64);
    else if (p.hd == 64 && G == 8) OVF_ATTN(8, 64);
    else OVF_ATTN(0, 0);
#undef OVF_ATTN
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "attention_kernel launch");
}

// ------------------------------------------------------------------ RMSNorm
// Runtime/CachedTransformerBlock.cs:525-552 (RmsNormalize): warp 0 runs
// the sequential sum of squares, then every thread scales its elements as
// (x * scale) * gamma.  Bit-identical to the reference.
__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ gm, float *__restrict__ y,
                               int64_t d, float eps) {
    __shared__ __align__(16) float stage[2048];
    const float scale = rms_scale(cta_seq_sumsq(x, (int)d, 0.0f, stage), (int)d, eps);
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) y[i] = gm ? fmul(fmul(x[i], scale), gm[i]) : fmul(x[i], scale);
}

ovf_status launch_rmsnorm(const float *x, const float *g, float *y, int64_t d, float eps, cudaStream_t st) {
    rmsnorm_kernel<<<1, 1024, 0, st>>>(x, g, y, d, eps);
    return cuda_status(cudaGetLastError(), "rmsnorm");
}

// Row-wise form for the batched prefill: one CTA per row, the same
// sequential sum of squares per row; `scales` (optional) receives each
// row's 1/rms.
__global__ void rmsnorm_rows_kernel(const float *__restrict__ x, const float *__restrict__ gm, float *__restrict__ y,
                                    int d, float eps, float *scales) {
    __shared__ __align__(16) float stage[2048];
    const float *xr = x + (size_t)blockIdx.x * d;
    float *yr = y + (size_t)blockIdx.x * d;
    const float scale = rms_scale(cta_seq_sumsq(xr, d, 0.0f, stage), d, eps);
    for (int i = threadIdx.x; i < d; i += blockDim.x) yr[i] = gm ? fmul(fmul(xr[i], scale), gm[i]) : fmul(xr[i], scale);
    if (scales && threadIdx.x == 0) scales[blockIdx.x] = scale;
}

ovf_status launch_rmsnorm_rows(const float *x, const float *g, float *y, int rows, int d, float eps, float *scales,
                               cudaStream_t st) {
    if (rows == 0) return OVF_OK;
    rmsnorm_rows_kernel<<<rows, 1024, 0, st>>>(x, g, y, d, eps, scales);
    return cuda_status(cudaGetLastError(), "rmsnorm_rows");
}

// --------------------------------------------------------------------- RoPE
__global__ void rope_kernel(float *v, int n_vec, int hd, const float *c, const float *s, int split_half) {
    const int vec = blockIdx.x;
    if (vec < n_vec) rope_rotate(v + (size_t)vec * hd, hd, c, s, split_half, threadIdx.x, blockDim.x);
}

ovf_status launch_rope(float *v, int n_vec, int hd, const float *c, const float *s, int split_half, cudaStream_t st) {
    if (n_vec == 0) return OVF_OK;
    rope_kernel<<<n_vec, 64, 0, st>>>(v, n_vec, hd, c, s, split_half);
    return cuda_status(cudaGetLastError(), "rope");
}

// ------------------------------------------------------------ embedding row
// CachedLlamaSession.EmbedAndAdvance (:851-868): decode row `token` of the
// embedding (DecodeWeight.DequantizeRow) into hidden and advance the
// position; then warp 0 runs the first layer's RMSNorm sum of squares in
// the reference's order and leaves the scale in norm_out (one CTA).
__global__ void embed_kernel(DevStep *step, int type, const uint8_t *__restrict__ w, const float *__restrict__ q8s,
                             int d, float *__restrict__ hidden, float *norm_out, float eps, TraceSlot *trace,
                             unsigned *epoch) {
    if (threadIdx.x == 0) trace_mark(trace, TR_START);
    pdl_wait();
    if (threadIdx.x == 0) trace_mark(trace, TR_WAITED);
    const int token = step->token;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        float v;
        if (type == OVF_TYPE_Q4_K) v = q4k_elem(w + ((int64_t)token * (d / 256) + i / 256) * 144, i % 256);
        else if (type == OVF_TYPE_Q6_K) v = q6k_elem(w + ((int64_t)token * (d / 256) + i / 256) * 210, i % 256);
        else if (type == OVF_TYPE_Q8_0)
            v = fmul(q8s[(int64_t)token * (d / 32) + i / 32], (float)reinterpret_cast<const int8_t *>(w)[(int64_t)token * d + i]);
        else v = reinterpret_cast<const float *>(w)[(int64_t)token * d + i];
        hidden[i] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        step->cur_pos = step->next_pos;
        step->next_pos += 1;
        if (epoch) *epoch += 1;  // tensor parallel: this step's exchange epoch
    }
    if (norm_out) {
        __shared__ __align__(16) float stage[2048];
        const float ss = cta_seq_sumsq(hidden, d, 0.0f, stage);
        if (threadIdx.x == 0) *norm_out = rms_scale(ss, d, eps);
    }
    if (threadIdx.x == 0) trace_mark(trace, TR_END);
    pdl_launch_dependents();
}

ovf_status launch_embed(const DevStep *, int type, const void *w, const float *q8s, int d, float *hidden,
                        DevStep *step, float *norm_out, float eps, TraceSlot *trace, cudaStream_t st, bool pdl,
                        unsigned *epoch) {
    cudaError_t e = launch_pdl(embed_kernel, dim3(1), dim3(1024), 0, st, pdl, step, type, (const uint8_t *)w, q8s, d,
                               hidden, norm_out, eps, trace, epoch);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "embed");
}

// Embedding rows of a prompt chunk (CachedLlamaSession.PrefillBatchedQuant
// :818-835, DequantizeRow per token), one CTA per token, the same element
// decode as embed_kernel.
__global__ void embed_rows_kernel(const int32_t *__restrict__ tokens, int type, const uint8_t *__restrict__ w,
                                  const float *__restrict__ q8s, int d, float *__restrict__ out) {
    const int64_t token = tokens[blockIdx.x];
    float *row = out + (size_t)blockIdx.x * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        float v;
        if (type == OVF_TYPE_Q4_K) v = q4k_elem(w + (token * (d / 256) + i / 256) * 144, i % 256);
        else if (type == OVF_TYPE_Q6_K) v = q6k_elem(w + (token * (d / 256) + i / 256) * 210, i % 256);
        else if (type == OVF_TYPE_Q8_0)
            v = fmul(q8s[token * (d / 32) + i / 32], (float)reinterpret_cast<const int8_t *>(w)[token * d + i]);
        else v = reinterpret_cast<const float *>(w)[token * d + i];
        row[i] = v;
    }
}

ovf_status launch_embed_rows(const int32_t *tokens, int n, int type, const void *w, const float *q8s, int d,
                             float *out, cudaStream_t st) {
    if (n == 0) return OVF_OK;
    embed_rows_kernel<<<n, 256, 0, st>>>(tokens, type, (const uint8_t *)w, q8s, d, out);
    return cuda_status(cudaGetLastError(), "embed_rows");
}

// Greedy token of each logits row (TokenSampler.ArgMax: first index of the
// maximum), one CTA per row, with the decode LM head's ordering key.
__global__ void argmax_rows_kernel(const float *__restrict__ logits, int vocab, int32_t *__restrict__ out) {
    __shared__ unsigned long long red[32];
    const float *row = logits + (size_t)blockIdx.x * vocab;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const unsigned long long k = argmax_key(row[i], i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
        out[blockIdx.x] = (int32_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    }
}

ovf_status launch_argmax_rows(const float *logits, int rows, int vocab, int32_t *out, cudaStream_t st) {
    if (rows == 0) return OVF_OK;
    argmax_rows_kernel<<<rows, 1024, 0, st>>>(logits, vocab, out);
    return cuda_status(cudaGetLastError(), "argmax_rows");
}

// A session's step state after one token of a multi-session batch: the
// position advanced and the sampled token logged, as its own decode step
// with logits leaves them.
__global__ void batch_finish_kernel(DevStep *step, int cur, int next, const int32_t *token, int32_t *tokens_log) {
    step->cur_pos = cur;
    step->next_pos = next;
    step->token = *token;
    if (tokens_log) tokens_log[step->n_generated] = *token;
    step->n_generated += 1;
}

ovf_status launch_batch_finish(DevStep *step, int cur, int next, const int32_t *token, int32_t *tokens_log,
                               cudaStream_t st) {
    batch_finish_kernel<<<1, 1, 0, st>>>(step, cur, next, token, tokens_log);
    return cuda_status(cudaGetLastError(), "batch_finish");
}

// Positions after a batched prefill: the state n single-token steps leave.
__global__ void set_step_pos_kernel(DevStep *step, int cur, int next) {
    step->cur_pos = cur;
    step->next_pos = next;
}

ovf_status launch_set_step_pos(DevStep *step, int cur, int next, cudaStream_t st) {
    set_step_pos_kernel<<<1, 1, 0, st>>>(step, cur, next);
    return cuda_status(cudaGetLastError(), "set_step_pos");
}

// --------------------------------------------------------------- SiLU * up
// Runtime/CachedFeedForwardBlock.cs:464-472 + :309: h = (g*sigmoid(g))*u, for
// gate/up pairs that cannot share one GEMV launch.
__global__ void silu_mul_kernel(const float *g, const float *u, float *h, int64_t n) {
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float x = g[i];
        const float sg = fdiv(1.0f, fadd(1.0f, exp_libm(-x)));
        h[i] = fmul(fmul(x, sg), u[i]);
    }
    pdl_launch_dependents();
}

// Reads and clears the device error word in one atomic step, ordered on a
// stream after the work whose waits may have set it.
__global__ void take_error_kernel(int *out) { *out = atomicExch(&g_dev_error, 0); }

ovf_status launch_take_error(int *dev_slot, cudaStream_t st) {
    take_error_kernel<<<1, 1, 0, st>>>(dev_slot);
    return cuda_status(cudaGetLastError(), "take_error");
}

// MathF.Exp elementwise (exp_libm), for callers and tests of the exp itself.
__global__ void exp_kernel(const float *x, float *y, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = exp_libm(x[i]);
}

ovf_status launch_exp(const float *x, float *y, int64_t n, cudaStream_t st) {
    if (n == 0) return OVF_OK;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
    exp_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, y, n);
    return cuda_status(cudaGetLastError(), "exp");
}

ovf_status launch_silu_mul(const float *g, const float *u, float *h, int64_t n, cudaStream_t st, bool pdl) {
    cudaError_t e = launch_pdl(silu_mul_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, pdl, g, u, h, n);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "silu_mul");
}

}  // namespace ovf
