// ovf_ops.cu — decode attention (flash-decode, GQA, fused RoPE + KV append),
// RMSNorm, RoPE, embedding lookup and SiLU*up for sm_100a.
#include "ovf_internal.cuh"

#include <algorithm>

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

int attn_splits(int n_kv_heads) { return std::max(1, std::min(64, 296 / std::max(1, n_kv_heads))); }

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

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float asmem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = kAttnThreads / 32;
    const int split = blockIdx.x, g = blockIdx.y;
    const int G = p.H / p.KVH, hd = p.hd;
    float *qs = asmem;                       // [G][hd]
    float *knew = qs + G * hd;               // [hd]
    float *vnew = knew + hd;                 // [hd]
    float *sc = vnew + hd;                   // [G][chunk_max]
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

    // Scores: one warp per key, lanes over the head dimension.
    const int per_lane = hd / 32;
    for (int t = warp; t < nt; t += nw) {
        const int pt = t0 + t;
        float kv[8];
        if (owns_new && pt == pos) {
            for (int j = 0; j < per_lane; ++j) kv[j] = knew[lane * per_lane + j];
        } else {
            const __half *kr = p.kc + cache_head + (size_t)pt * hd + lane * per_lane;
            for (int j = 0; j < per_lane; ++j) kv[j] = __half2float(kr[j]);
        }
        for (int h = 0; h < G; ++h) {
            const float *qh = qs + h * hd + lane * per_lane;
            float acc = 0.0f;
            for (int j = 0; j < per_lane; ++j) acc = fadd(acc, fmul(qh[j], kv[j]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc = fadd(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, o));
            if (lane == 0) sc[h * p.chunk_max + t] = fmul(acc, p.scale);
        }
    }
    __syncthreads();
    // Per head: max, exp, sum (warp per head).
    float *mh = reinterpret_cast<float *>(&sc[G * p.chunk_max]);  // [G] max, [G] sum
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
    // Weighted values: thread per dimension, all heads of the group.
    for (int d = tid; d < hd; d += kAttnThreads) {
        float o[16];
        for (int h = 0; h < G; ++h) o[h] = 0.0f;
        for (int t = 0; t < nt; ++t) {
            const int pt = t0 + t;
            const float v = (owns_new && pt == pos) ? vnew[d] : __half2float(p.vc[cache_head + (size_t)pt * hd + d]);
            for (int h = 0; h < G; ++h) o[h] = fadd(o[h], fmul(sc[h * p.chunk_max + t], v));
        }
        for (int h = 0; h < G; ++h)
            p.partial[((size_t)(g * G + h) * p.n_splits + split) * (hd + 2) + d] = o[h];
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
    for (int h = 0; h < G; ++h) {
        const float *base = p.partial + (size_t)(g * G + h) * p.n_splits * (hd + 2);
        float M = -INFINITY;
        for (int s = 0; s < p.n_splits; ++s) {
            const float ls = __ldcg(base + (size_t)s * (hd + 2) + hd + 1);
            if (ls > 0.0f) M = fmaxf(M, __ldcg(base + (size_t)s * (hd + 2) + hd));
        }
        float L = 0.0f;
        for (int s = 0; s < p.n_splits; ++s) {
            const float ls = __ldcg(base + (size_t)s * (hd + 2) + hd + 1);
            if (ls > 0.0f) L = fadd(L, fmul(ls, expf(fsub(__ldcg(base + (size_t)s * (hd + 2) + hd), M))));
        }
        const bool ok = L > 0.0f && isfinite(L);
        const float inv = ok ? fdiv(1.0f, L) : 0.0f;
        for (int d = tid; d < hd; d += kAttnThreads) {
            float acc = 0.0f;
            for (int s = 0; s < p.n_splits; ++s) {
                const float ls = __ldcg(base + (size_t)s * (hd + 2) + hd + 1);
                if (ls > 0.0f) {
                    const float w = expf(fsub(__ldcg(base + (size_t)s * (hd + 2) + hd), M));
                    acc = fadd(acc, fmul(w, __ldcg(base + (size_t)s * (hd + 2) + d)));
                }
            }
            p.out[(size_t)(g * G + h) * hd + d] = ok ? fmul(acc, inv) : 0.0f;
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
    const size_t smem = sizeof(float) * ((size_t)G * p.hd + 2 * p.hd + (size_t)G * p.chunk_max + 2 * G);
    OVF_CHECK_ARG(smem <= 200 * 1024, "attention: context too long for one split's score buffer");
    static bool attr_done = false;
    if (!attr_done) {
        OVF_CUDA_TRY(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr_done = true;
    }
    cudaError_t e = launch_pdl(attention_kernel, dim3(p.n_splits, p.KVH), dim3(kAttnThreads), smem, st, pdl, p);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "attention_kernel launch");
}

// ------------------------------------------------------------------ RMSNorm
__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ gm, float *__restrict__ y,
                               int64_t d, float eps) {
    __shared__ float red[33];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float s = 0.0f;
    for (int64_t i = tid; i < d; i += blockDim.x) s = fadd(s, fmul(x[i], x[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = fadd(s, __shfl_xor_sync(0xFFFFFFFFu, s, o));
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float v = lane < nw ? red[lane] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
        if (lane == 0) red[32] = fdiv(1.0f, sqrtf(fadd(fdiv(v, (float)d), eps)));
    }
    __syncthreads();
    const float sc = red[32];
    for (int64_t i = tid; i < d; i += blockDim.x) y[i] = gm ? fmul(fmul(x[i], sc), gm[i]) : fmul(x[i], sc);
}

ovf_status launch_rmsnorm(const float *x, const float *g, float *y, int64_t d, float eps, cudaStream_t st) {
    rmsnorm_kernel<<<1, 1024, 0, st>>>(x, g, y, d, eps);
    return cuda_status(cudaGetLastError(), "rmsnorm");
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
// position.  Block 0 / thread 0 owns the position update.
__global__ void embed_kernel(DevStep *step, int type, const uint8_t *__restrict__ w, const float *__restrict__ q8s,
                             int d, float *__restrict__ hidden) {
    pdl_wait();
    const int token = step->token;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < d) {
        float v;
        if (type == OVF_TYPE_Q4_K) v = q4k_elem(w + ((int64_t)token * (d / 256) + i / 256) * 144, (int)(i % 256));
        else if (type == OVF_TYPE_Q6_K) v = q6k_elem(w + ((int64_t)token * (d / 256) + i / 256) * 210, (int)(i % 256));
        else if (type == OVF_TYPE_Q8_0)
            v = fmul(q8s[(int64_t)token * (d / 32) + i / 32], (float)reinterpret_cast<const int8_t *>(w)[(int64_t)token * d + i]);
        else v = reinterpret_cast<const float *>(w)[(int64_t)token * d + i];
        hidden[i] = v;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        step->cur_pos = step->next_pos;
        step->next_pos += 1;
    }
    pdl_launch_dependents();
}

ovf_status launch_embed(const DevStep *, int type, const void *w, const float *q8s, int d, float *hidden,
                        DevStep *step, cudaStream_t st, bool pdl) {
    cudaError_t e = launch_pdl(embed_kernel, dim3((d + 255) / 256), dim3(256), 0, st, pdl, step, type,
                               (const uint8_t *)w, q8s, d, hidden);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "embed");
}

// --------------------------------------------------------------- SiLU * up
// Runtime/CachedFeedForwardBlock.cs:464-472 + :309: h = (g*sigmoid(g))*u, for
// gate/up pairs that cannot share one GEMV launch.
__global__ void silu_mul_kernel(const float *g, const float *u, float *h, int64_t n) {
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float x = g[i];
        const float sg = fdiv(1.0f, fadd(1.0f, expf(-x)));
        h[i] = fmul(fmul(x, sg), u[i]);
    }
    pdl_launch_dependents();
}

ovf_status launch_silu_mul(const float *g, const float *u, float *h, int64_t n, cudaStream_t st, bool pdl) {
    cudaError_t e = launch_pdl(silu_mul_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, pdl, g, u, h, n);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "silu_mul");
}

}  // namespace ovf
