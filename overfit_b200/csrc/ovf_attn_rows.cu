// ovf_attn_rows.cu — causal attention of a prefill chunk (the batched
// prefill's BatchedAttentionKernel, Runtime/BatchedAttentionKernel.cs:34-214),
// every row at its own position, in ComputeSingleHead's exact operation
// order (Runtime/CachedAttentionKernel.cs:36-128) on F32 and fp16 caches.
//
// A single decode token has only G query heads of sequential chains to run,
// so its kernel spreads one row's work over a cluster; a prompt chunk has
// M rows x H heads of independent chains, so here every chain gets its own
// thread and the rows run side by side:
//   1. one CTA per (row, head): RoPE of the query, the row's scores (one
//      thread per key, the reference's two-accumulator dot and lane fold),
//      the maximum, the exponentials, the sumExp chain (one thread, in
//      position order) and p_t = e_t * invSum, written to a scratch row;
//   2. one CTA per (row, head), one thread per dimension: out[d] =
//      sum_t p_t * v_t[d] in position order (v reads coalesced over d, p
//      broadcast).
// The keys and values of the chunk are appended beforehand
// (kv_append_rows), so every row reads its whole causal window from the cache.
#include "ovf_internal.cuh"

namespace ovf {

static constexpr int kRowsThreads = 256;

// 16 consecutive cache elements of a row (fp32 or fp16), widened to fp32.
template <bool F16>
__device__ __forceinline__ void load16(const void *src, float *dst) {
    if (F16) {
        const uint4 a = reinterpret_cast<const uint4 *>(src)[0], b = reinterpret_cast<const uint4 *>(src)[1];
        const __half2 *h = reinterpret_cast<const __half2 *>(&a);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            dst[2 * i] = f.x;
            dst[2 * i + 1] = f.y;
        }
        h = reinterpret_cast<const __half2 *>(&b);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            dst[8 + 2 * i] = f.x;
            dst[8 + 2 * i + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 v = reinterpret_cast<const float4 *>(src)[i];
            dst[4 * i] = v.x;
            dst[4 * i + 1] = v.y;
            dst[4 * i + 2] = v.z;
            dst[4 * i + 3] = v.w;
        }
    }
}

template <int HD, int KT>
__global__ void __launch_bounds__(kRowsThreads) attn_rows_scores_kernel(const AttnParams p, float *__restrict__ P,
                                                                        int pos0) {
    constexpr bool F16 = KT == OVF_KV_F16;
    constexpr int EB = F16 ? 2 : 4;
    extern __shared__ __align__(16) float rsm[];
    float *qs = rsm;               // [HD]
    float *red = qs + HD;          // [64]
    unsigned long long *etab = reinterpret_cast<unsigned long long *>(red + 64);  // [32]
    float *e = red + 128;          // [max_ctx] scores, then exponentials
    const int row = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.H / p.KVH, g = h / G;
    const int pos = pos0 + row, seq = pos + 1;
    if (tid < 32) etab[tid] = kExp2Tab32[tid];
    for (int i = tid; i < HD; i += kRowsThreads) qs[i] = p.q[((size_t)row * p.H + h) * HD + i];
    __syncthreads();
    if (p.rope_cos) {
        rope_rotate(qs, HD, p.rope_cos + (size_t)pos * (HD / 2), p.rope_sin + (size_t)pos * (HD / 2), p.split_half,
                    tid, kRowsThreads);
        __syncthreads();
    }
    const char *kb = reinterpret_cast<const char *>(p.kc) + (size_t)g * p.max_ctx * HD * EB;
    float lmax = -INFINITY;
    for (int t = tid; t < seq; t += kRowsThreads) {
        // the reference's Dot: lane j of two 8-wide accumulators over
        // 16-wide steps, then ((v0+v1)+(v2+v3))+((v4+v5)+(v6+v7))
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
        const char *kr = kb + (size_t)t * HD * EB;
#pragma unroll 2
        for (int i = 0; i < HD / 16; ++i) {
            float k[16];
            load16<F16>(kr + (size_t)16 * i * EB, k);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = fadd(acc[j], fmul(qs[16 * i + j], k[j]));
        }
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = fadd(acc[j], acc[j + 8]);
        const float dot = fadd(fadd(fadd(v[0], v[1]), fadd(v[2], v[3])), fadd(fadd(v[4], v[5]), fadd(v[6], v[7])));
        const float s = fmul(dot, p.scale);
        e[t] = s;
        lmax = s > lmax ? s : lmax;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xFFFFFFFFu, lmax, o));
    if (lane == 0) red[warp] = lmax;
    __syncthreads();
    float m = red[0];
    for (int w = 1; w < kRowsThreads / 32; ++w) m = fmaxf(m, red[w]);
    for (int t = tid; t < seq; t += kRowsThreads) e[t] = exp_libm(fsub(e[t], m), etab);
    __syncthreads();
    if (tid == 0) {
        // sumExp in position order, 32 exponentials in registers ahead
        float sum = 0.0f;
        const int s32 = seq & ~31;
        int t = 0;
        if (s32 > 0) {
            float4 a[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) a[j] = reinterpret_cast<const float4 *>(e)[j];
            for (; t < s32; t += 32) {
                float4 b[8];
                const int tn = t + 32 < s32 ? t + 32 : t;
#pragma unroll
                for (int j = 0; j < 8; ++j) b[j] = reinterpret_cast<const float4 *>(e + tn)[j];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    sum = fadd(sum, a[j].x);
                    sum = fadd(sum, a[j].y);
                    sum = fadd(sum, a[j].z);
                    sum = fadd(sum, a[j].w);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) a[j] = b[j];
            }
        }
        for (; t < seq; ++t) sum = fadd(sum, e[t]);
        const bool bad = !(sum > 0.0f) || isinf(sum);
        red[32] = bad ? 0.0f : fdiv(1.0f, sum);
        red[33] = bad ? 1.0f : 0.0f;
    }
    __syncthreads();
    const float inv = red[32];
    const bool bad = red[33] != 0.0f;
    float *pr = P + ((size_t)row * p.H + h) * p.max_ctx;
    // an empty or non-finite sum gives a zero output (all p_t = 0)
    for (int t = tid; t < seq; t += kRowsThreads) pr[t] = bad ? 0.0f : fmul(e[t], inv);
}

template <int HD, int KT>
__global__ void __launch_bounds__(HD) attn_rows_out_kernel(const AttnParams p, const float *__restrict__ P, int pos0) {
    constexpr bool F16 = KT == OVF_KV_F16;
    const int row = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const int G = p.H / p.KVH, g = h / G;
    const int seq = pos0 + row + 1;
    const float *pr = P + ((size_t)row * p.H + h) * p.max_ctx;
    float acc = 0.0f;
    int t = 0;
    if (F16) {
        const __half *vb = p.vc + (size_t)g * p.max_ctx * HD + d;
        for (; t + 8 <= seq; t += 8) {
            float pv[8], vv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                pv[j] = __ldg(pr + t + j);
                vv[j] = __half2float(vb[(size_t)(t + j) * HD]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) acc = fadd(acc, fmul(pv[j], vv[j]));
        }
        for (; t < seq; ++t) acc = fadd(acc, fmul(__ldg(pr + t), __half2float(vb[(size_t)t * HD])));
    } else {
        const float *vb = reinterpret_cast<const float *>(p.vc) + (size_t)g * p.max_ctx * HD + d;
        for (; t + 8 <= seq; t += 8) {
            float pv[8], vv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                pv[j] = __ldg(pr + t + j);
                vv[j] = vb[(size_t)(t + j) * HD];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) acc = fadd(acc, fmul(pv[j], vv[j]));
        }
        for (; t < seq; ++t) acc = fadd(acc, fmul(__ldg(pr + t), vb[(size_t)t * HD]));
    }
    p.out[((size_t)row * p.H + h) * HD + d] = acc;
}

bool attn_rows_supported(int hd, int kv_dtype) {
    return (kv_dtype == OVF_KV_F32 || kv_dtype == OVF_KV_F16) && (hd == 32 || hd == 64 || hd == 128 || hd == 256);
}

int64_t attn_rows_scratch_floats(int rows, int H, int max_ctx) { return (int64_t)rows * H * max_ctx; }

// Rows [0, p.rows) at positions pos0 .. pos0 + rows - 1; P holds
// attn_rows_scratch_floats(rows, H, max_ctx) floats.
ovf_status launch_attention_rows(const AttnParams &p, int pos0, float *P, cudaStream_t st, int kv_dtype) {
    OVF_CHECK_ARG(attn_rows_supported(p.hd, kv_dtype), "attention rows: unsupported head_dim / cache type");
    OVF_CHECK_ARG(p.rows >= 1 && p.rows <= 65535 && pos0 >= 0 && pos0 + p.rows <= p.max_ctx, "attention rows: range");
    const size_t smem = (size_t)(p.hd + 128 + p.max_ctx) * 4;
    OVF_CHECK_ARG(smem <= (size_t)smem_optin(current_device()), "attention rows: context too long");
    const dim3 grid((unsigned)p.rows, (unsigned)p.H);
    const bool f16 = kv_dtype == OVF_KV_F16;
    cudaError_t e = cudaSuccess;
#define OVF_ROWS(HDV)                                                                                         \
    do {                                                                                                       \
        auto ks = f16 ? attn_rows_scores_kernel<HDV, OVF_KV_F16> : attn_rows_scores_kernel<HDV, OVF_KV_F32>;   \
        auto ko = f16 ? attn_rows_out_kernel<HDV, OVF_KV_F16> : attn_rows_out_kernel<HDV, OVF_KV_F32>;         \
        if (smem > 48 * 1024) e = cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        if (e == cudaSuccess) {                                                                                \
            ks<<<grid, kRowsThreads, smem, st>>>(p, P, pos0);                                                  \
            e = cudaGetLastError();                                                                            \
        }                                                                                                      \
        if (e == cudaSuccess) {                                                                                \
            ko<<<grid, HDV, 0, st>>>(p, P, pos0);                                                              \
            e = cudaGetLastError();                                                                            \
        }                                                                                                      \
    } while (0)
    switch (p.hd) {
        case 32: OVF_ROWS(32); break;
        case 64: OVF_ROWS(64); break;
        case 128: OVF_ROWS(128); break;
        default: OVF_ROWS(256); break;
    }
#undef OVF_ROWS
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "attention rows launch");
}

}  // namespace ovf
