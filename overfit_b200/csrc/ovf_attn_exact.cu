// ovf_attn_exact.cu — decode attention over an F32 KV cache in the
// reference's exact operation order (Runtime/CachedAttentionKernel.cs:36-128,
// ComputeSingleHead), so its output is bit-identical to the reference's.
//
// The reference's order fixes three sequential chains per query head: the
// score dot (two 8-lane accumulators over 16-wide steps, :342-390), the sum
// of the exponentials over t, and, for every dimension d, the weighted sum
// of values over t.  The chains over t cannot be reassociated, so their
// latency (about 4 cycles per position) bounds the kernel; everything else
// is spread over a thread-block cluster per query head:
//   1. every CTA of the cluster scores a contiguous slice of the positions
//      (a half-warp per key: lane c runs the reference's accumulator c, the
//      8-lane fold is a fixed shuffle tree), keeping the scores in its
//      shared memory;
//   2. the cluster agrees on the maximum through distributed shared memory
//      (max is order-free), and each CTA exponentiates its slice;
//   3. every CTA walks all slices in position order to form sumExp (the
//      same chain, so the same value, in each CTA);
//   4. CTA r accumulates dimensions [r*hd/CL, (r+1)*hd/CL) over all
//      positions in order, reading the probabilities from the owners'
//      shared memory.
// The token being decoded is rotated (RoPE, Rope/RopeKernel.cs:46-93) and
// appended to the cache here (CachedSingleHeadAttention.cs:264-281); its
// own position is read from shared memory, never from the cache, so no CTA
// waits for the append.
#include <cooperative_groups.h>

#include "ovf_internal.cuh"

namespace ovf {

namespace cg = cooperative_groups;

static constexpr int kExactCluster = 8;     // CTAs per query head
static constexpr int kExactThreads = 128;

int64_t attn_exact_smem_bytes(int hd, int seq_len) {
    const int chunk = (seq_len + kExactCluster - 1) / kExactCluster;
    return (int64_t)(3 * hd + chunk + 8) * 4;
}

int attn_exact_max_seq(int hd) {
    // the per-CTA score slice lives in shared memory (up to ~200 KB)
    return (int)((200 * 1024 / 4 - 3 * hd - 8) * kExactCluster);
}

template <int HD>
__global__ void __cluster_dims__(kExactCluster, 1, 1) __launch_bounds__(kExactThreads)
    attention_exact_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float esm[];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int h = blockIdx.x / kExactCluster;
    const int G = p.H / p.KVH, g = h / G;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float *qs = esm, *kn = esm + HD, *vn = esm + 2 * HD, *red = esm + 3 * HD, *ex = esm + 3 * HD + 8;
    const float *kf = reinterpret_cast<const float *>(p.kc) + (size_t)g * p.max_ctx * HD;
    const float *vf = reinterpret_cast<const float *>(p.vc) + (size_t)g * p.max_ctx * HD;

    pdl_wait();
    const int pos = p.pos_dev ? *p.pos_dev : p.seq_len_host - 1;
    const int seq = pos + 1;
    const int chunk = (seq + kExactCluster - 1) / kExactCluster;
    const int t0 = min(seq, rank * chunk), t1 = min(seq, t0 + chunk);
    const bool has_new = p.k_new != nullptr;

    for (int i = tid; i < HD; i += kExactThreads) {
        qs[i] = p.q[(size_t)h * HD + i];
        if (has_new) {
            kn[i] = p.k_new[(size_t)g * HD + i];
            vn[i] = p.v_new[(size_t)g * HD + i];
        }
    }
    __syncthreads();
    if (p.rope_cos) {
        const float *c = p.rope_cos + (size_t)pos * (HD / 2), *s = p.rope_sin + (size_t)pos * (HD / 2);
        rope_rotate(qs, HD, c, s, p.split_half, tid, kExactThreads);
        if (has_new) rope_rotate(kn, HD, c, s, p.split_half, tid, kExactThreads);
        __syncthreads();
    }
    if (has_new && h % G == 0 && rank == 0) {
        float *kw = reinterpret_cast<float *>(p.kc) + ((size_t)g * p.max_ctx + pos) * HD;
        float *vw = reinterpret_cast<float *>(p.vc) + ((size_t)g * p.max_ctx + pos) * HD;
        for (int i = tid; i < HD; i += kExactThreads) {
            kw[i] = kn[i];
            vw[i] = vn[i];
        }
    }
    pdl_launch_dependents();

    // 1. scores of [t0, t1): half-warp per key, lane c = accumulator c
    const int c = lane & 15, hw = lane >> 4;
    float qreg[HD / 16];
#pragma unroll
    for (int i = 0; i < HD / 16; ++i) qreg[i] = qs[16 * i + c];
    float lmax = -INFINITY;
    constexpr int KPI = 2 * (kExactThreads / 32);  // keys per pass of the CTA
    for (int tb = t0; tb < t1; tb += 2 * KPI) {
        float acc[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int t = tb + u * KPI + 2 * warp + hw;
            const bool ok = t < t1;
            const float *kr = (has_new && t == pos) ? kn : kf + (size_t)(ok ? t : t0) * HD;
            float a = 0.0f;
#pragma unroll
            for (int i = 0; i < HD / 16; ++i) a = fadd(a, fmul(qreg[i], kr[16 * i + c]));
            acc[u] = a;
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int t = tb + u * KPI + 2 * warp + hw;
            // v[j] = acc0[j] + acc1[j], then ((v0+v1)+(v2+v3))+((v4+v5)+(v6+v7))
            float v = fadd(acc[u], __shfl_xor_sync(0xFFFFFFFFu, acc[u], 8));
            v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
            v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
            v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
            const float sc = fmul(v, p.scale);
            if (c == 0 && t < t1) {
                ex[t - t0] = sc;
                lmax = sc > lmax ? sc : lmax;
            }
        }
    }
    // 2. cluster-wide maximum
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xFFFFFFFFu, lmax, o));
    if (lane == 0) red[warp] = lmax;
    __syncthreads();
    if (tid == 0) {
        float m = red[0];
        for (int w = 1; w < kExactThreads / 32; ++w) m = fmaxf(m, red[w]);
        red[4] = m;
    }
    cluster.sync();
    float gmax = -INFINITY;
    for (int r = 0; r < kExactCluster; ++r) gmax = fmaxf(gmax, cluster.map_shared_rank(red, r)[4]);
    for (int t = t0 + tid; t < t1; t += kExactThreads) ex[t - t0] = exp_rn(fsub(ex[t - t0], gmax));
    cluster.sync();

    // 3. sumExp over t in order (every CTA forms the same chain)
    if (tid == 0) {
        float sum = 0.0f;
        for (int r = 0; r < kExactCluster; ++r) {
            const int a = min(seq, r * chunk), b = min(seq, a + chunk);
            const float *e = cluster.map_shared_rank(ex, r);
            int t = 0;
            for (; t + 8 <= b - a; t += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = e[t + j];
#pragma unroll
                for (int j = 0; j < 8; ++j) sum = fadd(sum, v[j]);
            }
            for (; t < b - a; ++t) sum = fadd(sum, e[t]);
        }
        red[5] = sum;
    }
    __syncthreads();
    const float sumExp = red[5];
    const bool bad = !(sumExp > 0.0f) || isinf(sumExp);
    const float invSum = bad ? 0.0f : fdiv(1.0f, sumExp);

    // 4. out[d] for this CTA's dimensions, over t in order
    constexpr int DPC = HD / kExactCluster;
    if (tid < DPC) {
        const int d = rank * DPC + tid;
        float acc = 0.0f;
        if (!bad) {
            for (int r = 0; r < kExactCluster; ++r) {
                const int a = min(seq, r * chunk), b = min(seq, a + chunk);
                const float *e = cluster.map_shared_rank(ex, r);
                int t = a;
                for (; t + 4 <= b; t += 4) {
                    float ev[4], vv[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        ev[j] = e[t + j - a];
                        vv[j] = (has_new && t + j == pos) ? vn[d] : vf[(size_t)(t + j) * HD + d];
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc = fadd(acc, fmul(fmul(ev[j], invSum), vv[j]));
                }
                for (; t < b; ++t) {
                    const float vv = (has_new && t == pos) ? vn[d] : vf[(size_t)t * HD + d];
                    acc = fadd(acc, fmul(fmul(e[t - a], invSum), vv));
                }
            }
        }
        p.out[(size_t)h * HD + d] = acc;
    }
    cluster.sync();  // no CTA leaves while another still reads its shared memory
}

bool attn_exact_supported(int hd) { return hd == 32 || hd == 64 || hd == 128 || hd == 256; }

ovf_status launch_attention_exact(const AttnParams &p, int seq_len_max, cudaStream_t st, bool pdl) {
    OVF_CHECK_ARG(attn_exact_supported(p.hd), "attention: head_dim %d unsupported (32, 64, 128 or 256)", p.hd);
    OVF_CHECK_ARG(p.H > 0 && p.KVH > 0 && p.H % p.KVH == 0, "attention: n_heads must be a multiple of n_kv_heads");
    OVF_CHECK_ARG(seq_len_max >= 1 && seq_len_max <= attn_exact_max_seq(p.hd),
                  "attention: sequence length %d outside [1, %d]", seq_len_max, attn_exact_max_seq(p.hd));
    const size_t smem = (size_t)attn_exact_smem_bytes(p.hd, seq_len_max);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.H * kExactCluster);
    cfg.blockDim = dim3(kExactThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaSuccess;
#define OVF_EXACT(HDV)                                                                                      \
    do {                                                                                                    \
        static bool attr_set = false;                                                                       \
        if (!attr_set && smem > 48 * 1024) {                                                                \
            e = cudaFuncSetAttribute(attention_exact_kernel<HDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                     (int)attn_exact_smem_bytes(HDV, attn_exact_max_seq(HDV)));             \
            attr_set = e == cudaSuccess;                                                                    \
        }                                                                                                   \
        if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, attention_exact_kernel<HDV>, p);                 \
    } while (0)
    switch (p.hd) {
        case 32: OVF_EXACT(32); break;
        case 64: OVF_EXACT(64); break;
        case 128: OVF_EXACT(128); break;
        default: OVF_EXACT(256); break;
    }
#undef OVF_EXACT
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "attention_exact_kernel launch");
}

}  // namespace ovf
