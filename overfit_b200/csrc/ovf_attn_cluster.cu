// ovf_attn_cluster.cu — single-token GQA attention for the decode step, one
// thread-block cluster per KV head.
//
// The split-K kernel in ovf_ops.cu merges its per-split softmax partials
// through global memory and an atomic ticket, which costs several dependent
// global round trips per launch (~20 us at any context length).  Here the
// NC CTAs of a cluster each own a contiguous slice of the sequence, stream
// their K/V rows through shared memory with 1-D bulk copies (the cache rows of
// one KV head are contiguous, so a tile of keys is one copy), keep an online
// softmax (running max, sum and weighted values, Runtime/
// CachedAttentionKernel.cs:36-128 restated as flash-decoding), and merge the
// partials of the cluster through distributed shared memory.  Nothing touches
// global memory but the query, the cache and the output.
//
// The CTA whose slice holds the current position also rotates the new key
// (RoPE at that position, Rope/RopeKernel.cs:46-93), appends key and value to
// the fp16 cache, and patches the freshly copied tile row in shared memory.
#include <cooperative_groups.h>

#include "ovf_internal.cuh"

namespace cg = cooperative_groups;

namespace ovf {

static constexpr int kCNC = 16;    // CTAs per cluster (non-portable size, allowed on B200)
static constexpr int kCThr = 512;  // threads per CTA
static constexpr int kCTK = 128;   // keys per tile
static constexpr int kCBuf = 2;    // tiles in flight

template <int GT, int HD>
__global__ void __launch_bounds__(kCThr) attention_cluster_kernel(const AttnParams p) {
    extern __shared__ __align__(128) uint8_t csm[];
    constexpr int G = GT, hd = HD;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int g = blockIdx.y;
    const int row = blockIdx.z;  // batched prefill: query row (position seq_len_host - 1 + row)
    // shared memory map (the mbarriers first: they need 8-byte alignment)
    uint64_t *bar = reinterpret_cast<uint64_t *>(csm);            // [kCBuf]
    __half *kt = reinterpret_cast<__half *>(csm + 128);         // [kCBuf][TK][hd]
    __half *vt = kt + kCBuf * kCTK * hd;                          // [kCBuf][TK][hd]
    float *qs = reinterpret_cast<float *>(vt + kCBuf * kCTK * hd);  // [G][hd]
    float *sc = qs + G * hd;                                      // [G][TK]
    float *st = sc + G * kCTK;                                    // m[G], l[G], alpha[G]
    float *po = st + 3 * G;                                       // [G][hd] partial (fold target)
    float *fold = po + G * hd;                                    // [G][hd] second key half
    float *knew = fold + G * hd;                                  // [hd]
    float *vnew = knew + hd;                                      // [hd]

    if (tid == 0) trace_mark(p.trace, TR_START);
    if (tid == 0 && p.pos_dev) {
        // The cache rows before this token do not depend on the previous
        // kernel: pull this CTA's keys and values into L2 while it finishes
        // (the position read here may still be the previous step's; it only
        // bounds the hint).
        const int sp = *(volatile const int *)p.pos_dev + 1;
        const int pr = (sp + kCNC - 1) / kCNC;
        const int a = min(sp, rank * pr), b = min(sp, a + pr);
        if (b > a) {
            L2Prefetch kv{};
            const size_t hb = (size_t)g * p.max_ctx * hd;
            kv.ptr[0] = p.kc + hb + (size_t)a * hd;
            kv.ptr[1] = p.vc + hb + (size_t)a * hd;
            kv.bytes[0] = kv.bytes[1] = (int64_t)(b - a) * hd * 2;
            kv.n = 2;
            prefetch_l2_slice(kv, 0, 1);
        }
    }
    pdl_wait();
    if (tid == 0) trace_mark(p.trace, TR_WAITED);
    const int pos = p.pos_dev ? *p.pos_dev : p.seq_len_host - 1 + row;
    const int seq = pos + 1;
    const int per = (seq + kCNC - 1) / kCNC;
    const int t0 = min(seq, rank * per), t1 = min(seq, t0 + per);
    const int nt = t1 - t0;
    const int ntiles = (nt + kCTK - 1) / kCTK;
    const size_t head = (size_t)g * p.max_ctx * hd;
    const uint64_t pol = l2_evict_first_policy();

    if (tid == 0) {
        for (int b = 0; b < kCBuf; ++b) mbar_init(&bar[b], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int tile, int buf) {
        const int a = t0 + tile * kCTK, n = min(kCTK, t1 - a);
        const uint32_t bytes = (uint32_t)n * hd * 2;
        mbar_arrive_expect_tx(&bar[buf], 2 * bytes);
        bulk_g2s(kt + (size_t)buf * kCTK * hd, p.kc + head + (size_t)a * hd, bytes, &bar[buf], pol);
        bulk_g2s(vt + (size_t)buf * kCTK * hd, p.vc + head + (size_t)a * hd, bytes, &bar[buf], pol);
    };
    if (tid == 0)
        for (int b = 0; b < kCBuf && b < ntiles; ++b) issue(b, b);
    for (int i = tid; i < G * hd; i += kCThr) qs[i] = p.q[(size_t)row * p.H * hd + (size_t)g * G * hd + i];
    const bool owns_new = p.k_new != nullptr && pos >= t0 && pos < t1;
    if (owns_new)
        for (int i = tid; i < hd; i += kCThr) {
            knew[i] = p.k_new[(size_t)g * hd + i];
            vnew[i] = p.v_new[(size_t)g * hd + i];
        }
    if (tid < G) {
        st[tid] = -INFINITY;
        st[G + tid] = 0.0f;
    }
    __syncthreads();
    pdl_launch_dependents();
    if (p.rope_cos) {
        const float *c = p.rope_cos + (size_t)pos * (hd / 2), *s = p.rope_sin + (size_t)pos * (hd / 2);
        for (int h = 0; h < G; ++h) rope_rotate(qs + h * hd, hd, c, s, p.split_half, tid, kCThr);
        if (owns_new) rope_rotate(knew, hd, c, s, p.split_half, tid, kCThr);
        __syncthreads();
    }
    if (owns_new) {
        for (int i = tid; i < hd; i += kCThr) {
            const __half kh = __float2half_rn(knew[i]), vh = __float2half_rn(vnew[i]);
            p.kc[head + (size_t)pos * hd + i] = kh;
            p.vc[head + (size_t)pos * hd + i] = vh;
            knew[i] = __half2float(kh);
            vnew[i] = __half2float(vh);
        }
    }

    // Weighted-value accumulators: thread = (key half, dimension pair).
    const int d2 = tid % (hd / 2), part = tid / (hd / 2);  // HD=128: 2 parts; HD=64: 4 parts
    constexpr int NPART = kCThr / (HD / 2);
    float o0[G], o1[G];
#pragma unroll
    for (int h = 0; h < G; ++h) o0[h] = o1[h] = 0.0f;

    bool failed = false;
    for (int tile = 0; tile < ntiles; ++tile) {
        const int buf = tile % kCBuf;
        const int a = t0 + tile * kCTK, n = min(kCTK, t1 - a);
        if (!mbar_wait_bounded(&bar[buf], (uint32_t)((tile / kCBuf) & 1))) {
            failed = true;
            break;
        }
        __half *K = kt + (size_t)buf * kCTK * hd, *V = vt + (size_t)buf * kCTK * hd;
        if (owns_new && pos >= a && pos < a + n) {
            for (int i = tid; i < hd; i += kCThr) {
                K[(size_t)(pos - a) * hd + i] = __float2half_rn(knew[i]);
                V[(size_t)(pos - a) * hd + i] = __float2half_rn(vnew[i]);
            }
            __syncthreads();
        }
        // scores: LPK lanes per key, each one 16-byte chunk (8 halves) of the
        // key row, so the lanes of a quarter-warp read 128 contiguous bytes
        // (no shared-memory bank conflicts); partial dots are reduced over
        // the LPK lanes.  (This path is within tolerance of the reference,
        // not bit-exact: fused multiply-adds.)
        {
            constexpr int LPK = HD / 8 < 32 ? HD / 8 : 32;
            constexpr int KPP = kCThr / LPK;  // keys per pass
            const int c16 = tid % LPK;
            for (int kb = 0; kb < n; kb += KPP) {
                const int t = kb + tid / LPK;
                const bool ok = t < n;
                float kv[8];
                const uint4 w = *reinterpret_cast<const uint4 *>(K + (size_t)(ok ? t : 0) * hd + 8 * c16);
                const __half2 *h2 = reinterpret_cast<const __half2 *>(&w);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(h2[j]);
                    kv[2 * j] = f.x;
                    kv[2 * j + 1] = f.y;
                }
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float4 qa = *reinterpret_cast<const float4 *>(qs + h * hd + 8 * c16);
                    const float4 qb = *reinterpret_cast<const float4 *>(qs + h * hd + 8 * c16 + 4);
                    float acc = qa.x * kv[0];
                    acc = fmaf(qa.y, kv[1], acc);
                    acc = fmaf(qa.z, kv[2], acc);
                    acc = fmaf(qa.w, kv[3], acc);
                    acc = fmaf(qb.x, kv[4], acc);
                    acc = fmaf(qb.y, kv[5], acc);
                    acc = fmaf(qb.z, kv[6], acc);
                    acc = fmaf(qb.w, kv[7], acc);
#pragma unroll
                    for (int o = 1; o < LPK; o <<= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
                    if (ok && c16 == 0) sc[h * kCTK + t] = acc * p.scale;
                }
            }
        }
        __syncthreads();
        // online softmax: warp per head
        for (int h = warp; h < G; h += kCThr / 32) {
            float m = -INFINITY;
            for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[h * kCTK + t]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
            const float mold = st[h];
            const float mnew = fmaxf(mold, m);
            float l = 0.0f;
            for (int t = lane; t < n; t += 32) {
                const float e = expf(fsub(sc[h * kCTK + t], mnew));
                sc[h * kCTK + t] = e;
                l = fadd(l, e);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) l = fadd(l, __shfl_xor_sync(0xFFFFFFFFu, l, o));
            if (lane == 0) {
                const float alpha = mold == -INFINITY ? 0.0f : expf(fsub(mold, mnew));
                st[h] = mnew;
                st[G + h] = fadd(fmul(st[G + h], alpha), l);
                st[2 * G + h] = alpha;
            }
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float al = st[2 * G + h];
            o0[h] = fmul(o0[h], al);
            o1[h] = fmul(o1[h], al);
        }
        for (int t = part; t < n; t += NPART) {
            const float2 v = __half22float2(reinterpret_cast<const __half2 *>(V + (size_t)t * hd)[d2]);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float pr = sc[h * kCTK + t];
                o0[h] = fmaf(pr, v.x, o0[h]);
                o1[h] = fmaf(pr, v.y, o1[h]);
            }
        }
        __syncthreads();  // tile buffers and scores are free again
        if (tid == 0 && tile + kCBuf < ntiles) {
            fence_proxy_async_smem();
            issue(tile + kCBuf, buf);
        }
    }
    (void)failed;
    // fold the key parts of each dimension pair into po
    for (int q = 0; q < NPART; ++q) {
        if (part == q) {
#pragma unroll
            for (int h = 0; h < G; ++h) {
                if (q == 0) {
                    po[h * hd + 2 * d2] = o0[h];
                    po[h * hd + 2 * d2 + 1] = o1[h];
                } else {
                    po[h * hd + 2 * d2] = fadd(po[h * hd + 2 * d2], o0[h]);
                    po[h * hd + 2 * d2 + 1] = fadd(po[h * hd + 2 * d2 + 1], o1[h]);
                }
            }
        }
        __syncthreads();
    }
    (void)fold;
    // merge the cluster's partials through distributed shared memory: every
    // rank copies all ranks' (max, sum) per head, then finalises its own
    // 1/kCNC of the outputs (16 independent remote loads per output)
    cluster.sync();
    float *stm = fold, *stl = fold + kCNC * G;  // [kCNC][G] each (fold is free here)
    for (int idx = tid; idx < kCNC * G; idx += kCThr) {
        const int r = idx / G, h = idx % G;
        const float *rst = cluster.map_shared_rank(st, r);
        stm[idx] = rst[h];
        stl[idx] = rst[G + h];
    }
    __syncthreads();
    {
        constexpr int PER = G * HD / kCNC;
        for (int i = rank * PER + tid; i < (rank + 1) * PER; i += kCThr) {
            const int h = i / hd;
            float pv[kCNC];
#pragma unroll
            for (int r = 0; r < kCNC; ++r) pv[r] = cluster.map_shared_rank(po, r)[i];
            float M = -INFINITY;
#pragma unroll
            for (int r = 0; r < kCNC; ++r)
                if (stl[r * G + h] > 0.0f) M = fmaxf(M, stm[r * G + h]);
            float L = 0.0f, acc = 0.0f;
#pragma unroll
            for (int r = 0; r < kCNC; ++r) {
                const float lr = stl[r * G + h];
                if (lr > 0.0f) {
                    const float w = expf(fsub(stm[r * G + h], M));
                    L = fadd(L, fmul(lr, w));
                    acc = fadd(acc, fmul(w, pv[r]));
                }
            }
            const bool ok = L > 0.0f && isfinite(L);
            p.out[(size_t)row * p.H * hd + (size_t)g * G * hd + i] = ok ? fdiv(acc, L) : 0.0f;
        }
    }
    cluster.sync();  // partners' shared memory must outlive the other ranks' reads
    if (tid == 0) trace_mark(p.trace, TR_END);
}

size_t attn_cluster_smem(int G, int hd) {
    return 128 + (size_t)2 * kCBuf * kCTK * hd * 2 +
           sizeof(float) * ((size_t)G * hd + G * kCTK + 3 * G + 2 * G * hd + 2 * hd);
}

template <int GT, int HD>
static cudaError_t launch_cluster_inst(const AttnParams &p, size_t smem, cudaStream_t st, bool pdl) {
    static PerDeviceOnce attr_once;
    const int dev = current_device();
    if (attr_once.pending(dev)) {
        cudaError_t e = cudaFuncSetAttribute(attention_cluster_kernel<GT, HD>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attention_cluster_kernel<GT, HD>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        attr_once.mark(dev);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCNC, p.KVH, p.rows > 1 ? p.rows : 1);
    cfg.blockDim = dim3(kCThr);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = kCNC;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    static const bool no_pdl = [] {
        const char *v = getenv("OVF_NO_PDL");
        return v && v[0] == '1';
    }();
    attrs[1].val.programmaticStreamSerializationAllowed = (pdl && !no_pdl) ? 1 : 0;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, attention_cluster_kernel<GT, HD>, p);
}

bool attn_cluster_supported(int G, int hd) {
    return (hd == 128 && (G == 1 || G == 2 || G == 4 || G == 8)) || (hd == 64 && (G == 1 || G == 2 || G == 4 || G == 7 || G == 8)) ||
           (hd == 32 && (G == 4 || G == 7));
}

ovf_status launch_attention_cluster(const AttnParams &p, cudaStream_t st, bool pdl) {
    const int G = p.H / p.KVH;
    OVF_CHECK_ARG(p.H % p.KVH == 0 && attn_cluster_supported(G, p.hd),
                  "attention (cluster): unsupported head layout %d/%d x %d", p.H, p.KVH, p.hd);
    const size_t smem = attn_cluster_smem(G, p.hd);
    cudaError_t e = cudaErrorInvalidValue;
#define OVF_CL(gt, hdv)                                              \
    if (G == gt && p.hd == hdv) e = launch_cluster_inst<gt, hdv>(p, smem, st, pdl);
    OVF_CL(1, 128) OVF_CL(2, 128) OVF_CL(4, 128) OVF_CL(8, 128)
    OVF_CL(1, 64) OVF_CL(2, 64) OVF_CL(4, 64) OVF_CL(7, 64) OVF_CL(8, 64)
    OVF_CL(4, 32) OVF_CL(7, 32)
#undef OVF_CL
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "attention_cluster_kernel launch");
}

}  // namespace ovf
