// ovf_attn_group.cu — decode attention in the reference's exact operation
// order (Runtime/CachedAttentionKernel.cs:36-128, ComputeSingleHead) with one
// thread-block cluster per KV head: the F32 and fp16 caches of sessions whose
// context fits the cluster's shared memory.
//
// The reference's order fixes, per query head, two sequential fp32 chains
// over the positions t: sumExp = sum e_t, and for every dimension d,
// out[d] = sum (e_t * invSum) * v_t[d].  Their latency (one dependent add,
// about 4 cycles, per position) is the kernel's floor; the layout is built
// around running them back to back with nothing else in the way:
//   1. the 16 CTAs of the cluster each score a contiguous slice of the
//      positions for all G query heads of the KV head (every key is read once
//      per cluster; a half-warp per key, lane c holding the reference's
//      accumulator lane c, the 8-lane fold a fixed shuffle tree);
//   2. per-head maxima are agreed through distributed shared memory and each
//      CTA exponentiates its slice;
//   3. every CTA copies all heads' exponentials into its own shared memory
//      (16-byte remote loads), then G lanes of warp 0 run the G sumExp chains
//      while the other seven warps stage this CTA's value columns
//      [d0, d0 + HD/16) of every position, transposed and widened to fp32;
//   4. after the probabilities p_t = e_t * invSum are formed, G * HD/16 lanes
//      run the output chains with 16-byte loads of p and v, no barrier
//      inside the chain.
// The decoded token is rotated (Rope/RopeKernel.cs:46-93) and appended
// (CachedSingleHeadAttention.cs:264-281) here; its own position is attended
// from shared memory, never from the cache, so no CTA waits for the append.
#include <cooperative_groups.h>

#include "ovf_internal.cuh"

namespace ovf {

namespace gcg = cooperative_groups;

static constexpr int kGrpCluster = 16;
static constexpr int kGrpThreads = 256;
static constexpr int kGrpMaxHeads = 8;  // query heads per KV head held in registers while scoring

struct GroupLayout {
    int chunk_cap, sp_cap;  // per-CTA slice capacity and padded sequence capacity (multiples of 4)
    int64_t floats;
};

__host__ __device__ inline GroupLayout group_layout(int G, int hd, int seq_cap) {
    GroupLayout L;
    L.chunk_cap = (((seq_cap + kGrpCluster - 1) / kGrpCluster) + 3) & ~3;
    L.sp_cap = (seq_cap + 3) & ~3;
    const int dpc = hd / kGrpCluster;
    L.floats = (int64_t)G * hd + 2 * hd + 128 + (int64_t)G * L.chunk_cap + (int64_t)G * L.sp_cap + (int64_t)dpc * L.sp_cap;
    return L;
}

// DPC consecutive cache elements of one row, widened to fp32.
template <int DPC, bool F16>
__device__ __forceinline__ void load_cols(const void *src, float *dst) {
    if (F16) {
        const __half *h = static_cast<const __half *>(src);
        if (DPC == 8) {
            const uint4 u = *reinterpret_cast<const uint4 *>(h);
            const __half2 *p2 = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(p2[i]);
                dst[2 * i] = f.x;
                dst[2 * i + 1] = f.y;
            }
        } else if (DPC == 4) {
            const uint2 u = *reinterpret_cast<const uint2 *>(h);
            const __half2 *p2 = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float2 f = __half22float2(p2[i]);
                dst[2 * i] = f.x;
                dst[2 * i + 1] = f.y;
            }
        } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(h));
            dst[0] = f.x;
            dst[1] = f.y;
        }
    } else {
        const float *f = static_cast<const float *>(src);
        if (DPC == 8) {
            const float4 a = *reinterpret_cast<const float4 *>(f), b = *reinterpret_cast<const float4 *>(f + 4);
            dst[0] = a.x; dst[1] = a.y; dst[2] = a.z; dst[3] = a.w;
            dst[4] = b.x; dst[5] = b.y; dst[6] = b.z; dst[7] = b.w;
        } else if (DPC == 4) {
            const float4 a = *reinterpret_cast<const float4 *>(f);
            dst[0] = a.x; dst[1] = a.y; dst[2] = a.z; dst[3] = a.w;
        } else {
            const float2 a = *reinterpret_cast<const float2 *>(f);
            dst[0] = a.x;
            dst[1] = a.y;
        }
    }
}

template <int HD, int KT>
__global__ void __launch_bounds__(kGrpThreads) attention_group_kernel(const AttnParams p, int seq_cap) {
    constexpr bool F16 = KT == OVF_KV_F16;
    constexpr int CL = kGrpCluster, DPC = HD / CL, NT = kGrpThreads, EB = F16 ? 2 : 4;
    extern __shared__ __align__(16) float gsm[];
    gcg::cluster_group cluster = gcg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int g = blockIdx.x / CL, row = blockIdx.y;
    const int G = p.H / p.KVH;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const GroupLayout GL = group_layout(G, HD, seq_cap);
    const int cc = GL.chunk_cap, spc = GL.sp_cap;
    float *qs = gsm;               // [G][HD]
    float *kn = qs + G * HD;       // [HD] current key (rotated)
    float *vn = kn + HD;           // [HD] current value
    float *red = vn + HD;          // [128]: warp maxima [8][8] | local max [64..72) | max [96..104) | inv [80..88) | bad [88..96)
    float *sc = red + 128;         // [G][cc] own slice: scores, then exponentials
    float *eall = sc + G * cc;     // [G][spc] all exponentials, then probabilities
    float *vt = eall + G * spc;    // [DPC][spc] this CTA's value columns, transposed
    const char *kbase = reinterpret_cast<const char *>(p.kc) + (size_t)g * p.max_ctx * HD * EB;
    const char *vbase = reinterpret_cast<const char *>(p.vc) + (size_t)g * p.max_ctx * HD * EB;
    const int d0 = rank * DPC;

    if (tid == 0) trace_mark(p.trace, TR_START);
    if (tid == 0 && p.pf.n) prefetch_l2_slice(p.pf, blockIdx.x, gridDim.x);
    if (tid == 0 && p.pos_dev && !p.no_kv_prefetch) {
        // the cache rows before this token do not depend on the previous
        // kernel: pull this CTA's key slice into L2 now (the position read
        // here may be the previous step's; it only bounds the hint)
        const int sp = *(volatile const int *)p.pos_dev + 1;
        const int ch = (((sp + CL - 1) / CL) + 3) & ~3;
        const int a = min(sp, rank * ch), b = min(sp, a + ch);
        if (b > a) {
            L2Prefetch kv{};
            kv.ptr[0] = kbase + (size_t)a * HD * EB;
            kv.bytes[0] = (int64_t)(b - a) * HD * EB;
            kv.n = 1;
            prefetch_l2_slice(kv, 0, 1);
        }
    }
    pdl_wait();
    if (tid == 0) trace_mark(p.trace, TR_WAITED);
    const int pos = p.pos_dev ? *p.pos_dev : p.seq_len_host - 1 + row;
    const int seq = pos + 1;
    const int chunk = (((seq + CL - 1) / CL) + 3) & ~3;
    const int t0 = min(seq, rank * chunk), t1 = min(seq, t0 + chunk);
    const bool has_new = p.k_new != nullptr;

    for (int i = tid; i < G * HD; i += NT) qs[i] = p.q[((size_t)row * p.H + (size_t)g * G) * HD + i];
    if (has_new)
        for (int i = tid; i < HD; i += NT) {
            kn[i] = p.k_new[(size_t)g * HD + i];
            vn[i] = p.v_new[(size_t)g * HD + i];
        }
    __syncthreads();
    if (p.rope_cos) {
        const float *c = p.rope_cos + (size_t)pos * (HD / 2), *s = p.rope_sin + (size_t)pos * (HD / 2);
        for (int h = 0; h < G; ++h) rope_rotate(qs + h * HD, HD, c, s, p.split_half, tid, NT);
        if (has_new) rope_rotate(kn, HD, c, s, p.split_half, tid, NT);
        __syncthreads();
    }
    if (F16 && has_new) {
        // the cache keeps the rotated key and the value rounded to fp16; the
        // current token is attended from the same rounded values
        for (int i = tid; i < HD; i += NT) {
            kn[i] = __half2float(__float2half_rn(kn[i]));
            vn[i] = __half2float(__float2half_rn(vn[i]));
        }
        __syncthreads();
    }
    if (has_new && rank == 0) {
        if (F16) {
            __half *kw = p.kc + ((size_t)g * p.max_ctx + pos) * HD, *vw = p.vc + ((size_t)g * p.max_ctx + pos) * HD;
            for (int i = tid; i < HD; i += NT) {
                kw[i] = __float2half_rn(kn[i]);
                vw[i] = __float2half_rn(vn[i]);
            }
        } else {
            float *kw = reinterpret_cast<float *>(p.kc) + ((size_t)g * p.max_ctx + pos) * HD;
            float *vw = reinterpret_cast<float *>(p.vc) + ((size_t)g * p.max_ctx + pos) * HD;
            for (int i = tid; i < HD; i += NT) {
                kw[i] = kn[i];
                vw[i] = vn[i];
            }
        }
    }
    pdl_launch_dependents();

    // 1. scores of [t0, t1) for every head of the group
    const int c = lane & 15, hw = lane >> 4;
    float qreg[kGrpMaxHeads][HD / 16];
#pragma unroll
    for (int h = 0; h < kGrpMaxHeads; ++h)
#pragma unroll
        for (int i = 0; i < HD / 16; ++i) qreg[h][i] = h < G ? qs[h * HD + 16 * i + c] : 0.0f;
    float lmax[kGrpMaxHeads];
#pragma unroll
    for (int h = 0; h < kGrpMaxHeads; ++h) lmax[h] = -INFINITY;
    constexpr int KPI = 2 * (NT / 32);  // keys per step (a half-warp each)
    constexpr int U = 4;                // keys per half-warp in flight
    for (int tb = t0; tb < t1; tb += U * KPI) {
        float kv[U][HD / 16];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + u * KPI + 2 * warp + hw;
            const int tt = t < t1 ? t : t0;
            if (has_new && tt == pos) {
#pragma unroll
                for (int i = 0; i < HD / 16; ++i) kv[u][i] = kn[16 * i + c];
            } else if (F16) {
                const __half *kr = reinterpret_cast<const __half *>(kbase) + (size_t)tt * HD;
#pragma unroll
                for (int i = 0; i < HD / 16; ++i) kv[u][i] = __half2float(kr[16 * i + c]);
            } else {
                const float *kr = reinterpret_cast<const float *>(kbase) + (size_t)tt * HD;
#pragma unroll
                for (int i = 0; i < HD / 16; ++i) kv[u][i] = kr[16 * i + c];
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + u * KPI + 2 * warp + hw;
#pragma unroll
            for (int h = 0; h < kGrpMaxHeads; ++h) {
                if (h < G) {
                    float a = 0.0f;
#pragma unroll
                    for (int i = 0; i < HD / 16; ++i) a = fadd(a, fmul(qreg[h][i], kv[u][i]));
                    // v[j] = acc0[j] + acc1[j], then ((v0+v1)+(v2+v3))+((v4+v5)+(v6+v7))
                    float v = fadd(a, __shfl_xor_sync(0xFFFFFFFFu, a, 8));
                    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
                    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
                    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
                    const float s = fmul(v, p.scale);
                    if (c == 0 && t < t1) {
                        sc[h * cc + (t - t0)] = s;
                        lmax[h] = s > lmax[h] ? s : lmax[h];
                    }
                }
            }
        }
    }
    // 2. per-head maxima over the cluster (max is order-free)
#pragma unroll
    for (int h = 0; h < kGrpMaxHeads; ++h) {
        float m = lmax[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        if (lane == 0) red[warp * 8 + h] = m;
    }
    __syncthreads();
    if (tid < G) {
        float m = red[tid];
        for (int w = 1; w < NT / 32; ++w) m = fmaxf(m, red[w * 8 + tid]);
        red[64 + tid] = m;
    }
    cluster.sync();
    if (tid < G) {
        float m = -INFINITY;
        for (int r = 0; r < CL; ++r) m = fmaxf(m, cluster.map_shared_rank(red, r)[64 + tid]);
        red[96 + tid] = m;
    }
    __syncthreads();
    const int own = t1 - t0;
    for (int i = tid; i < G * own; i += NT) {
        const int h = i / own, t = i - h * own;
        sc[h * cc + t] = exp_libm(fsub(sc[h * cc + t], red[96 + h]));
    }
    cluster.sync();

    // 3. all heads' exponentials into this CTA, 16 bytes per remote load
    const int nq = (seq + 3) >> 2;
    for (int base = 0; base < G * nq; base += 4 * NT) {
        float4 tmp[4];
        int dst[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = base + j * NT + tid;
            dst[j] = -1;
            if (i < G * nq) {
                const int h = i / nq, t = 4 * (i - h * nq), r = t / chunk;
                tmp[j] = *reinterpret_cast<const float4 *>(cluster.map_shared_rank(sc, r) + h * cc + (t - r * chunk));
                dst[j] = h * spc + t;
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (dst[j] >= 0) *reinterpret_cast<float4 *>(eall + dst[j]) = tmp[j];
    }
    __syncthreads();

    if (warp == 0) {
        // sumExp chains, one lane per head, in position order
        if (lane < G) {
            const float *e = eall + lane * spc;
            float sum = 0.0f;
            int t = 0;
            const int s32 = seq & ~31;
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
            red[80 + lane] = bad ? 0.0f : fdiv(1.0f, sum);
            red[88 + lane] = bad ? 1.0f : 0.0f;
        }
    } else {
        // meanwhile: this CTA's value columns [d0, d0 + DPC), transposed to
        // vt[d][t] and widened to fp32
        for (int t = tid - 32; t < seq; t += NT - 32) {
            float v[DPC];
            if (has_new && t == pos) {
#pragma unroll
                for (int d = 0; d < DPC; ++d) v[d] = vn[d0 + d];
            } else {
                load_cols<DPC, F16>(vbase + ((size_t)t * HD + d0) * EB, v);
            }
#pragma unroll
            for (int d = 0; d < DPC; ++d) vt[d * spc + t] = v[d];
        }
    }
    __syncthreads();
    // p_t = e_t * invSum (the reference's probability), all threads
    for (int i = tid; i < G * nq * 4; i += NT) {
        const int h = i / (nq * 4), t = i - h * nq * 4;
        if (t < seq) eall[h * spc + t] = fmul(eall[h * spc + t], red[80 + h]);
    }
    __syncthreads();

    // 4. output chains: lane (h, d) sums p_t * v_t[d] over t in order
    if (tid < G * DPC) {
        const int h = tid / DPC, d = tid - h * DPC;
        float acc = 0.0f;
        if (red[88 + h] == 0.0f) {
            const float *pp = eall + h * spc, *vv = vt + d * spc;
            const int s16 = seq & ~15;
            int t = 0;
            if (s16 > 0) {
                float4 pa[4], va[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    pa[j] = reinterpret_cast<const float4 *>(pp)[j];
                    va[j] = reinterpret_cast<const float4 *>(vv)[j];
                }
                for (; t < s16; t += 16) {
                    float4 pb[4], vb[4];
                    const int tn = t + 16 < s16 ? t + 16 : t;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        pb[j] = reinterpret_cast<const float4 *>(pp + tn)[j];
                        vb[j] = reinterpret_cast<const float4 *>(vv + tn)[j];
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc = fadd(acc, fmul(pa[j].x, va[j].x));
                        acc = fadd(acc, fmul(pa[j].y, va[j].y));
                        acc = fadd(acc, fmul(pa[j].z, va[j].z));
                        acc = fadd(acc, fmul(pa[j].w, va[j].w));
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        pa[j] = pb[j];
                        va[j] = vb[j];
                    }
                }
            }
            for (; t < seq; ++t) acc = fadd(acc, fmul(pp[t], vv[t]));
        }
        p.out[((size_t)row * p.H + (size_t)g * G + h) * HD + d0 + d] = acc;
    }
    cluster.sync();  // no CTA leaves while another may still read its shared memory
    if (tid == 0) trace_mark(p.trace, TR_END);
}

// Whether the group kernel takes this launch; otherwise the per-head exact
// kernel (ovf_attn_exact.cu) does.
bool attn_group_supported(int H, int KVH, int hd, int kv_dtype, int seq_cap, int smem_optin_bytes) {
    if (kv_dtype != OVF_KV_F32 && kv_dtype != OVF_KV_F16) return false;
    if (hd != 32 && hd != 64 && hd != 128) return false;
    if (KVH <= 0 || H % KVH != 0) return false;
    const int G = H / KVH;
    if (G > kGrpMaxHeads || G * (hd / kGrpCluster) > kGrpThreads) return false;
    return group_layout(G, hd, seq_cap).floats * 4 <= smem_optin_bytes;
}

template <int HD, int KT>
static cudaError_t launch_group_inst(const AttnParams &p, int seq_cap, size_t smem, cudaStream_t st, bool pdl) {
    static PerDeviceOnce attr_once;
    const int dev = current_device();
    if (attr_once.pending(dev)) {
        cudaError_t e = cudaFuncSetAttribute(attention_group_kernel<HD, KT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin(dev));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attention_group_kernel<HD, KT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        attr_once.mark(dev);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.KVH * kGrpCluster, p.rows > 1 ? p.rows : 1);
    cfg.blockDim = dim3(kGrpThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = kGrpCluster;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, attention_group_kernel<HD, KT>, p, seq_cap);
}

ovf_status launch_attention_group(const AttnParams &p, int seq_cap, cudaStream_t st, bool pdl, int kv_dtype) {
    const int G = p.H / p.KVH;
    const size_t smem = (size_t)group_layout(G, p.hd, seq_cap).floats * 4;
    OVF_CHECK_ARG(p.rows <= 1 || (p.k_new == nullptr && !p.pos_dev && p.rows <= 65535), "attention: bad row batch");
    cudaError_t e = cudaErrorInvalidValue;
    const bool f16 = kv_dtype == OVF_KV_F16;
    switch (p.hd) {
        case 32: e = f16 ? launch_group_inst<32, OVF_KV_F16>(p, seq_cap, smem, st, pdl)
                         : launch_group_inst<32, OVF_KV_F32>(p, seq_cap, smem, st, pdl); break;
        case 64: e = f16 ? launch_group_inst<64, OVF_KV_F16>(p, seq_cap, smem, st, pdl)
                         : launch_group_inst<64, OVF_KV_F32>(p, seq_cap, smem, st, pdl); break;
        case 128: e = f16 ? launch_group_inst<128, OVF_KV_F16>(p, seq_cap, smem, st, pdl)
                          : launch_group_inst<128, OVF_KV_F32>(p, seq_cap, smem, st, pdl); break;
        default: break;
    }
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "attention_group_kernel launch");
}

}  // namespace ovf
