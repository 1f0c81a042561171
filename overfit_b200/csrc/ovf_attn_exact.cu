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
static constexpr int kExactThreads = 256;
static constexpr int kExactMaxSeq = 16384;  // the whole probability vector sits in each CTA's shared memory
static constexpr int kVBlock = 128;         // positions per staged value block
static constexpr int kVRow = kVBlock + 4;   // one dimension's values of a block, padded (16-byte rows)
static constexpr int kVBufs = 8;            // value blocks in flight (hd <= 128; 4 for hd 256)
template <int HD>
struct VStage {
    static constexpr int bufs = HD <= 128 ? kVBufs : kVBufs / 2;
};

// shared memory: q, k_new, v_new [hd each] | 16 scalars | quantized new
// K/V row (Q8 cache, 2 x hd bytes) | value blocks
// [kVBufs][kVBlock][hd/CL] | own score slice [chunk] | all probabilities [seq]
int64_t attn_exact_smem_bytes(int hd, int seq_len) {
    const int chunk = (seq_len + kExactCluster - 1) / kExactCluster;
    const int dpc = hd / kExactCluster;
    const int bufs = hd <= 128 ? kVBufs : kVBufs / 2;
    return (int64_t)(3 * hd + 16 + hd / 2 + bufs * kVRow * dpc + chunk + ((seq_len + 3) & ~3)) * 4 + 16;
}


int attn_exact_max_seq(int) { return kExactMaxSeq; }

// KT = OVF_KV_Q8: the reference's Q8 KV cache (KvCacheDType.Q8, per-vector
// int8 + one fp32 scale, Runtime/Q8KvQuant.cs) attended in
// ComputeSingleHeadQ8's order (Runtime/CachedAttentionKernel.cs:139-235):
// score = DotF32I8(q, kQ) * keyScale * scale, out[d] += (p * invSum *
// valueScale) * vQ[d].  KT = OVF_KV_F16: the cache holds K/V rounded to fp16
// (half the bytes of F32) and every value read widens exactly to fp32, so the
// arithmetic is ComputeSingleHead's on the rounded cache.
template <int HD, int KT>
__global__ void __cluster_dims__(kExactCluster, 1, 1) __launch_bounds__(kExactThreads)
    attention_exact_kernel(const AttnParams p) {
    constexpr bool Q8 = KT == OVF_KV_Q8, F16 = KT == OVF_KV_F16, RAW = Q8 || F16;
    extern __shared__ __align__(16) float esm[];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int h = blockIdx.x / kExactCluster;
    const int row = blockIdx.y;  // batched prefill: query row (position seq_len_host - 1 + row)
    const int G = p.H / p.KVH, g = h / G;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int DPC = HD / kExactCluster;
    float *qs = esm, *kn = esm + HD, *vn = esm + 2 * HD, *red = esm + 3 * HD;
    int8_t *kq8n = reinterpret_cast<int8_t *>(esm + 3 * HD + 16), *vq8n = kq8n + HD;  // Q8: the new row
    float *vbuf = esm + 3 * HD + 16 + HD / 2;           // [kVBufs][kVBlock][DPC]
    constexpr int NBUF = VStage<HD>::bufs;
    float *ex = vbuf + NBUF * kVRow * DPC;              // own slice of scores / exponentials
    const float *kf = reinterpret_cast<const float *>(p.kc) + (size_t)g * p.max_ctx * HD;
    const float *vf = reinterpret_cast<const float *>(p.vc) + (size_t)g * p.max_ctx * HD;
    const int8_t *k8 = reinterpret_cast<const int8_t *>(p.kc) + (size_t)g * p.max_ctx * HD;
    const int8_t *v8 = reinterpret_cast<const int8_t *>(p.vc) + (size_t)g * p.max_ctx * HD;
    const __half *k16 = p.kc + (size_t)g * p.max_ctx * HD;
    const __half *v16 = p.vc + (size_t)g * p.max_ctx * HD;
    const float *ksc = Q8 ? p.ks + (size_t)g * p.max_ctx : nullptr;
    const float *vsc = Q8 ? p.vs + (size_t)g * p.max_ctx : nullptr;
    constexpr int EB = Q8 ? 1 : F16 ? 2 : 4;  // bytes per cached element

    // the next projections' weights do not depend on this kernel: pull them
    // into L2 while the (latency-bound) attention runs
    if (tid == 0) trace_mark(p.trace, TR_START);
    if (tid == 0 && p.pf.n) prefetch_l2_slice(p.pf, blockIdx.x, gridDim.x);
    if (tid == 0 && p.pos_dev && !p.no_kv_prefetch) {
        // The cache rows before this token do not depend on the previous
        // kernel: pull this CTA's key slice and a slice of the value rows
        // into L2 now.  The position read here may still be the previous
        // step's (the bound only matters for the hint); the real one is
        // read after griddepcontrol.wait.
        const int sp = *(volatile const int *)p.pos_dev + 1;
        const int ch = (sp + kExactCluster - 1) / kExactCluster;
        const int a = min(sp, rank * ch), b = min(sp, a + ch);
        L2Prefetch kv{};
        if (b > a) {
            kv.ptr[0] = reinterpret_cast<const char *>(p.kc) + ((size_t)g * p.max_ctx + a) * HD * EB;
            kv.bytes[0] = (int64_t)(b - a) * HD * EB;
            kv.ptr[1] = reinterpret_cast<const char *>(p.vc) + ((size_t)g * p.max_ctx + a) * HD * EB;
            kv.bytes[1] = (int64_t)(b - a) * HD * EB;
            kv.n = 2;
            prefetch_l2_slice(kv, 0, 1);
        }
    }
    pdl_wait();
    if (tid == 0) trace_mark(p.trace, TR_WAITED);
    const int pos = p.pos_dev ? *p.pos_dev : p.seq_len_host - 1 + row;
    const int seq = pos + 1;
    const int chunk = (seq + kExactCluster - 1) / kExactCluster;
    const int t0 = min(seq, rank * chunk), t1 = min(seq, t0 + chunk);
    const bool has_new = p.k_new != nullptr;
    const int d0 = rank * DPC;
    const int nblk = (seq + kVBlock - 1) / kVBlock;
    // value block b -> vbuf[b % kVBufs] with 16-byte asynchronous copies
    // (the row at `pos` is replaced from v_new when it is used)
    // block b is stored transposed, [DPC][kVRow]: dimension d's values of
    // the block are contiguous for its chain thread (4-byte copies; the
    // global reads stay coalesced along d)
    // (Q8: raw int8 rows [kVBlock][DPC], 4-byte pieces)
    constexpr int NE = kVBlock * DPC / kExactThreads;
    constexpr int NE8 = (kVBlock * DPC * EB / 4 + kExactThreads - 1) / kExactThreads;
    auto stage_values = [&](int blk) {
        if (blk < nblk) {
            float *dst = vbuf + (blk % NBUF) * kVRow * DPC;
            const int tb = blk * kVBlock, n = min(kVBlock, seq - tb);
            if (RAW) {
                // raw rows [kVBlock][DPC] of EB-byte elements, 4-byte pieces
                constexpr int PPR = DPC * EB / 4;  // pieces per row
                char *d8 = reinterpret_cast<char *>(dst);
                const char *src = Q8 ? reinterpret_cast<const char *>(v8) : reinterpret_cast<const char *>(v16);
#pragma unroll
                for (int j = 0; j < NE8; ++j) {
                    const int i = tid + j * kExactThreads, t = i / PPR, q4 = i % PPR;
                    if (i < kVBlock * PPR && t < n)
                        cp_async4(d8 + (t * DPC) * EB + 4 * q4, src + ((size_t)(tb + t) * HD + d0) * EB + 4 * q4);
                }
            } else {
#pragma unroll
                for (int j = 0; j < NE; ++j) {
                    const int i = tid + j * kExactThreads, t = i / DPC, dd = i % DPC;
                    if (t < n) cp_async4(dst + dd * kVRow + t, vf + (size_t)(tb + t) * HD + d0 + dd);
                }
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int b = 0; b < NBUF; ++b) stage_values(b);

    for (int i = tid; i < HD; i += kExactThreads) {
        qs[i] = p.q[((size_t)row * p.H + h) * HD + i];
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
    if (F16 && has_new) {
        // the cache keeps the rotated key and the value rounded to fp16; the
        // current token is attended from the same rounded values
        for (int i = tid; i < HD; i += kExactThreads) {
            kn[i] = __half2float(__float2half_rn(kn[i]));
            vn[i] = __half2float(__float2half_rn(vn[i]));
        }
        __syncthreads();
    }
    if (Q8 && has_new) {
        // Q8KvQuant.Quantize of the rotated key and the value (every CTA
        // computes the same bytes; the current token is attended from them)
        if (warp == 0) {
            float mk = 0.0f, mv = 0.0f;
            for (int i = lane; i < HD; i += 32) {
                mk = fmaxf(mk, fabsf(kn[i]));
                mv = fmaxf(mv, fabsf(vn[i]));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                mk = fmaxf(mk, __shfl_xor_sync(0xFFFFFFFFu, mk, o));
                mv = fmaxf(mv, __shfl_xor_sync(0xFFFFFFFFu, mv, o));
            }
            if (lane == 0) {
                red[10] = mk > 0.0f ? fdiv(mk, 127.0f) : 0.0f;
                red[11] = mv > 0.0f ? fdiv(mv, 127.0f) : 0.0f;
                red[12] = mk > 0.0f ? fdiv(127.0f, mk) : 0.0f;
                red[13] = mv > 0.0f ? fdiv(127.0f, mv) : 0.0f;
            }
        }
        __syncthreads();
        for (int i = tid; i < HD; i += kExactThreads) {
            kq8n[i] = (int8_t)quant_elem(kn[i], red[12]);
            vq8n[i] = (int8_t)quant_elem(vn[i], red[13]);
        }
        __syncthreads();
    }
    if (has_new && h % G == 0 && rank == 0) {
        if (Q8) {
            int8_t *kw = reinterpret_cast<int8_t *>(p.kc) + ((size_t)g * p.max_ctx + pos) * HD;
            int8_t *vw = reinterpret_cast<int8_t *>(p.vc) + ((size_t)g * p.max_ctx + pos) * HD;
            for (int i = tid; i < HD; i += kExactThreads) {
                kw[i] = kq8n[i];
                vw[i] = vq8n[i];
            }
            if (tid == 0) {
                p.ks[(size_t)g * p.max_ctx + pos] = red[10];
                p.vs[(size_t)g * p.max_ctx + pos] = red[11];
            }
        } else if (F16) {
            __half *kw = p.kc + ((size_t)g * p.max_ctx + pos) * HD;
            __half *vw = p.vc + ((size_t)g * p.max_ctx + pos) * HD;
            for (int i = tid; i < HD; i += kExactThreads) {
                kw[i] = __float2half_rn(kn[i]);
                vw[i] = __float2half_rn(vn[i]);
            }
        } else {
            float *kw = reinterpret_cast<float *>(p.kc) + ((size_t)g * p.max_ctx + pos) * HD;
            float *vw = reinterpret_cast<float *>(p.vc) + ((size_t)g * p.max_ctx + pos) * HD;
            for (int i = tid; i < HD; i += kExactThreads) {
                kw[i] = kn[i];
                vw[i] = vn[i];
            }
        }
    }
    pdl_launch_dependents();

    // 1. scores of [t0, t1): half-warp per key, lane c = accumulator c
    const int c = lane & 15, hw = lane >> 4;
    float qreg[HD / 16];
#pragma unroll
    for (int i = 0; i < HD / 16; ++i) qreg[i] = qs[16 * i + c];
    float lmax = -INFINITY;
    constexpr int KPI = 2 * (kExactThreads / 32);  // keys per step of the CTA (a half-warp each)
    constexpr int U = HD <= 128 ? 8 : 4;            // keys per half-warp in flight
    for (int tb = t0; tb < t1; tb += U * KPI) {
        float kv[U][HD / 16];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + u * KPI + 2 * warp + hw;
            const bool ok = t < t1;
            if (Q8) {
                const int8_t *kr = (has_new && t == pos) ? kq8n : k8 + (size_t)(ok ? t : t0) * HD;
#pragma unroll
                for (int i = 0; i < HD / 16; ++i) kv[u][i] = (float)kr[16 * i + c];
            } else if (F16) {
                if (has_new && t == pos) {
#pragma unroll
                    for (int i = 0; i < HD / 16; ++i) kv[u][i] = kn[16 * i + c];
                } else {
                    const __half *kr = k16 + (size_t)(ok ? t : t0) * HD;
#pragma unroll
                    for (int i = 0; i < HD / 16; ++i) kv[u][i] = __half2float(kr[16 * i + c]);
                }
            } else {
                const float *kr = (has_new && t == pos) ? kn : kf + (size_t)(ok ? t : t0) * HD;
#pragma unroll
                for (int i = 0; i < HD / 16; ++i) kv[u][i] = kr[16 * i + c];
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + u * KPI + 2 * warp + hw;
            float a = 0.0f;
#pragma unroll
            for (int i = 0; i < HD / 16; ++i) a = fadd(a, fmul(qreg[i], kv[u][i]));
            // v[j] = acc0[j] + acc1[j], then ((v0+v1)+(v2+v3))+((v4+v5)+(v6+v7))
            float v = fadd(a, __shfl_xor_sync(0xFFFFFFFFu, a, 8));
            v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
            v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
            v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
            float sc;
            if (Q8) {
                const float kscale = (has_new && t == pos) ? red[10] : (t < t1 ? ksc[t] : 0.0f);
                sc = fmul(fmul(v, kscale), p.scale);
            } else {
                sc = fmul(v, p.scale);
            }
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
        red[8] = m;
    }
    cluster.sync();
    float gmax = -INFINITY;
    for (int r = 0; r < kExactCluster; ++r) gmax = fmaxf(gmax, cluster.map_shared_rank(red, r)[8]);
    for (int t = t0 + tid; t < t1; t += kExactThreads) ex[t - t0] = exp_libm(fsub(ex[t - t0], gmax));
    cluster.sync();

    // 3. every CTA gathers all probabilities' numerators into its own shared
    //    memory, then thread 0 forms sumExp over t in order (the same chain,
    //    so the same value, in every CTA)
    float *eall = ex + chunk;  // [seq], 16-byte aligned below
    eall = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(eall) + 15) & ~uintptr_t(15));
    {
        // all slices at once: eight remote loads in flight per thread
        constexpr int GU = 8;
        for (int base = 0; base < seq; base += GU * kExactThreads) {
            float tmp[GU];
#pragma unroll
            for (int j = 0; j < GU; ++j) {
                const int t = base + j * kExactThreads + tid;
                const int r = t < seq ? t / chunk : 0;
                tmp[j] = t < seq ? cluster.map_shared_rank(ex, r)[t - r * chunk] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < GU; ++j) {
                const int t = base + j * kExactThreads + tid;
                if (t < seq) eall[t] = tmp[j];
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
        const int s64 = seq & ~63;
        const float4 *e4 = reinterpret_cast<const float4 *>(eall);
        for (int i = 0; i < s64; i += 64) {
            float4 a[8], b[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) a[j] = e4[i / 4 + j];
#pragma unroll
            for (int j = 0; j < 8; ++j) b[j] = e4[i / 4 + 8 + j];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                sum = fadd(sum, a[j].x);
                sum = fadd(sum, a[j].y);
                sum = fadd(sum, a[j].z);
                sum = fadd(sum, a[j].w);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                sum = fadd(sum, b[j].x);
                sum = fadd(sum, b[j].y);
                sum = fadd(sum, b[j].z);
                sum = fadd(sum, b[j].w);
            }
        }
        const int s32 = s64;
        for (int t = s32; t < seq; ++t) sum = fadd(sum, eall[t]);
        red[9] = sum;
    }
    __syncthreads();
    const float sumExp = red[9];
    const bool bad = !(sumExp > 0.0f) || isinf(sumExp);
    const float invSum = bad ? 0.0f : fdiv(1.0f, sumExp);

    // 4. out[d] for this CTA's dimensions over t in order; the values are
    //    staged block by block in shared memory by all threads while the
    //    DPC chain threads consume the previous block
    // p_t = e_t * invSum once, by all threads (the reference's probability)
    // (Q8: coef_t = p_t * invSum * valueScale_t, the reference's AxpyI8 factor)
    if (!bad)
        for (int t = tid; t < seq; t += kExactThreads) {
            float pr = fmul(eall[t], invSum);
            if (Q8) pr = fmul(pr, (has_new && t == pos) ? red[11] : vsc[t]);
            eall[t] = pr;
        }
    float acc = 0.0f;
    for (int blk = 0; blk < nblk; ++blk) {
        cp_async_wait<NBUF - 1>();  // block blk has landed (this thread's part)
        __syncthreads();
        if (F16 && tid < DPC && !bad) {
            __half *vb16 = reinterpret_cast<__half *>(vbuf + (blk % NBUF) * kVRow * DPC) + tid;
            const int tb = blk * kVBlock, n = min(kVBlock, seq - tb);
            if (has_new && pos >= tb && pos < tb + n) vb16[(pos - tb) * DPC] = __float2half_rn(vn[d0 + tid]);
            const float *pb = eall + tb;
            int i = 0;
#pragma unroll 1
            for (; i + 16 <= n; i += 16) {
                float pv[16], vv[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    pv[j] = pb[i + j];
                    vv[j] = __half2float(vb16[(i + j) * DPC]);
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) acc = fadd(acc, fmul(pv[j], vv[j]));
            }
            for (; i < n; ++i) acc = fadd(acc, fmul(pb[i], __half2float(vb16[i * DPC])));
        }
        if (Q8 && tid < DPC && !bad) {
            int8_t *vb8 = reinterpret_cast<int8_t *>(vbuf + (blk % NBUF) * kVRow * DPC) + tid;
            const int tb = blk * kVBlock, n = min(kVBlock, seq - tb);
            if (has_new && pos >= tb && pos < tb + n) vb8[(pos - tb) * DPC] = vq8n[d0 + tid];
            const float *pb = eall + tb;
            int i = 0;
#pragma unroll 1
            for (; i + 16 <= n; i += 16) {
                float pv[16], vv[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    pv[j] = pb[i + j];
                    vv[j] = (float)vb8[(i + j) * DPC];
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) acc = fadd(acc, fmul(pv[j], vv[j]));
            }
            for (; i < n; ++i) acc = fadd(acc, fmul(pb[i], (float)vb8[i * DPC]));
        }
        if (!RAW && tid < DPC && !bad) {
            float *vb = vbuf + (blk % NBUF) * kVRow * DPC + tid * kVRow;
            const int tb = blk * kVBlock, n = min(kVBlock, seq - tb);
            // the current token's value was not in the cache when staged
            if (has_new && pos >= tb && pos < tb + n) vb[pos - tb] = vn[d0 + tid];
            const float *pb = eall + tb;
            int i = 0;
            // 32 values and probabilities in registers ahead of the adds
#pragma unroll 1
            for (; i + 32 <= n; i += 32) {
                float4 pv[8], vv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    pv[j] = *reinterpret_cast<const float4 *>(pb + i + 4 * j);
                    vv[j] = *reinterpret_cast<const float4 *>(vb + i + 4 * j);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    acc = fadd(acc, fmul(pv[j].x, vv[j].x));
                    acc = fadd(acc, fmul(pv[j].y, vv[j].y));
                    acc = fadd(acc, fmul(pv[j].z, vv[j].z));
                    acc = fadd(acc, fmul(pv[j].w, vv[j].w));
                }
            }
            for (; i < n; ++i) acc = fadd(acc, fmul(pb[i], vb[i]));
        }
        __syncthreads();
        stage_values(blk + NBUF);  // into the buffer just consumed
    }
    cp_async_wait<0>();
    if (tid < DPC) p.out[((size_t)row * p.H + h) * HD + d0 + tid] = acc;
    cluster.sync();  // no CTA leaves while another may still read its shared memory
    if (tid == 0) trace_mark(p.trace, TR_END);
}

// One CTA per (row, KV head): the key rotated with RoPE at the row's
// position and, with the value, stored as the attention kernels store the
// token they decode — fp32, fp16 (round to nearest) or Q8KvQuant (absmax/127
// per vector, the same ops as attention_exact_kernel's Q8 append).
template <int HD>
__global__ void kv_append_rows_kernel(const AttnParams p, const float *__restrict__ k, const float *__restrict__ v,
                                      int pos0, int kv_dtype) {
    __shared__ float kn[HD], vn[HD];
    __shared__ float sc[4];
    const int row = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    const int pos = pos0 + row;
    const size_t src = ((size_t)row * p.KVH + g) * HD;
    for (int i = tid; i < HD; i += blockDim.x) {
        kn[i] = k[src + i];
        vn[i] = v[src + i];
    }
    __syncthreads();
    if (p.rope_cos) {
        rope_rotate(kn, HD, p.rope_cos + (size_t)pos * (HD / 2), p.rope_sin + (size_t)pos * (HD / 2), p.split_half,
                    tid, blockDim.x);
        __syncthreads();
    }
    const size_t dst = ((size_t)g * p.max_ctx + pos) * HD;
    if (kv_dtype == OVF_KV_F32) {
        float *kw = reinterpret_cast<float *>(p.kc) + dst, *vw = reinterpret_cast<float *>(p.vc) + dst;
        for (int i = tid; i < HD; i += blockDim.x) {
            kw[i] = kn[i];
            vw[i] = vn[i];
        }
    } else if (kv_dtype == OVF_KV_F16) {
        for (int i = tid; i < HD; i += blockDim.x) {
            p.kc[dst + i] = __float2half_rn(kn[i]);
            p.vc[dst + i] = __float2half_rn(vn[i]);
        }
    } else {
        if (tid < 32) {
            float mk = 0.0f, mv = 0.0f;
            for (int i = lane; i < HD; i += 32) {
                mk = fmaxf(mk, fabsf(kn[i]));
                mv = fmaxf(mv, fabsf(vn[i]));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                mk = fmaxf(mk, __shfl_xor_sync(0xFFFFFFFFu, mk, o));
                mv = fmaxf(mv, __shfl_xor_sync(0xFFFFFFFFu, mv, o));
            }
            if (lane == 0) {
                sc[0] = mk > 0.0f ? fdiv(mk, 127.0f) : 0.0f;
                sc[1] = mv > 0.0f ? fdiv(mv, 127.0f) : 0.0f;
                sc[2] = mk > 0.0f ? fdiv(127.0f, mk) : 0.0f;
                sc[3] = mv > 0.0f ? fdiv(127.0f, mv) : 0.0f;
            }
        }
        __syncthreads();
        int8_t *kw = reinterpret_cast<int8_t *>(p.kc) + dst, *vw = reinterpret_cast<int8_t *>(p.vc) + dst;
        for (int i = tid; i < HD; i += blockDim.x) {
            kw[i] = (int8_t)quant_elem(kn[i], sc[2]);
            vw[i] = (int8_t)quant_elem(vn[i], sc[3]);
        }
        if (tid == 0) {
            p.ks[(size_t)g * p.max_ctx + pos] = sc[0];
            p.vs[(size_t)g * p.max_ctx + pos] = sc[1];
        }
    }
}

ovf_status launch_kv_append_rows(const AttnParams &p, const float *k, const float *v, int rows, int pos0, int kv_dtype,
                                 cudaStream_t st) {
    if (rows == 0) return OVF_OK;
    OVF_CHECK_ARG(rows <= 65535 && pos0 >= 0 && pos0 + rows <= p.max_ctx, "kv append: rows out of range");
    OVF_CHECK_ARG(kv_dtype != OVF_KV_Q8 || (p.ks && p.vs), "kv append: Q8 cache without its scales");
    const dim3 grid((unsigned)rows, (unsigned)p.KVH);
    switch (p.hd) {
        case 32: kv_append_rows_kernel<32><<<grid, 64, 0, st>>>(p, k, v, pos0, kv_dtype); break;
        case 64: kv_append_rows_kernel<64><<<grid, 64, 0, st>>>(p, k, v, pos0, kv_dtype); break;
        case 128: kv_append_rows_kernel<128><<<grid, 64, 0, st>>>(p, k, v, pos0, kv_dtype); break;
        case 256: kv_append_rows_kernel<256><<<grid, 128, 0, st>>>(p, k, v, pos0, kv_dtype); break;
        default: OVF_CHECK_ARG(false, "kv append: head_dim %d unsupported", p.hd);
    }
    return cuda_status(cudaGetLastError(), "kv_append_rows");
}

// OVF_ATTN_NO_GROUP=1 keeps every launch on the per-head kernel (same
// results; for comparisons).
static bool getenv_flag_cached_no_group() {
    static const bool v = [] {
        const char *e = getenv("OVF_ATTN_NO_GROUP");
        return e && e[0] == '1';
    }();
    return v;
}

bool attn_exact_supported(int hd) { return hd == 32 || hd == 64 || hd == 128 || hd == 256; }

ovf_status launch_attention_exact(const AttnParams &p, int seq_len_max, cudaStream_t st, bool pdl, int kv_dtype) {
    const bool q8 = kv_dtype == OVF_KV_Q8;
    OVF_CHECK_ARG(kv_dtype == OVF_KV_F32 || q8 || kv_dtype == OVF_KV_F16, "attention: unknown KV type %d", kv_dtype);
    OVF_CHECK_ARG(attn_exact_supported(p.hd), "attention: head_dim %d unsupported (32, 64, 128 or 256)", p.hd);
    OVF_CHECK_ARG(p.H > 0 && p.KVH > 0 && p.H % p.KVH == 0, "attention: n_heads must be a multiple of n_kv_heads");
    OVF_CHECK_ARG(!q8 || (p.ks && p.vs), "attention: Q8 cache without its scales");
    OVF_CHECK_ARG(seq_len_max >= 1 && seq_len_max <= attn_exact_max_seq(p.hd),
                  "attention: sequence length %d outside [1, %d]", seq_len_max, attn_exact_max_seq(p.hd));
    if (!getenv_flag_cached_no_group() &&
        attn_group_supported(p.H, p.KVH, p.hd, kv_dtype, seq_len_max, smem_optin(current_device())))
        return launch_attention_group(p, seq_len_max, st, pdl, kv_dtype);
    const size_t smem = (size_t)attn_exact_smem_bytes(p.hd, seq_len_max);
    cudaLaunchConfig_t cfg = {};
    OVF_CHECK_ARG(p.rows <= 1 || (p.k_new == nullptr && !p.pos_dev && p.rows <= 65535), "attention: bad row batch");
    cfg.gridDim = dim3(p.H * kExactCluster, p.rows > 1 ? p.rows : 1);
    cfg.blockDim = dim3(kExactThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaSuccess;
#define OVF_EXACT(HDV, Q)                                                                                      \
    do {                                                                                                       \
        static PerDeviceOnce attr_once;                                                                        \
        const int dev_ = current_device();                                                                     \
        if (smem > 48 * 1024 && attr_once.pending(dev_)) {                                                     \
            e = cudaFuncSetAttribute(attention_exact_kernel<HDV, Q>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                     (int)attn_exact_smem_bytes(HDV, attn_exact_max_seq(HDV)));                \
            if (e == cudaSuccess) attr_once.mark(dev_);                                                        \
        }                                                                                                      \
        if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, attention_exact_kernel<HDV, Q>, p);                 \
    } while (0)
    switch (p.hd) {
#define OVF_EXACT_KT(HDV)                                                                                      \
    do {                                                                                                       \
        if (kv_dtype == OVF_KV_Q8) OVF_EXACT(HDV, OVF_KV_Q8);                                                  \
        else if (kv_dtype == OVF_KV_F16) OVF_EXACT(HDV, OVF_KV_F16);                                           \
        else OVF_EXACT(HDV, OVF_KV_F32);                                                                       \
    } while (0)
        case 32: OVF_EXACT_KT(32); break;
        case 64: OVF_EXACT_KT(64); break;
        case 128: OVF_EXACT_KT(128); break;
        default: OVF_EXACT_KT(256); break;
    }
#undef OVF_EXACT_KT
#undef OVF_EXACT
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "attention_exact_kernel launch");
}

}  // namespace ovf
