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
//      (bulk copies between the cluster's CTAs), then G lanes of warp 0 run
//      the G sumExp chains; this CTA's value columns [d0, d0 + HD/16) of
//      every position are staged transposed (fp32 cache: [d][t] read from the
//      cache; fp16 cache: copied early as [t][d] in 16-position blocks, each
//      block transposed in place, so the fp16 layout costs 32 bytes per
//      position and two CTAs share an SM up to ~3.5K positions);
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

#ifdef OVF_PHASE_PROBE
__device__ unsigned long long g_phase[16];
#define OVF_PHASE(i) \
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) g_phase[i] = clock64()
}  // namespace ovf
// Probe builds only: the last launch's phase clocks of CTA (0, 0).
extern "C" __attribute__((visibility("default"))) int ovf_debug_attn_phases(unsigned long long *out) {
    return (int)cudaMemcpyFromSymbol(out, ovf::g_phase, sizeof(ovf::g_phase));
}
namespace ovf {
#else
#define OVF_PHASE(i)
#endif

static constexpr int kGrpCluster = 16;
static constexpr int kGrpThreads = 256;

struct GroupLayout {
    int chunk_cap, sp_cap;  // per-CTA slice capacity and padded row stride (floats)
    int64_t o_sc, o_eall, o_reg2, o_vraw, floats;  // offsets (floats) and total
};

// Shared memory (floats): qs [G][hd] | kn, vn [hd] | red [264] | exp table
// [64] | sc [G][chunk] | eall [G][sp] | then, fp32 cache: the key rows
// [chunk][hd] while scoring, then vt [hd/16][sp]; fp16 cache: the value
// columns in 16-position blocks (keys are scored from L2).  For Llama-3-8B
// heads the fp16 layout is ~32 bytes per position, so two CTAs fit an SM
// (and a 16-CTA cluster packs into a GPC) up to ~3.5K positions.
__host__ __device__ inline GroupLayout group_layout(int G, int hd, int seq_cap, int eb) {
    GroupLayout L;
    L.chunk_cap = (((seq_cap + kGrpCluster - 1) / kGrpCluster) + 3) & ~3;
    // rows of the [heads][t] and [d][t] arrays start 4 banks apart (stride
    // = 4 mod 32 floats), so lanes reading 8 rows at one t with 16-byte loads
    // hit 32 distinct banks
    L.sp_cap = (((seq_cap + 3) & ~3) + 31) / 32 * 32 + 4;
    const int dpc = hd / kGrpCluster;
    L.o_sc = (int64_t)G * hd + 2 * hd + 264 + 64;
    L.o_eall = L.o_sc + (int64_t)G * L.chunk_cap;
    L.o_reg2 = L.o_eall + (int64_t)G * L.sp_cap;
    if (eb == 2) {
        // fp16 cache: keys are scored straight from global memory (L2); the
        // value columns land in 16-position blocks [t][dpc] and each block is
        // transposed in place to [dpc][16] — 32 bytes per position in all
        L.o_vraw = L.o_reg2;
        L.floats = L.o_reg2 + (int64_t)((seq_cap + 15) / 16) * 16 * dpc * 2 / 4;
    } else {
        const int64_t kraw = ((int64_t)L.chunk_cap * hd * eb / 4 + 3) & ~int64_t(3);
        const int64_t vt = (int64_t)dpc * L.sp_cap * eb / 4;
        L.o_vraw = L.o_reg2 + (kraw > vt ? kraw : vt);
        L.floats = L.o_vraw;
    }
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

// Rotation of row d of an fp16 value block (see the transposition).
__device__ __forceinline__ int vrot(int d) { return ((d >> 2) & 1) * 8; }

// Async copy of n (4, 8 or a multiple of 16) bytes, 16 at a time.
__device__ __forceinline__ void cp_async_n(char *dst, const char *src, int n) {
    if (n >= 16) {
        for (int o = 0; o < n; o += 16) cp_async16(dst + o, src + o);
    } else if (n == 8) {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
    } else {
        cp_async4(dst, src);
    }
}

template <int HD, int KT, int GT>
__global__ void __launch_bounds__(kGrpThreads) attention_group_kernel(const AttnParams p, int seq_cap) {
    constexpr bool F16 = KT == OVF_KV_F16;
    constexpr int CL = kGrpCluster, DPC = HD / CL, NT = kGrpThreads, EB = F16 ? 2 : 4;
    constexpr int G = GT;  // query heads of the KV head
    extern __shared__ __align__(16) float gsm[];
    gcg::cluster_group cluster = gcg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int g = blockIdx.x / CL, row = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const GroupLayout GL = group_layout(G, HD, seq_cap, EB);
    const int cc = GL.chunk_cap, spc = GL.sp_cap;
    float *qs = gsm;               // [G][HD]
    float *kn = qs + G * HD;       // [HD] current key (rotated)
    float *vn = kn + HD;           // [HD] current value
    float *red = vn + HD;          // [264]: warp maxima [8][8] | inv [80..88) | bad [88..96) | max [96..104) |
                                   //        every rank's maxima [128 + rank * G + h] | mbarrier at [256]
    uint64_t *bar = reinterpret_cast<uint64_t *>(red + 256);
    unsigned long long *etab = reinterpret_cast<unsigned long long *>(red + 264);
    float *sc = gsm + GL.o_sc;     // [G][cc] own slice: scores, then exponentials
    float *eall = gsm + GL.o_eall; // [G][spc] all exponentials, then probabilities
    char *kraw = reinterpret_cast<char *>(gsm + GL.o_reg2);  // key rows [t0, t1) while scoring
    float *vt = gsm + GL.o_reg2;   // then: [DPC][spc] this CTA's value columns, transposed (fp32 cache)
    char *vraw = reinterpret_cast<char *>(gsm + GL.o_vraw);  // fp16 cache: [spc][DPC] value columns as cached
    const char *kbase = reinterpret_cast<const char *>(p.kc) + (size_t)g * p.max_ctx * HD * EB;
    const char *vbase = reinterpret_cast<const char *>(p.vc) + (size_t)g * p.max_ctx * HD * EB;
    const int d0 = rank * DPC;

    if (tid == 0) trace_mark(p.trace, TR_START);
    if (tid < 32) etab[tid] = kExp2Tab32[tid];
    if (tid == 0 && p.pf.n) prefetch_l2_slice(p.pf, blockIdx.x, gridDim.x);
    OVF_PHASE(0);
    pdl_wait();
    if (tid == 0) trace_mark(p.trace, TR_WAITED);
    const int pos = p.pos_dev ? *p.pos_dev : p.seq_len_host - 1 + row;
    const int seq = pos + 1;
    const int chunk = (((seq + CL - 1) / CL) + 3) & ~3;
    const int t0 = min(seq, rank * chunk), t1 = min(seq, t0 + chunk);
    const int own = t1 - t0;
    const bool has_new = p.k_new != nullptr;
    // the cached rows arrive by asynchronous copies while the prologue runs:
    // the CTA's key rows [t0, t1) (contiguous), then its value columns
    // [d0, d0 + DPC) of every earlier position
    if (!F16) {
        const char *src = kbase + (size_t)t0 * HD * EB;
        const int n16 = own * HD * EB / 16;
        for (int i = tid; i < n16; i += NT) cp_async16(kraw + 16 * i, src + 16 * (size_t)i);
        cp_async_commit();
    }
    // the exponentials of every slice arrive by bulk copies from the owners:
    // G rows of own_pad(r) floats from each rank r
    if (tid == 0) {
        uint32_t expect = 0;
        for (int r = 0; r < CL; ++r) {
            const int a = min(seq, r * chunk), b = min(seq, a + chunk);
            expect += (uint32_t)(G * ((b - a + 3) & ~3) * 4);
        }
        mbar_init(bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(bar, expect);
    }

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
    OVF_PHASE(1);

    // 1. scores of [t0, t1) for every head of the group
    const int c = lane & 15, hw = lane >> 4;
    float qreg[G][HD / 16];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int i = 0; i < HD / 16; ++i) qreg[h][i] = qs[h * HD + 16 * i + c];
    float lmax[G];
#pragma unroll
    for (int h = 0; h < G; ++h) lmax[h] = -INFINITY;
    cp_async_wait<0>();  // this thread's key copies
    __syncthreads();
    constexpr int KPI = 2 * (NT / 32);  // keys per step (a half-warp each)
    constexpr int U = G <= 4 ? 4 : 2;   // keys per half-warp per step
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
                for (int i = 0; i < HD / 16; ++i) kv[u][i] = __half2float(__ldg(kr + 16 * i + c));
            } else {
                const float *kr = reinterpret_cast<const float *>(kraw) + (size_t)(tt - t0) * HD;
#pragma unroll
                for (int i = 0; i < HD / 16; ++i) kv[u][i] = kr[16 * i + c];
            }
        }
        // all (key, head) dots first, then each fold round over all of them:
        // the shuffles of independent dots overlap
        float v[U][G];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float a = 0.0f;
#pragma unroll
                for (int i = 0; i < HD / 16; ++i) a = fadd(a, fmul(qreg[h][i], kv[u][i]));
                v[u][h] = a;
            }
        // v[j] = acc0[j] + acc1[j], then ((v0+v1)+(v2+v3))+((v4+v5)+(v6+v7))
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int h = 0; h < G; ++h) v[u][h] = fadd(v[u][h], __shfl_xor_sync(0xFFFFFFFFu, v[u][h], 8));
#pragma unroll
        for (int o = 1; o <= 4; o <<= 1)
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int h = 0; h < G; ++h) v[u][h] = fadd(v[u][h], __shfl_xor_sync(0xFFFFFFFFu, v[u][h], o));
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + u * KPI + 2 * warp + hw;
            if (c == 0 && t < t1) {
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float sv = fmul(v[u][h], p.scale);
                    sc[h * cc + (t - t0)] = sv;
                    lmax[h] = sv > lmax[h] ? sv : lmax[h];
                }
            }
        }
    }
    OVF_PHASE(2);
    if (F16) {
        // the value columns [d0, d0 + DPC) of every earlier position arrive
        // while the maxima and exponentials are formed
        const int nv = has_new ? pos : seq;  // the decoded token's row is not cached yet
        for (int t = tid; t < nv; t += NT)
            cp_async_n(vraw + (size_t)t * DPC * EB, vbase + ((size_t)t * HD + d0) * EB, DPC * EB);
        cp_async_commit();
    }
    // 2. per-head maxima over the cluster (max is order-free)
#pragma unroll
    for (int h = 0; h < G; ++h) {
        float m = lmax[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        if (lane == 0) red[warp * 8 + h] = m;
    }
    __syncthreads();
    if (tid < G * CL) {
        // this CTA's maximum of head h, pushed to every rank's table
        const int r = tid / G, h = tid - r * G;
        float m = red[h];
        for (int w = 1; w < NT / 32; ++w) m = fmaxf(m, red[w * 8 + h]);
        cluster.map_shared_rank(red, r)[128 + rank * G + h] = m;
    }
    OVF_PHASE(3);
    cluster.sync();
    OVF_PHASE(4);
    if (tid < G) {
        float m = -INFINITY;
#pragma unroll
        for (int r = 0; r < CL; ++r) m = fmaxf(m, red[128 + r * G + tid]);
        red[96 + tid] = m;
    }
    __syncthreads();
    // the slice's exponentials, one per thread, then one bulk copy per
    // (rank, head) of them into every CTA's eall (t0 is a multiple of 4; a
    // last partial quad only fills positions past the sequence)
#pragma unroll
    for (int h = 0; h < G; ++h)
        for (int t = tid; t < own; t += NT) sc[h * cc + t] = exp_libm(fsub(sc[h * cc + t], red[96 + h]), etab);
    fence_proxy_async_smem();  // the writes above are read by the bulk-copy engine
    __syncthreads();
    const int own_pad = (own + 3) & ~3;
    if (tid < CL * G && own_pad > 0) {
        const int r = tid / G, h = tid - r * G;
        bulk_s2cluster(mapa_shared(smem_u32(eall + h * spc + t0), (uint32_t)r), sc + h * cc, (uint32_t)own_pad * 4,
                       mapa_shared(smem_u32(bar), (uint32_t)r));
    }
    OVF_PHASE(5);
    // meanwhile: this CTA's value columns, transposed to vt[d][t] over the
    // dead key rows, four positions per thread (fp16 cache: from the copies
    // already in shared memory, kept in fp16; fp32 cache: from the cache)
    cp_async_wait<0>();
    __syncthreads();
    const int nq = (seq + 3) >> 2;
    if (F16) {
        // block b = positions [16b, 16b + 16): [16][DPC] halves as copied ->
        // [DPC][16] in place, 16 lanes per block (lane j holds position j
        // between the warp's read and its writes).  Row d is rotated by
        // vrot(d) positions so that the output chains' 8-byte loads of rows
        // d and d + 4 fall in different banks.
        const int nblk = (seq + 15) >> 4, half = lane >> 4, j = lane & 15;
        for (int b0 = 2 * warp; b0 < nblk; b0 += 2 * (NT / 32)) {
            const int b = b0 + half, t = 16 * b + j;
            __half *bh = reinterpret_cast<__half *>(vraw) + (size_t)b * 16 * DPC;
            __half h[DPC];
            if (b < nblk) {
                if (has_new && t == pos) {
#pragma unroll
                    for (int d = 0; d < DPC; ++d) h[d] = __float2half_rn(vn[d0 + d]);
                } else if (t < seq) {
                    if (DPC == 8) {
                        const uint4 u = *reinterpret_cast<const uint4 *>(bh + j * DPC);
#pragma unroll
                        for (int d = 0; d < DPC; ++d) h[d] = reinterpret_cast<const __half *>(&u)[d];
                    } else if (DPC == 4) {
                        const uint2 u = *reinterpret_cast<const uint2 *>(bh + j * DPC);
#pragma unroll
                        for (int d = 0; d < DPC; ++d) h[d] = reinterpret_cast<const __half *>(&u)[d];
                    } else {
#pragma unroll
                        for (int d = 0; d < DPC; ++d) h[d] = bh[j * DPC + d];
                    }
                } else {
#pragma unroll
                    for (int d = 0; d < DPC; ++d) h[d] = __float2half_rn(0.0f);
                }
            }
            __syncwarp();
            if (b < nblk) {
#pragma unroll
                for (int d = 0; d < DPC; ++d) bh[d * 16 + ((j + vrot(d)) & 15)] = h[d];
            }
            __syncwarp();
        }
    }
    // fp32 cache: this CTA's value columns from the cache, transposed to
    // vt[d][t] over the dead key rows, four positions per thread
    for (int q = tid; q < (F16 ? 0 : nq); q += NT) {
        float v[4][DPC];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int t = 4 * q + j;
            if (has_new && t == pos) {
#pragma unroll
                for (int d = 0; d < DPC; ++d) v[j][d] = vn[d0 + d];
            } else if (t < seq) {
                load_cols<DPC, false>(vbase + ((size_t)t * HD + d0) * EB, v[j]);
            } else {
#pragma unroll
                for (int d = 0; d < DPC; ++d) v[j][d] = 0.0f;
            }
        }
#pragma unroll
        for (int d = 0; d < DPC; ++d)
            *reinterpret_cast<float4 *>(vt + d * spc + 4 * q) = make_float4(v[0][d], v[1][d], v[2][d], v[3][d]);
    }
    mbar_wait_sleep_bounded(bar, 0);  // every slice's exponentials have landed
    __syncthreads();
    OVF_PHASE(8);

    if (warp == 0 && lane < G) {
        // sumExp chains, one lane per head, in position order
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
    OVF_PHASE(9);
    __syncthreads();
    OVF_PHASE(10);
    // p_t = e_t * invSum (the reference's probability), all threads
    for (int h = 0; h < G; ++h) {
        const float inv = red[80 + h];
        float4 *e4 = reinterpret_cast<float4 *>(eall + h * spc);
        for (int q = tid; q < nq; q += NT) {
            float4 v = e4[q];
            v.x = fmul(v.x, inv);
            v.y = fmul(v.y, inv);
            v.z = fmul(v.z, inv);
            v.w = fmul(v.w, inv);
            e4[q] = v;
        }
    }
    __syncthreads();
    OVF_PHASE(11);
    // 4. output chains: lane (h, d) sums p_t * v_t[d] over t in order
    if (tid < G * DPC) {
        const int h = tid / DPC, d = tid - h * DPC;
        float acc = 0.0f;
        if (red[88 + h] == 0.0f) {
            const float *pp = eall + h * spc;
            const size_t vrow = (size_t)d * spc;
            // four values of dimension d at positions t..t+3 (t a multiple of 4)
            auto v4 = [&](int t) -> float4 {
                if (F16) {
                    // blocked layout: block t/16, column d, positions t%16..
                    const uint2 u = *reinterpret_cast<const uint2 *>(
                        reinterpret_cast<const __half *>(vraw) + (size_t)(t >> 4) * (16 * DPC) + d * 16 +
                        (((t & 15) + vrot(d)) & 15));
                    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
                    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
                    return make_float4(a.x, a.y, b.x, b.y);
                }
                return *reinterpret_cast<const float4 *>(vt + vrow + t);
            };
            const int s16 = seq & ~15;
            int t = 0;
            if (s16 > 0) {
                // the products of a block are formed while the previous
                // block's adds run; each add then waits only on the last one
                float pr[16];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 a = reinterpret_cast<const float4 *>(pp)[j];
                    const float4 b = v4(4 * j);
                    pr[4 * j] = fmul(a.x, b.x);
                    pr[4 * j + 1] = fmul(a.y, b.y);
                    pr[4 * j + 2] = fmul(a.z, b.z);
                    pr[4 * j + 3] = fmul(a.w, b.w);
                }
                for (; t < s16; t += 16) {
                    const int tn = t + 16 < s16 ? t + 16 : t;
                    float nx[16];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float4 a = reinterpret_cast<const float4 *>(pp + tn)[j];
                        const float4 b = v4(tn + 4 * j);
                        nx[4 * j] = fmul(a.x, b.x);
                        nx[4 * j + 1] = fmul(a.y, b.y);
                        nx[4 * j + 2] = fmul(a.z, b.z);
                        nx[4 * j + 3] = fmul(a.w, b.w);
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc = fadd(acc, pr[j]);
#pragma unroll
                    for (int j = 0; j < 16; ++j) pr[j] = nx[j];
                }
            }
            for (; t < seq; ++t) {
                const float4 b = v4(t & ~3);
                const float vv = (t & 3) == 0 ? b.x : (t & 3) == 1 ? b.y : (t & 3) == 2 ? b.z : b.w;
                acc = fadd(acc, fmul(pp[t], vv));
            }
        }
        p.out[((size_t)row * p.H + (size_t)g * G + h) * HD + d0 + d] = acc;
    }
    OVF_PHASE(12);
    cluster.sync();  // no CTA leaves while another may still read its shared memory
    OVF_PHASE(13);
    if (tid == 0) trace_mark(p.trace, TR_END);
}

// Whether the group kernel takes this launch; otherwise the per-head exact
// kernel (ovf_attn_exact.cu) does.
bool attn_group_supported(int H, int KVH, int hd, int kv_dtype, int seq_cap, int smem_optin_bytes) {
    if (kv_dtype != OVF_KV_F32 && kv_dtype != OVF_KV_F16) return false;
    if (hd != 32 && hd != 64 && hd != 128) return false;
    if (KVH <= 0 || H % KVH != 0) return false;
    const int G = H / KVH;
    if (G * (hd / kGrpCluster) > kGrpThreads) return false;
    const bool inst = G == 1 || G == 4 || G == 8 || (G == 2 && hd != 32) || (G == 7 && hd != 128);
    if (!inst) return false;
    return group_layout(G, hd, seq_cap, kv_dtype == OVF_KV_F16 ? 2 : 4).floats * 4 <= smem_optin_bytes;
}

template <int HD, int KT, int GT>
static cudaError_t launch_group_inst(const AttnParams &p, int seq_cap, size_t smem, cudaStream_t st, bool pdl) {
    static PerDeviceOnce attr_once;
    const int dev = current_device();
    if (attr_once.pending(dev)) {
        cudaError_t e = cudaFuncSetAttribute(attention_group_kernel<HD, KT, GT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin(dev));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attention_group_kernel<HD, KT, GT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
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
    return cudaLaunchKernelEx(&cfg, attention_group_kernel<HD, KT, GT>, p, seq_cap);
}

ovf_status launch_attention_group(const AttnParams &p, int seq_cap, cudaStream_t st, bool pdl, int kv_dtype) {
    const int G = p.H / p.KVH;
    const size_t smem = (size_t)group_layout(G, p.hd, seq_cap, kv_dtype == OVF_KV_F16 ? 2 : 4).floats * 4;
    OVF_CHECK_ARG(p.rows <= 1 || (p.k_new == nullptr && !p.pos_dev && p.rows <= 65535), "attention: bad row batch");
    cudaError_t e = cudaErrorInvalidValue;
    const bool f16 = kv_dtype == OVF_KV_F16;
#define OVF_GRP(HDV, GV)                                                                                      \
    if (p.hd == HDV && G == GV)                                                                               \
        e = f16 ? launch_group_inst<HDV, OVF_KV_F16, GV>(p, seq_cap, smem, st, pdl)                           \
                : launch_group_inst<HDV, OVF_KV_F32, GV>(p, seq_cap, smem, st, pdl);
    OVF_GRP(128, 1) OVF_GRP(128, 2) OVF_GRP(128, 4) OVF_GRP(128, 8)
    OVF_GRP(64, 1) OVF_GRP(64, 2) OVF_GRP(64, 4) OVF_GRP(64, 7) OVF_GRP(64, 8)
    OVF_GRP(32, 1) OVF_GRP(32, 4) OVF_GRP(32, 7) OVF_GRP(32, 8)
#undef OVF_GRP
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "attention_group_kernel launch");
}

}  // namespace ovf
