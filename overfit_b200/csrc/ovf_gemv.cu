// ovf_gemv.cu — quantized decode GEMV for sm_100a (see ovf_gemv.cuh).
//
// Work decomposition ("lanes own rows").  A warp owns a group of 32/L
// consecutive weight rows; L lanes (1, 2 or 4) share a row.  The warp streams
// its rows through a private ring of shared-memory stages, C blocks of every
// row per stage: each row's chunk is one 1-D bulk copy (the TMA engine) issued
// by the row's first lane, so every stage is 32/L independent contiguous
// copies landing on one mbarrier.  The first stages are requested before
// griddepcontrol.wait, while the previous kernel of the decode step is still
// finishing (programmatic dependent launch).
//
// Because a lane group owns whole rows, every lane contracts the same
// activation block at the same time (shared-memory broadcast), and the row's
// block terms are accumulated in registers in ascending block order — the
// reference's sequential fp32 loop (Runtime/Q4KDotKernel.cs:528-552,
// Q6KDotKernel.cs:364-380, Q8DotKernel.cs:311-328) — with no reduction pass.
// Integer parts are exact and the fp32 tails use explicitly rounded ops in
// the reference's operand order, so results are bit-identical to it.
//
// Chunks are copied from the 16-byte boundary at or below their first byte
// (Q6_K blocks are 210 bytes), so a block may start 4/8/12 bytes into its
// smem row; the Q6_K unit reads through a funnel shift.  A copy that would
// run past the end of the weight buffer stops at the last 16-byte boundary
// and its last few bytes are copied by the lane itself.
#include "ovf_gemv.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>

namespace ovf {

static constexpr int kQ8kActStride = 272;  // 256 quants + 16 pad
static constexpr int kQ8kMetaStride = 64;  // int16 bsums[16] | f32 scale | pad | int16 pair sums[8]
static constexpr int kQ80ActStride = 48;   // 32 quants + f32 scale + pad
static constexpr int kMaxUnits = 4;        // blocks per lane per chunk

int block_bytes(int type) {
    switch (type) {
        case OVF_TYPE_Q4_K: return 144;
        case OVF_TYPE_Q6_K: return 210;
        case OVF_TYPE_Q8_0: return 36;
        default: return 0;
    }
}

static __host__ __device__ inline bool is_kquant(int t) { return t == OVF_TYPE_Q4_K || t == OVF_TYPE_Q6_K; }
static __host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
static __host__ __device__ inline int kq_block_bytes(int type) { return type == OVF_TYPE_Q4_K ? 144 : 210; }

// Row stride in shared memory for a copied span of `bytes` that may start up
// to 15 bytes before its data: an odd number of 16-byte units, so the lanes'
// 16-byte reads of 8 consecutive rows fall in distinct banks.
static __host__ __device__ inline int smem_stride(int bytes) {
    int s = (int)align_up((size_t)bytes + 30, 16);
    if (((s / 16) & 1) == 0) s += 16;
    return s;
}

struct Layout {
    int act_q_off, act_meta_off, red_off, terms_off, stage_off;
    int stage_bytes, q_stride, s_stride, s_region;  // Q8_0: quants rows then scales rows
    int part_bytes, s_part;                         // whole-row stages: bytes per matrix part
    int nb;
};

// Shared memory: mbarriers | activation | reduction scratch | two term
// buffers [T][C] | stage ring.  Stage rows are sized for the launch's
// largest block (K-quant launches may mix Q4_K and Q6_K rows).
static __host__ __device__ inline Layout make_layout(const GemvParams &p) {
    Layout L{};
    const int type0 = p.seg[0].type;
    const bool kq = is_kquant(type0);
    L.nb = kq ? p.K / 256 : p.K / 32;
    const int T = p.rows_per_group;
    size_t off = align_up(sizeof(uint64_t) * 2 * p.stages, 128);
    L.act_q_off = (int)off;
    if (kq) {
        off = align_up(off + (size_t)L.nb * kQ8kActStride, 128);
        L.act_meta_off = (int)off;
        off = align_up(off + (size_t)L.nb * kQ8kMetaStride, 128);
    } else {
        off = align_up(off + (size_t)L.nb * kQ80ActStride, 128);
        L.act_meta_off = L.act_q_off;
    }
    L.red_off = (int)off;
    off = align_up(off + 64 * sizeof(float) + 32 * sizeof(unsigned long long), 128);
    L.terms_off = (int)off;
    off = align_up(off + (size_t)p.stages * T * p.chunk * sizeof(float), 128);
    L.stage_off = (int)off;
    if (p.chunk == L.nb) {
        // Whole rows: a tile's rows are contiguous in the weight buffer, so a
        // stage is one copy per matrix (quants and scales for Q8_0).
        const int parts = p.pair ? 2 : 1, per = T / parts;
        if (kq) {
            int rb = 0;
            for (int s = 0; s < p.nseg; ++s) rb = max(rb, L.nb * kq_block_bytes(p.seg[s].type));
            L.q_stride = rb;
            L.part_bytes = (int)align_up((size_t)per * rb + 16, 16);
            L.s_stride = 0;
            L.s_part = 0;
            L.s_region = parts * L.part_bytes;
        } else {
            L.q_stride = p.K;
            L.part_bytes = (int)align_up((size_t)per * p.K + 16, 16);
            L.s_stride = p.K / 8;
            L.s_part = (int)align_up((size_t)per * (p.K / 8) + 16, 16);
            L.s_region = parts * L.part_bytes;
        }
        L.stage_bytes = (int)align_up((size_t)L.s_region + (size_t)parts * L.s_part, 128);
    } else if (kq) {
        int mx = 0;
        for (int s = 0; s < p.nseg; ++s) mx = max(mx, smem_stride(p.chunk * kq_block_bytes(p.seg[s].type)));
        L.q_stride = mx;
        L.s_stride = 0;
        L.s_region = 0;
        L.stage_bytes = (int)align_up((size_t)T * mx, 128);
    } else {
        L.q_stride = smem_stride(32 * p.chunk);
        L.s_stride = smem_stride(4 * p.chunk);
        L.s_region = T * L.q_stride;
        L.stage_bytes = (int)align_up((size_t)T * (L.q_stride + L.s_stride), 128);
    }
    return L;
}

static __host__ __device__ inline size_t layout_smem(const Layout &L, int stages) {
    return (size_t)L.stage_off + (size_t)stages * L.stage_bytes;
}

// ------------------------------------------------------------- dot units
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// Q4_K x Q8_K over one super-block (Runtime/Q4KDotKernel.cs:216-256).
__device__ __forceinline__ float q4k_unit(const uint8_t *blk, const uint8_t *q8, const uint8_t *meta) {
    const uint4 h = *reinterpret_cast<const uint4 *>(blk);
    const float d = h2f_bits((uint16_t)(h.x & 0xFFFFu));
    const float dmin = h2f_bits((uint16_t)(h.x >> 16));
    // 6-bit scales and mins (Loading/GgmlDequant.cs:49-77), four per word
    const uint32_t sc03 = h.y & 0x3F3F3F3Fu, mn03 = h.z & 0x3F3F3F3Fu;
    const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    int mainAcc = 0, mainAccH = 0;  // mainAccH: exact multiple of 16
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * p);
        const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * p);
        const uint4 l0 = *reinterpret_cast<const uint4 *>(q8 + 64 * p);
        const uint4 l1 = *reinterpret_cast<const uint4 *>(q8 + 64 * p + 16);
        const uint4 h0 = *reinterpret_cast<const uint4 *>(q8 + 64 * p + 32);
        const uint4 h1 = *reinterpret_cast<const uint4 *>(q8 + 64 * p + 48);
        const uint32_t M = 0x0F0F0F0Fu, HM = 0xF0F0F0F0u;
        // High nibbles stay in place (16 * nibble as the unsigned operand):
        // that sum is 16x the nibble dot and is divided out exactly below.
        int lo = dp4a((int)(qa.x & M), (int)l0.x, 0);
        int lo2 = dp4a((int)(qb.x & M), (int)l1.x, 0);
        int hi = dp4a_us(qa.x & HM, (int)h0.x, 0);
        int hi2 = dp4a_us(qb.x & HM, (int)h1.x, 0);
        lo = dp4a((int)(qa.y & M), (int)l0.y, lo);
        lo2 = dp4a((int)(qb.y & M), (int)l1.y, lo2);
        hi = dp4a_us(qa.y & HM, (int)h0.y, hi);
        hi2 = dp4a_us(qb.y & HM, (int)h1.y, hi2);
        lo = dp4a((int)(qa.z & M), (int)l0.z, lo);
        lo2 = dp4a((int)(qb.z & M), (int)l1.z, lo2);
        hi = dp4a_us(qa.z & HM, (int)h0.z, hi);
        hi2 = dp4a_us(qb.z & HM, (int)h1.z, hi2);
        lo = dp4a((int)(qa.w & M), (int)l0.w, lo);
        lo2 = dp4a((int)(qb.w & M), (int)l1.w, lo2);
        hi = dp4a_us(qa.w & HM, (int)h0.w, hi);
        hi2 = dp4a_us(qb.w & HM, (int)h1.w, hi2);
        const uint32_t scw = p < 2 ? sc03 : sc47;
        mainAcc += (int)byte_of(scw, (2 * p) & 3) * (lo + lo2);
        mainAccH += (int)byte_of(scw, (2 * p + 1) & 3) * (hi + hi2);
    }
    mainAcc += mainAccH >> 4;
    // min correction: sum_s m[s] * (bsum[2s] + bsum[2s+1]) as four dp2a
    const uint4 ps = *reinterpret_cast<const uint4 *>(meta + 48);
    const float q8s = *reinterpret_cast<const float *>(meta + 32);
    int minAcc = __dp2a_lo((int)ps.x, (int)mn03, 0);
    minAcc = __dp2a_hi((int)ps.y, (int)mn03, minAcc);
    minAcc = __dp2a_lo((int)ps.z, (int)mn47, minAcc);
    minAcc = __dp2a_hi((int)ps.w, (int)mn47, minAcc);
    return fmul(q8s, fsub(fmul(d, i2f(mainAcc)), fmul(dmin, i2f(minAcc))));
}

// 32-bit word `w` of a 210-byte block that may start 2 bytes past a word.
__device__ __forceinline__ uint32_t ldw_shifted(const uint32_t *base, int w, int sh) {
    return __funnelshift_r(base[w], base[w + 1], sh);
}

// Q6_K x Q8_K over one super-block (Runtime/Q6KDotKernel.cs:77-121 with the
// unsigned dot :186-215).
__device__ __forceinline__ float q6k_unit(const uint8_t *blk, const uint8_t *q8, const uint8_t *meta) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
    const uint32_t *base = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const int sh = (int)(a & 3u) * 8;
    int sc[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t w = ldw_shifted(base, 48 + i, sh);
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[4 * i + j] = (int)(int8_t)byte_of(w, j);
    }
    const float d = h2f_bits((uint16_t)(ldw_shifted(base, 52, sh) & 0xFFFFu));
    const uint32_t *q8w = reinterpret_cast<const uint32_t *>(q8);
    int sum = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int lw = 0; lw < 8; ++lw) {
            const uint32_t qla = ldw_shifted(base, 16 * h + lw, sh);
            const uint32_t qlb = ldw_shifted(base, 16 * h + 8 + lw, sh);
            const uint32_t qhw = ldw_shifted(base, 32 + 8 * h + lw, sh);
            const uint32_t M = 0x0F0F0F0Fu, H = 0x30303030u;
            const int q1 = (int)((qla & M) | ((qhw << 4) & H));
            const int q2 = (int)((qlb & M) | ((qhw << 2) & H));
            const int q3 = (int)(((qla >> 4) & M) | (qhw & H));
            const int q4 = (int)(((qlb >> 4) & M) | ((qhw >> 2) & H));
            const int is = lw >> 2;
            const int base8 = 32 * h + lw;
            sum += sc[8 * h + is] * dp4a(q1, (int)q8w[base8], 0) + sc[8 * h + is + 2] * dp4a(q2, (int)q8w[base8 + 8], 0) +
                   sc[8 * h + is + 4] * dp4a(q3, (int)q8w[base8 + 16], 0) +
                   sc[8 * h + is + 6] * dp4a(q4, (int)q8w[base8 + 24], 0);
        }
    }
    const uint4 b0 = *reinterpret_cast<const uint4 *>(meta);
    const uint4 b1 = *reinterpret_cast<const uint4 *>(meta + 16);
    const float q8s = *reinterpret_cast<const float *>(meta + 32);
    const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    int bsumTerm = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        bsumTerm += sc[2 * s] * (int)(int16_t)(bw[s] & 0xFFFFu) + sc[2 * s + 1] * (int)(int16_t)(bw[s] >> 16);
    }
    const int mainAcc = sum - 32 * bsumTerm;
    return fmul(fmul(d, q8s), i2f(mainAcc));
}

// Q8_0 x Q8_0 over one 32-block (Runtime/Q8DotKernel.cs:99-140).
__device__ __forceinline__ float q80_unit(const uint8_t *wq, float ws, const uint8_t *act) {
    const uint4 w0 = *reinterpret_cast<const uint4 *>(wq);
    const uint4 w1 = *reinterpret_cast<const uint4 *>(wq + 16);
    const uint4 a0 = *reinterpret_cast<const uint4 *>(act);
    const uint4 a1 = *reinterpret_cast<const uint4 *>(act + 16);
    const float xs = *reinterpret_cast<const float *>(act + 32);
    int dot = 0;
    dot = dp4a((int)w0.x, (int)a0.x, dot);
    dot = dp4a((int)w0.y, (int)a0.y, dot);
    dot = dp4a((int)w0.z, (int)a0.z, dot);
    dot = dp4a((int)w0.w, (int)a0.w, dot);
    dot = dp4a((int)w1.x, (int)a1.x, dot);
    dot = dp4a((int)w1.y, (int)a1.y, dot);
    dot = dp4a((int)w1.z, (int)a1.z, dot);
    dot = dp4a((int)w1.w, (int)a1.w, dot);
    return fmul(fmul(ws, xs), i2f(dot));
}

// --------------------------------------------------------- activation prep
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

// RMSNorm scale s = 1/sqrt(sum(x^2)/K + eps) with a fixed-order block
// reduction (Runtime/CachedTransformerBlock.cs:525-552; the reference's sum
// is sequential, so this one agrees to rounding, not bit for bit).
__device__ float block_rms_scale(const float *x, int K, float eps, float *red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float s = 0.0f;
    for (int i = tid; i < K; i += blockDim.x) s = fadd(s, fmul(x[i], x[i]));
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float v = lane < nw ? red[lane] : 0.0f;
        v = warp_sum(v);
        if (lane == 0) red[32] = fdiv(1.0f, sqrtf(fadd(fdiv(v, (float)K), eps)));
    }
    __syncthreads();
    return red[32];
}

// Block-wide sum of one value per thread (fixed order), broadcast to all.
__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nw ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

// Activation prologue, Q8_K form.  Every lane first issues the loads of all
// its elements (independent 16-byte loads, one memory round trip), then the
// CTA reduces the RMSNorm sum of squares (Runtime/CachedTransformerBlock.cs:
// 525-552; fixed-order tree, so equal to the reference's sequential sum up to
// rounding) and quantizes per 256 (Runtime/Q4KDotKernel.cs:71-136).
__device__ void prep_q8k(const GemvParams &p, const Layout &L, uint8_t *smem) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint8_t *aq = smem + L.act_q_off;
    uint8_t *meta = smem + L.act_meta_off;
    const int nsb = L.nb;
    if (p.act_mode == ACT_PREQ_Q8K) {
        for (int b = warp; b < nsb; b += nw) {
            *reinterpret_cast<uint2 *>(aq + b * kQ8kActStride + 8 * lane) =
                *reinterpret_cast<const uint2 *>(p.aq + (size_t)b * 256 + 8 * lane);
            if (lane < 16) reinterpret_cast<int16_t *>(meta + b * kQ8kMetaStride)[lane] = p.ab[(size_t)b * 16 + lane];
            if (lane < 8)
                reinterpret_cast<int16_t *>(meta + b * kQ8kMetaStride + 48)[lane] =
                    (int16_t)(p.ab[(size_t)b * 16 + 2 * lane] + p.ab[(size_t)b * 16 + 2 * lane + 1]);
            if (lane == 0) *reinterpret_cast<float *>(meta + b * kQ8kMetaStride + 32) = p.as[b];
        }
        return;
    }
    float *red = reinterpret_cast<float *>(smem + L.red_off);
    const bool norm = p.act_mode == ACT_F32_RMSNORM;
    const bool write_out = blockIdx.x == 0 && p.aq_out != nullptr;
    constexpr int MB = 4;  // blocks per warp held in registers per batch
    float s = 1.0f;
    if (norm) {
        float ss = 0.0f;
        for (int b0 = warp; b0 < nsb; b0 += nw * MB) {
            float4 x0[MB], x1[MB];
#pragma unroll
            for (int i = 0; i < MB; ++i) {
                const int b = b0 + i * nw;
                if (b < nsb) {
                    x0[i] = *reinterpret_cast<const float4 *>(p.x + b * 256 + 8 * lane);
                    x1[i] = *reinterpret_cast<const float4 *>(p.x + b * 256 + 8 * lane + 4);
                }
            }
#pragma unroll
            for (int i = 0; i < MB; ++i) {
                if (b0 + i * nw < nsb) {
                    ss = fadd(ss, fmul(x0[i].x, x0[i].x)); ss = fadd(ss, fmul(x0[i].y, x0[i].y));
                    ss = fadd(ss, fmul(x0[i].z, x0[i].z)); ss = fadd(ss, fmul(x0[i].w, x0[i].w));
                    ss = fadd(ss, fmul(x1[i].x, x1[i].x)); ss = fadd(ss, fmul(x1[i].y, x1[i].y));
                    ss = fadd(ss, fmul(x1[i].z, x1[i].z)); ss = fadd(ss, fmul(x1[i].w, x1[i].w));
                }
            }
        }
        const float tot = block_sum(ss, red);
        s = fdiv(1.0f, sqrtf(fadd(fdiv(tot, (float)p.K), p.eps)));
    }
    for (int b0 = warp; b0 < nsb; b0 += nw * MB) {
        float v[MB][8];
        float gm[MB][8];
#pragma unroll
        for (int i = 0; i < MB; ++i) {
            const int b = b0 + i * nw;
            if (b < nsb) {
                const float4 x0 = *reinterpret_cast<const float4 *>(p.x + b * 256 + 8 * lane);
                const float4 x1 = *reinterpret_cast<const float4 *>(p.x + b * 256 + 8 * lane + 4);
                v[i][0] = x0.x; v[i][1] = x0.y; v[i][2] = x0.z; v[i][3] = x0.w;
                v[i][4] = x1.x; v[i][5] = x1.y; v[i][6] = x1.z; v[i][7] = x1.w;
                if (norm && p.gamma) {
                    const float4 g0 = *reinterpret_cast<const float4 *>(p.gamma + b * 256 + 8 * lane);
                    const float4 g1 = *reinterpret_cast<const float4 *>(p.gamma + b * 256 + 8 * lane + 4);
                    gm[i][0] = g0.x; gm[i][1] = g0.y; gm[i][2] = g0.z; gm[i][3] = g0.w;
                    gm[i][4] = g1.x; gm[i][5] = g1.y; gm[i][6] = g1.z; gm[i][7] = g1.w;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MB; ++i) {
            const int b = b0 + i * nw;
            if (b >= nsb) continue;
            if (norm) {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] = p.gamma ? fmul(fmul(v[i][j], s), gm[i][j]) : fmul(v[i][j], s);
            }
            float amax = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
            amax = warp_max(amax);
            const float scale = fdiv(amax, 127.0f);
            const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
            uint32_t w0 = 0, w1 = 0;
            int sum8 = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int q = quant_elem(v[i][j], inv);
                sum8 += q;
                if (j < 4) w0 |= ((uint32_t)(q & 0xFF)) << (8 * j);
                else w1 |= ((uint32_t)(q & 0xFF)) << (8 * (j - 4));
            }
            const int g16 = sum8 + __shfl_xor_sync(0xFFFFFFFFu, sum8, 1);
            const int g32 = g16 + __shfl_xor_sync(0xFFFFFFFFu, g16, 2);
            *reinterpret_cast<uint2 *>(aq + b * kQ8kActStride + 8 * lane) = make_uint2(w0, w1);
            if ((lane & 1) == 0) reinterpret_cast<int16_t *>(meta + b * kQ8kMetaStride)[lane >> 1] = (int16_t)g16;
            if ((lane & 3) == 0) reinterpret_cast<int16_t *>(meta + b * kQ8kMetaStride + 48)[lane >> 2] = (int16_t)g32;
            if (lane == 0) *reinterpret_cast<float *>(meta + b * kQ8kMetaStride + 32) = scale;
            if (write_out) {
                *reinterpret_cast<uint2 *>(p.aq_out + b * 256 + 8 * lane) = make_uint2(w0, w1);
                if ((lane & 1) == 0) p.ab_out[(size_t)b * 16 + (lane >> 1)] = (int16_t)g16;
                if (lane == 0) p.as_out[b] = scale;
            }
        }
    }
}

// Activation prologue, Q8_0 form (Runtime/Q8DotKernel.cs:42-91), same
// load-everything-first structure.
__device__ void prep_q80(const GemvParams &p, const Layout &L, uint8_t *smem) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint8_t *act = smem + L.act_q_off;
    float *red = reinterpret_cast<float *>(smem + L.red_off);
    const bool norm = p.act_mode == ACT_F32_RMSNORM;
    const bool write_out = blockIdx.x == 0 && p.aq_out != nullptr;
    constexpr int MB = 16;
    const int nb = L.nb;
    float s = 1.0f;
    if (norm) {
        float ss = 0.0f;
        for (int b0 = warp; b0 < nb; b0 += nw * MB) {
            float xv[MB];
#pragma unroll
            for (int i = 0; i < MB; ++i) xv[i] = (b0 + i * nw < nb) ? p.x[(b0 + i * nw) * 32 + lane] : 0.0f;
#pragma unroll
            for (int i = 0; i < MB; ++i) ss = fadd(ss, fmul(xv[i], xv[i]));
        }
        const float tot = block_sum(ss, red);
        s = fdiv(1.0f, sqrtf(fadd(fdiv(tot, (float)p.K), p.eps)));
    }
    for (int b0 = warp; b0 < nb; b0 += nw * MB) {
        float xv[MB], gv[MB];
#pragma unroll
        for (int i = 0; i < MB; ++i) {
            const int b = b0 + i * nw;
            xv[i] = b < nb ? p.x[b * 32 + lane] : 0.0f;
            gv[i] = (norm && p.gamma && b < nb) ? p.gamma[b * 32 + lane] : 1.0f;
        }
#pragma unroll
        for (int i = 0; i < MB; ++i) {
            const int b = b0 + i * nw;
            if (b >= nb) continue;
            float v = xv[i];
            if (norm) v = p.gamma ? fmul(fmul(v, s), gv[i]) : fmul(v, s);
            const float amax = warp_max(fabsf(v));
            const float scale = fdiv(amax, 127.0f);
            const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
            const int q = quant_elem(v, inv);
            act[b * kQ80ActStride + lane] = (uint8_t)(int8_t)q;
            if (lane == 0) *reinterpret_cast<float *>(act + b * kQ80ActStride + 32) = scale;
            if (write_out) {
                p.aq_out[b * 32 + lane] = (int8_t)q;
                if (lane == 0) p.as_out[b] = scale;
            }
        }
    }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}


// ------------------------------------------------------------ row tiles
struct GroupRef {
    int seg, r0, nr;  // nr: valid rows (per matrix in pair mode)
};

__device__ __forceinline__ GroupRef locate(const GemvParams &p, int g) {
    int s = 0;
    const int rows_per = p.pair ? p.rows_per_group / 2 : p.rows_per_group;
    if (!p.pair) {
        while (s < p.nseg - 1 && g >= p.seg[s].groups) {
            g -= p.seg[s].groups;
            ++s;
        }
    }
    GroupRef r;
    r.seg = s;
    r.r0 = g * rows_per;
    r.nr = min(rows_per, p.seg[s].rows - r.r0);
    return r;
}

// Row slot of a tile -> (segment, row); false for an empty slot.  Pair
// mode: slots [0, T/2) are gate rows, [T/2, T) the same up rows.
__device__ __forceinline__ bool slot_row(const GemvParams &p, const GroupRef &g, int slot, int *seg, int *row) {
    if (p.pair) {
        const int half = p.rows_per_group / 2;
        const int m = slot >= half ? 1 : 0, i = slot - m * half;
        *seg = m;
        *row = g.r0 + i;
        return i < g.nr;
    }
    *seg = g.seg;
    *row = g.r0 + slot;
    return slot < g.nr;
}

// Copies bytes [off, off+len) of `src` (total `total` bytes) so that they sit
// at dst + (off & 15): the bulk engine moves whole 16-byte units, the lane
// itself the bytes past the buffer's last 16-byte boundary.  Returns the bulk
// bytes (for the stage's transaction count); `issue` false only counts.
__device__ __forceinline__ uint32_t copy_span(uint8_t *dst, const uint8_t *src, size_t off, size_t len, size_t total,
                                              uint64_t *bar, uint64_t pol, bool issue) {
    const size_t a = off & ~size_t(15);
    const size_t e = min(align_up(off + len, 16), total);
    const size_t be = e & ~size_t(15);
    const uint32_t bulk = be > a ? (uint32_t)(be - a) : 0u;
    if (issue) {
        if (bulk) bulk_g2s(dst, src + a, bulk, bar, pol);
        for (size_t i = max(a, be); i < e; ++i) dst[i - a] = src[i];
    }
    return bulk;
}

// Issued by warp 0: chunk `c` of every row of tile `g`, one copy per row
// (two for Q8_0: quants and scales), lane i copying row slot i.
__device__ __forceinline__ void issue_stage(const GemvParams &p, const Layout &L, const GroupRef &g, int c,
                                            uint8_t *stage, uint64_t *bar, uint64_t pol, int lane) {
    if (p.chunk == L.nb) {
        // Whole rows: lane `part` copies the tile's rows of its matrix.
        const int parts = p.pair ? 2 : 1;
        const GemvSeg &sg = p.seg[p.pair ? min(lane, 1) : g.seg];
        uint32_t bytes = 0;
        const bool mine = lane < parts && g.nr > 0;
        for (int pass = 0; pass < 2; ++pass) {
            const bool issue = pass == 1;
            if (issue) {
                const uint32_t total = __reduce_add_sync(0xFFFFFFFFu, bytes);
                if (lane == 0) mbar_arrive_expect_tx(bar, total);
                __syncwarp();
            }
            if (!mine) continue;
            if (is_kquant(sg.type)) {
                // The part is cut into `split` copies issued by consecutive
                // lanes: more copies in flight keep more DRAM requests open.
                const size_t rb = (size_t)L.nb * kq_block_bytes(sg.type);
                const size_t off = (size_t)g.r0 * rb, len = (size_t)g.nr * rb;
                const size_t a0 = off & ~size_t(15);
                const size_t piece = align_up((len + (off - a0) + p.copy_split - 1) / p.copy_split, 16);
                bytes = 0;
                for (int q = 0; q < p.copy_split; ++q) {
                    const size_t ps = a0 + q * piece;
                    if (ps >= off + len) break;
                    const size_t s0 = q == 0 ? off : ps;
                    const size_t e0 = min(off + len, ps + piece);
                    bytes += copy_span(stage + lane * L.part_bytes + (s0 - a0) - (s0 & 15), sg.w, s0, e0 - s0,
                                       (size_t)sg.rows * rb, bar, pol, issue);
                }
            } else {
                const size_t K = p.K;
                const uint32_t b1 = copy_span(stage + lane * L.part_bytes, sg.w, (size_t)g.r0 * K, (size_t)g.nr * K,
                                              (size_t)sg.rows * K, bar, pol, issue);
                const uint32_t b2 = copy_span(stage + L.s_region + lane * L.s_part,
                                              reinterpret_cast<const uint8_t *>(sg.ws), (size_t)g.r0 * (K / 8),
                                              (size_t)g.nr * (K / 8), (size_t)sg.rows * (K / 8), bar, pol, issue);
                bytes = b1 + b2;
            }
        }
        return;
    }
    const int slot = lane;
    int seg = 0, row = 0;
    const bool mine = slot < p.rows_per_group && slot_row(p, g, slot, &seg, &row);
    uint32_t bytes = 0;
    const GemvSeg &sg = p.seg[seg];
    const int type = sg.type;
    const int nbk = is_kquant(type) ? p.K / 256 : p.K / 32;
    const int cc = min(p.chunk, nbk - c * p.chunk);  // the last chunk may be short
    for (int pass = 0; pass < 2; ++pass) {
        const bool issue = pass == 1;
        if (issue) {
            const uint32_t total = __reduce_add_sync(0xFFFFFFFFu, bytes);
            if (lane == 0) mbar_arrive_expect_tx(bar, total);
            __syncwarp();
        }
        if (!mine) continue;
        if (is_kquant(type)) {
            const int bb = kq_block_bytes(type);
            const size_t rb = (size_t)nbk * bb;
            const size_t off = (size_t)row * rb + (size_t)c * p.chunk * bb;
            bytes = copy_span(stage + slot * L.q_stride, sg.w, off, (size_t)cc * bb, (size_t)sg.rows * rb, bar, pol,
                              issue);
        } else {
            const size_t K = p.K;
            const size_t offq = (size_t)row * K + (size_t)c * p.chunk * 32;
            const size_t offs = (size_t)row * (K / 8) + (size_t)c * p.chunk * 4;
            const uint32_t b1 = copy_span(stage + slot * L.q_stride, sg.w, offq, (size_t)cc * 32, (size_t)sg.rows * K,
                                          bar, pol, issue);
            const uint32_t b2 =
                copy_span(stage + L.s_region + slot * L.s_stride, reinterpret_cast<const uint8_t *>(sg.ws), offs,
                          (size_t)cc * 4, (size_t)sg.rows * (K / 8), bar, pol, issue);
            bytes = b1 + b2;
        }
    }
}

// ------------------------------------------------------------------ kernel
// A CTA owns T-row tiles (persistent, tile = blockIdx.x + i*gridDim.x) and
// streams each through a ring of `stages` shared-memory buffers, C blocks of
// every row per stage.  Warp specialisation: the last warp issues the bulk
// copies and keeps the ordered row sums; the other (compute) warps contract
// each stage (thread -> row slot and block, so the lanes of a warp read at
// most two activation blocks) into the stage's [T][C] term buffer and
// arrive on the stage's `done` mbarrier.  The row warp then adds row r's
// terms in ascending block order (lane r), refills the stage and, after a
// row's last chunk, runs the epilogue.  No CTA-wide barrier sits in the loop.
static constexpr int kComputeWarps = 8;

__global__ void __launch_bounds__((kComputeWarps + 1) * 32, 1) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const Layout L = make_layout(p);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *done = full + p.stages;
    uint8_t *ring = smem + L.stage_off;
    float *tbuf = reinterpret_cast<float *>(smem + L.terms_off);
    const int T = p.rows_per_group, C = p.chunk, nb = L.nb;
    const int my_tiles = blockIdx.x < p.total_groups ? (p.total_groups - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const int items = my_tiles * p.nchunks;
    const uint64_t pol = l2_evict_first_policy();
    const bool row_warp = warp == kComputeWarps;

    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&done[s], kComputeWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    // Weights do not depend on the previous kernel: start streaming now.
    if (row_warp)
        for (int it = 0; it < p.stages && it < items; ++it) {
            const GroupRef g = locate(p, blockIdx.x + (it / p.nchunks) * gridDim.x);
            issue_stage(p, L, g, it % p.nchunks, ring + (size_t)it * L.stage_bytes, &full[it], pol, lane);
        }

    pdl_wait();
    if (is_kquant(p.seg[0].type)) prep_q8k(p, L, smem);
    else prep_q80(p, L, smem);
    __syncthreads();
    pdl_launch_dependents();

    const bool kq = is_kquant(p.seg[0].type);
    if (!row_warp) {
        // ------------------------------------------------ compute warps
        const int ct = warp * 32 + lane, nct = kComputeWarps * 32;
        const int rs = ct % T, m0 = ct / T, mstep = nct / T;
        GroupRef g{0, 0, 0};
        for (int it = 0; it < items; ++it) {
            const int s = it % p.stages;
            const int c = it % p.nchunks;
            if (c == 0) g = locate(p, blockIdx.x + (it / p.nchunks) * gridDim.x);
            if (!mbar_wait_bounded(&full[s], (uint32_t)((it / p.stages) & 1))) break;
            const uint8_t *stage = ring + (size_t)s * L.stage_bytes;
            float *tb = tbuf + (size_t)s * T * C;
            int seg = 0, row = 0;
            const bool valid = slot_row(p, g, rs, &seg, &row);
            const int type = p.seg[seg].type;
            const int cc = min(C, nb - c * C);
            if (C == nb) {
                // Whole rows: unit u -> (row slot u / nb, block u % nb); the
                // lanes of a warp walk consecutive blocks of one or two rows.
                if (!p.skip_compute) {
                    const int half = p.pair ? T / 2 : T;
                    for (int u = ct; u < T * nb; u += nct) {
                        const int us = u / nb, m = u - us * nb;
                        int useg = 0, urow = 0;
                        if (!slot_row(p, g, us, &useg, &urow)) continue;
                        const int part = us / half, i = us - part * half;
                        const int utype = p.seg[useg].type;
                        float t;
                        if (kq) {
                            const int bb = kq_block_bytes(utype);
                            const size_t off0 = (size_t)g.r0 * nb * bb;
                            const uint8_t *blk = stage + part * L.part_bytes + (off0 & 15) + (size_t)i * L.q_stride +
                                                 (size_t)m * bb;
                            t = utype == OVF_TYPE_Q4_K
                                    ? q4k_unit(blk, smem + L.act_q_off + m * kQ8kActStride,
                                               smem + L.act_meta_off + m * kQ8kMetaStride)
                                    : q6k_unit(blk, smem + L.act_q_off + m * kQ8kActStride,
                                               smem + L.act_meta_off + m * kQ8kMetaStride);
                        } else {
                            const size_t offq0 = (size_t)g.r0 * p.K, offs0 = (size_t)g.r0 * (p.K / 8);
                            const uint8_t *wq = stage + part * L.part_bytes + (offq0 & 15) + (size_t)i * p.K + 32 * m;
                            const float ws = *reinterpret_cast<const float *>(
                                stage + L.s_region + part * L.s_part + (offs0 & 15) + (size_t)i * (p.K / 8) + 4 * m);
                            t = q80_unit(wq, ws, smem + L.act_q_off + m * kQ80ActStride);
                        }
                        tb[us * C + m] = t;
                    }
                }
            } else if (valid && !p.skip_compute) {
                for (int m = m0; m < cc; m += mstep) {
                    const int j = c * C + m;
                    float t;
                    if (kq) {
                        const int bb = kq_block_bytes(type);
                        const size_t off = (size_t)row * nb * bb + (size_t)c * C * bb;
                        const uint8_t *blk = stage + rs * L.q_stride + (off & 15) + (size_t)m * bb;
                        const uint8_t *aq = smem + L.act_q_off + j * kQ8kActStride;
                        const uint8_t *am = smem + L.act_meta_off + j * kQ8kMetaStride;
                        t = type == OVF_TYPE_Q4_K ? q4k_unit(blk, aq, am) : q6k_unit(blk, aq, am);
                    } else {
                        const size_t offq = (size_t)row * p.K + (size_t)c * C * 32;
                        const size_t offs = (size_t)row * (p.K / 8) + (size_t)c * C * 4;
                        const uint8_t *wq = stage + rs * L.q_stride + (offq & 15) + 32 * m;
                        const float ws = *reinterpret_cast<const float *>(stage + L.s_region + rs * L.s_stride +
                                                                          (offs & 15) + 4 * m);
                        t = q80_unit(wq, ws, smem + L.act_q_off + j * kQ80ActStride);
                    }
                    tb[rs * C + m] = t;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&done[s]);
        }
        return;
    }

    // ------------------------------------------------------ row warp
    const int G = kq ? nb : p.q8_group;
    const bool grouped = G < nb;
    unsigned long long best = 0ull;
    float sum = 0.0f, grp = 0.0f, acc = 0.0f;  // lane r: running sums of row slot r
    int gpos = 0;
    GroupRef g{0, 0, 0};
    for (int it = 0; it < items; ++it) {
        const int s = it % p.stages;
        const int c = it % p.nchunks;
        if (c == 0) g = locate(p, blockIdx.x + (it / p.nchunks) * gridDim.x);
        if (!mbar_wait_bounded(&done[s], (uint32_t)((it / p.stages) & 1))) break;
        int seg = 0, row = 0;
        const bool valid = lane < T && slot_row(p, g, lane, &seg, &row);
        const int cc = min(C, nb - c * C);
        const float *tb = tbuf + (size_t)s * T * C;
        if (lane < T) {
            if (c == 0) {
                sum = 0.0f;
                grp = 0.0f;
                gpos = 0;
                acc = (valid && p.seg[seg].bias) ? p.seg[seg].bias[row] : 0.0f;
            }
            const float *tr = tb + lane * C;
            for (int m = 0; m < cc; ++m) {
                const float v = tr[m];
                if (grouped) {
                    grp = gpos == 0 ? fadd(0.0f, v) : fadd(grp, v);
                    if (++gpos == G) {
                        acc = fadd(acc, grp);
                        gpos = 0;
                    }
                } else {
                    sum = fadd(sum, v);
                }
            }
        }
        __syncwarp();
        // The stage and its terms are consumed: refill with item it + stages.
        const int nx = it + p.stages;
        if (nx < items) {
            if (lane == 0) fence_proxy_async_smem();
            __syncwarp();
            const GroupRef gn = locate(p, blockIdx.x + (nx / p.nchunks) * gridDim.x);
            issue_stage(p, L, gn, nx % p.nchunks, ring + (size_t)s * L.stage_bytes, &full[s], pol, lane);
        }
        if (c == p.nchunks - 1) {
            float y;
            if (grouped) y = acc;
            else y = (valid && p.seg[seg].bias) ? fadd(p.seg[seg].bias[row], sum) : sum;
            if (p.epi == EPI_SILU_PAIR) {
                const int half = T / 2;
                const float u = __shfl_down_sync(0xFFFFFFFFu, y, half);
                if (lane < half && valid) {
                    const float sg = fdiv(1.0f, fadd(1.0f, expf(-y)));
                    p.seg[0].out[row] = fmul(fmul(y, sg), u);
                }
            } else if (valid) {
                float *out = p.seg[seg].out;
                if (p.epi == EPI_RESIDUAL) out[row] = fadd(p.resid[row], y);
                else out[row] = y;
                if (p.epi == EPI_LOGITS_ARGMAX) {
                    const unsigned long long kk = argmax_key(y, row);
                    best = kk > best ? kk : best;
                }
            }
        }
    }

    if (p.epi == EPI_LOGITS_ARGMAX) {
        // the row warp holds the CTA's rows: warp max -> one global atomic per
        // CTA; the last CTA to finish turns the winning key into the next token.
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) {
            atomicMax(&p.step->argmax_key, best);
            __threadfence();
            const int ticket = atomicAdd(&p.step->done_ctas, 1);
            if (ticket == (int)gridDim.x - 1) {
                __threadfence();
                const unsigned long long k = atomicAdd(&p.step->argmax_key, 0ull);
                const int idx = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
                p.step->token = idx;
                if (p.tokens_out) p.tokens_out[p.step->n_generated] = idx;
                p.step->n_generated += 1;
                p.step->argmax_key = 0ull;
                p.step->done_ctas = 0;
                __threadfence();
            }
        }
    }
}

// ---------------------------------------------------------------- host side
int sm_count(int device) {
    static int cached[64] = {0};
    if (device < 0 || device >= 64) return 148;
    if (!cached[device]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
        cached[device] = v > 0 ? v : 148;
    }
    return cached[device];
}

static int smem_optin(int device) {
    static int cached[64] = {0};
    if (device < 0 || device >= 64) return 227 * 1024;
    if (!cached[device]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        cached[device] = v > 0 ? v : 227 * 1024;
    }
    return cached[device];
}

ovf_status gemv_launch(GemvParams p, cudaStream_t stream, bool pdl, GemvPlan *plan_out) {
    OVF_CHECK_ARG(p.nseg >= 1 && p.nseg <= 3, "gemv: 1..3 weight segments");
    const int type0 = p.seg[0].type;
    const bool kq = is_kquant(type0);
    OVF_CHECK_ARG(kq || type0 == OVF_TYPE_Q8_0, "gemv: unsupported weight type %d", type0);
    for (int s = 0; s < p.nseg; ++s) {
        OVF_CHECK_ARG(is_kquant(p.seg[s].type) == kq, "gemv: K-quant and Q8_0 segments cannot share a launch");
        OVF_CHECK_ARG(p.seg[s].w && aligned16(p.seg[s].w), "gemv: weight pointer must be non-null and 16-byte aligned");
        OVF_CHECK_ARG(kq || (p.seg[s].ws && aligned16(p.seg[s].ws)), "gemv: Q8_0 scales must be 16-byte aligned");
        OVF_CHECK_ARG(p.seg[s].out, "gemv: output pointer is null");
        OVF_CHECK_ARG(p.seg[s].rows >= 0, "gemv: negative rows");
    }
    OVF_CHECK_ARG(p.K > 0 && (kq ? p.K % 256 == 0 : p.K % 32 == 0), "gemv: K=%d must be a multiple of %d", p.K,
                  kq ? 256 : 32);
    if (p.act_mode == ACT_PREQ_Q8K) {
        OVF_CHECK_ARG(kq, "gemv: pre-quantized Q8_K activations need K-quant weights");
        OVF_CHECK_ARG(p.aq && p.as && p.ab && aligned16(p.aq), "gemv: pre-quantized activation buffers");
    } else {
        OVF_CHECK_ARG(p.x && aligned16(p.x), "gemv: x must be non-null and 16-byte aligned");
    }
    if (p.pair)
        OVF_CHECK_ARG(p.nseg == 2 && p.seg[0].rows == p.seg[1].rows && p.seg[0].type == p.seg[1].type &&
                          p.epi == EPI_SILU_PAIR,
                      "gemv: pair mode needs 2 segments of equal shape and type");
    if (p.epi == EPI_RESIDUAL) OVF_CHECK_ARG(p.resid != nullptr, "gemv: residual epilogue without residual");
    if (p.epi == EPI_LOGITS_ARGMAX) OVF_CHECK_ARG(p.step != nullptr, "gemv: argmax epilogue without step state");

    int device = 0;
    OVF_CUDA_TRY(cudaGetDevice(&device));
    const int nsm = sm_count(device);
    const int nb = kq ? p.K / 256 : p.K / 32;
    if (!kq && p.q8_group <= 0) p.q8_group = nb;
    OVF_CHECK_ARG(kq || nb % p.q8_group == 0, "gemv: Q8_0 group must divide the block count");
    // Whole-row tiles of T rows (~40 KB of weights, up to 16 rows; pair
    // launches take T/2 gate + T/2 up rows): one bulk copy per matrix per
    // stage.  OVF_GEMV_C selects the per-row chunked mode instead.
    int T = 16, C = nb;
    int rb = 0;
    for (int s = 0; s < p.nseg; ++s) rb = std::max(rb, kq ? nb * kq_block_bytes(p.seg[s].type) : p.K + p.K / 8);
    T = (int)std::max<int64_t>(1, std::min<int64_t>(16, (40 * 1024) / rb));
    if (p.pair) T = std::max(2, T & ~1);
    if (const char *e = getenv("OVF_GEMV_T")) T = std::max(1, std::min(32, atoi(e)));
    if (const char *e = getenv("OVF_GEMV_C")) if (atoi(e) > 0) C = std::max(1, std::min(nb, atoi(e)));
    p.copy_split = 1;
    if (const char *e = getenv("OVF_GEMV_SPLIT")) p.copy_split = std::max(1, std::min(16, atoi(e)));
    OVF_CHECK_ARG(T * C <= 32 * 128, "gemv: tile too large");
    p.rows_per_group = T;
    p.chunk = C;
    p.nchunks = (nb + C - 1) / C;
    p.lanes_per_row = 1;
    p.units_per_lane = 1;
    const int rows_per = p.pair ? T / 2 : T;
    int total = 0;
    for (int s = 0; s < p.nseg; ++s) {
        p.seg[s].groups = (p.seg[s].rows + rows_per - 1) / rows_per;
        if (!p.pair) total += p.seg[s].groups;
    }
    if (p.pair) total = p.seg[0].groups;
    p.total_groups = total;
    if (total == 0) return OVF_OK;

    const int budget = smem_optin(device) - 1024;
    const int grid = std::min(nsm, total);
    const int warps = kComputeWarps + 1;
    int stages = 0;
    size_t smem = 0;
    int s_hi = 6, s_lo = 2;
    if (const char *e = getenv("OVF_GEMV_S")) s_hi = s_lo = std::max(2, std::min(8, atoi(e)));
    if (const char *e = getenv("OVF_GEMV_SKIP")) p.skip_compute = atoi(e);
    for (int S = s_hi; S >= s_lo; --S) {
        p.stages = S;
        const Layout L = make_layout(p);
        if (layout_smem(L, S) <= (size_t)budget) {
            stages = S;
            smem = layout_smem(L, S);
            break;
        }
    }
    OVF_CHECK_ARG(stages >= 2, "gemv: K=%d does not fit shared memory", p.K);
    p.stages = stages;
    static bool attr_done[64] = {false};
    if (device < 64 && !attr_done[device]) {
        OVF_CUDA_TRY(cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          smem_optin(device)));
        attr_done[device] = true;
    }
    if (plan_out) *plan_out = GemvPlan{T, p.chunk, stages, warps, grid, smem};
    cudaError_t e = launch_pdl(gemv_kernel, dim3(grid), dim3(warps * 32), smem, stream, pdl, p);
    if (e != cudaSuccess) return cuda_status(e, "gemv_kernel launch");
    return OVF_OK;
}

}  // namespace ovf
