// ovf_gemv.cu — quantized decode GEMV for sm_100a (see ovf_gemv.cuh).
//
// Work decomposition.  The rows of a launch (up to three weight segments,
// e.g. Q/K/V, or a gate/up pair) are cut into tiles of T whole rows; each
// CTA (one per SM, persistent) takes tiles blockIdx.x, blockIdx.x + grid, ...
// A tile's rows are contiguous in HBM, so one 1-D bulk copy (the TMA engine)
// per matrix part fills a shared-memory stage; a ring of stages keeps
// several copies in flight.  A dedicated producer thread does nothing but
// wait for a free stage and issue its copies, so the copy engine is never
// starved by arithmetic; the first stages are requested before
// griddepcontrol.wait, while the previous kernel of the decode step is
// still finishing (programmatic dependent launch).
//
// Six compute warps contract a stage with dp4a: one thread per (row,
// block), each thread holding the quantized activation of its block (Q8_K
// or Q8_0, quantized in the prologue, optionally after RMSNorm) in
// registers for the whole launch.  A sum warp then adds each row's terms in
// ascending block order — the reference's sequential fp32 loop
// (Runtime/Q4KDotKernel.cs:528-552, Q6KDotKernel.cs:364-380,
// Q8DotKernel.cs:311-328) — and runs the fused epilogue, overlapped with
// the next tiles' contraction.  Integer parts are exact and the fp32 tails
// use explicitly rounded ops in the reference's operand order, so results
// are bit-identical to it.
//
// Spans are copied from the 16-byte boundary at or below their first byte
// (Q6_K blocks are 210 bytes), so a row may start 4/8/12 bytes into its
// stage; the Q6_K unit reads through a funnel shift.  A copy that would run
// past the end of the weight buffer stops at the last 16-byte boundary and
// its last few bytes are stored by the producer thread itself.
#include "ovf_gemv.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>

namespace ovf {

static constexpr int kQ8kActStride = 272;  // 256 quants + 16 pad
static constexpr int kQ8kMetaStride = 64;  // int16 bsums[16] | f32 scale | pad | int16 pair sums[8]
static constexpr int kQ80ActStride = 48;   // 32 quants + f32 scale + pad
static constexpr int kTermBufs = 4;        // term buffers between the compute warps and the sum warp

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

struct Layout {
    int act_q_off, act_meta_off, red_off, terms_off, stage_off;
    int stage_bytes;
    int part_bytes;  // quants of one matrix part of a stage (16 bytes of slack for an unaligned start)
    int s_region;    // Q8_0: offset of the scales parts in a stage
    int s_part;      // Q8_0: scales of one matrix part
    int nb;          // blocks per row
};

// Shared memory: mbarriers | activation | reduction scratch | kTermBufs
// term buffers [T][nb] | stage ring.  A stage holds one tile: the tile's rows of
// each matrix part (pair launches: gate part, up part), copied as one
// contiguous span each; Q8_0 stages append the parts' fp32 scale spans.
// Parts are sized for the launch's largest row (K-quant launches may mix
// Q4_K and Q6_K segments).
static __host__ __device__ inline int row_bytes(int type, int K) {
    return is_kquant(type) ? (K / 256) * kq_block_bytes(type) : K;
}

static __host__ __device__ inline Layout make_layout(const GemvParams &p) {
    Layout L{};
    const bool kq = is_kquant(p.seg[0].type);
    L.nb = kq ? p.K / 256 : p.K / 32;
    const int T = p.rows_per_group;
    size_t off = align_up(sizeof(uint64_t) * (2 * p.stages + 2 * kTermBufs) + 16, 128);
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
    off = align_up(off + (size_t)kTermBufs * T * L.nb * sizeof(float), 128);
    L.stage_off = (int)off;
    const int parts = p.pair ? 2 : 1, per = T / parts;
    int rb = 0;
    for (int s = 0; s < p.nseg; ++s) rb = max(rb, row_bytes(p.seg[s].type, p.K));
    L.part_bytes = (int)align_up((size_t)per * rb + 16, 16);
    L.s_region = parts * L.part_bytes;
    L.s_part = kq ? 0 : (int)align_up((size_t)per * (p.K / 8) + 16, 16);
    L.stage_bytes = (int)align_up((size_t)L.s_region + (size_t)parts * L.s_part, 128);
    return L;
}

static __host__ __device__ inline size_t layout_smem(const Layout &L, int stages) {
    return (size_t)L.stage_off + (size_t)stages * L.stage_bytes;
}

// ------------------------------------------------------------- dot units
// One thread contracts one block of a row: a K-quant super-block (256
// weights, activation block read from shared memory) or a Q8_0 block (32;
// the activation block is kept in registers for the whole launch).  The
// integer parts are exact and the fp32 tail of every block follows the
// reference's operand order.
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

struct Q8Act {        // Q8_0 block: 32 quants + scale
    uint32_t q[8];
    float s;
};

__device__ __forceinline__ void load_q8_act(const uint8_t *act, Q8Act &a) {
    const uint4 v0 = *reinterpret_cast<const uint4 *>(act);
    const uint4 v1 = *reinterpret_cast<const uint4 *>(act + 16);
    a.q[0] = v0.x; a.q[1] = v0.y; a.q[2] = v0.z; a.q[3] = v0.w;
    a.q[4] = v1.x; a.q[5] = v1.y; a.q[6] = v1.z; a.q[7] = v1.w;
    a.s = *reinterpret_cast<const float *>(act + 32);
}

// 32-bit word `w` of a block that may start 2 bytes past a word boundary.
__device__ __forceinline__ uint32_t ldw_shifted(const uint32_t *base, int w, int sh) {
    return __funnelshift_r(base[w], base[w + 1], sh);
}

// Q8_0 x Q8_0 over one 32-block (Runtime/Q8DotKernel.cs:99-140).
__device__ __forceinline__ float q80_block(const uint8_t *wq, float ws, const Q8Act &a) {
    const uint4 w0 = *reinterpret_cast<const uint4 *>(wq);
    const uint4 w1 = *reinterpret_cast<const uint4 *>(wq + 16);
    int dot = 0;
    dot = dp4a((int)w0.x, (int)a.q[0], dot);
    dot = dp4a((int)w0.y, (int)a.q[1], dot);
    dot = dp4a((int)w0.z, (int)a.q[2], dot);
    dot = dp4a((int)w0.w, (int)a.q[3], dot);
    dot = dp4a((int)w1.x, (int)a.q[4], dot);
    dot = dp4a((int)w1.y, (int)a.q[5], dot);
    dot = dp4a((int)w1.z, (int)a.q[6], dot);
    dot = dp4a((int)w1.w, (int)a.q[7], dot);
    return fmul(fmul(ws, a.s), i2f(dot));
}

// Shared-memory-activation forms of the block dots (the activation block is
// read from shared memory for every row).
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
        for (int is = 0; is < 2; ++is) {
            // the four 16-element groups sharing scales sc[8h+is+{0,2,4,6}]:
            // integer dots first, one scale multiply per group
            int d1 = 0, d2 = 0, d3 = 0, d4 = 0;
#pragma unroll
            for (int l4 = 0; l4 < 4; ++l4) {
                const int lw = 4 * is + l4;
                const uint32_t qla = ldw_shifted(base, 16 * h + lw, sh);
                const uint32_t qlb = ldw_shifted(base, 16 * h + 8 + lw, sh);
                const uint32_t qhw = ldw_shifted(base, 32 + 8 * h + lw, sh);
                const uint32_t M = 0x0F0F0F0Fu, H = 0x30303030u;
                const int q1 = (int)((qla & M) | ((qhw << 4) & H));
                const int q2 = (int)((qlb & M) | ((qhw << 2) & H));
                const int q3 = (int)(((qla >> 4) & M) | (qhw & H));
                const int q4 = (int)(((qlb >> 4) & M) | ((qhw >> 2) & H));
                const int base8 = 32 * h + lw;
                d1 = dp4a(q1, (int)q8w[base8], d1);
                d2 = dp4a(q2, (int)q8w[base8 + 8], d2);
                d3 = dp4a(q3, (int)q8w[base8 + 16], d3);
                d4 = dp4a(q4, (int)q8w[base8 + 24], d4);
            }
            sum += sc[8 * h + is] * d1 + sc[8 * h + is + 2] * d2 + sc[8 * h + is + 4] * d3 + sc[8 * h + is + 6] * d4;
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

// Activation prologue, Q8_K form.  Every lane first issues the loads of all
// its elements (independent 16-byte loads, one memory round trip), applies
// RMSNorm as (x * scale) * gamma with the scale its producer computed in the
// reference's order (Runtime/CachedTransformerBlock.cs:525-552), and
// quantizes per 256 (Runtime/Q4KDotKernel.cs:71-136).
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
    const bool norm = p.act_mode == ACT_F32_RMSNORM;
    const bool write_out = blockIdx.x == 0 && p.aq_out != nullptr;
    constexpr int MB = 4;  // blocks per warp held in registers per batch
    const float s = norm ? *p.norm_scale : 1.0f;
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
    const bool norm = p.act_mode == ACT_F32_RMSNORM;
    const bool write_out = blockIdx.x == 0 && p.aq_out != nullptr;
    constexpr int MB = 16;
    const int nb = L.nb;
    const float s = norm ? *p.norm_scale : 1.0f;
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

// Stages bytes [off, off+len) of `src` (a buffer of `total` bytes) at
// dst + (off & 15).  The bulk engine moves the whole 16-byte units from the
// boundary at or below `off`; the bytes past the buffer's last 16-byte
// boundary (only a segment's final tile can have them) are stored by the
// thread itself.  `bulk` false: store those tail bytes and return the bulk
// byte count; `bulk` true: issue the bulk copy.
__device__ __forceinline__ uint32_t copy_span(uint8_t *dst, const uint8_t *src, size_t off, size_t len, size_t total,
                                              uint64_t *bar, uint64_t pol, bool bulk) {
    const size_t a = off & ~size_t(15);
    const size_t e = min(align_up(off + len, 16), total);
    const size_t be = e & ~size_t(15);
    const uint32_t n = be > a ? (uint32_t)(be - a) : 0u;
    if (!bulk) {
        for (size_t i = max(a, be); i < e; ++i) dst[i - a] = src[i];
    } else if (n) {
        bulk_g2s(dst, src + a, n, bar, pol);
    }
    return n;
}

// Fills one stage with tile `g`; run by the producer thread alone.  Pass 0
// stores the tail bytes and counts the bulk bytes, the arrive (which
// releases those stores) announces the transaction count, pass 1 issues the
// copies.
__device__ __forceinline__ void issue_stage(const GemvParams &p, const Layout &L, const GroupRef &g, uint8_t *stage,
                                            uint64_t *bar, uint64_t pol, size_t eoff_w = 0, size_t eoff_s = 0) {
    const int parts = p.pair ? 2 : 1;
    uint32_t bytes = 0;
    for (int pass = 0; pass < 2; ++pass) {
        const bool bulk = pass == 1;
        for (int part = 0; part < parts && g.nr > 0; ++part) {
            const GemvSeg &sg = p.seg[p.pair ? part : g.seg];
            const size_t rb = (size_t)row_bytes(sg.type, p.K);
            bytes += copy_span(stage + part * L.part_bytes, sg.w + eoff_w, (size_t)g.r0 * rb, (size_t)g.nr * rb,
                               (size_t)sg.rows * rb, bar, pol, bulk);
            if (!is_kquant(sg.type)) {
                const size_t sb = (size_t)(p.K / 8);
                bytes += copy_span(stage + L.s_region + part * L.s_part,
                                   reinterpret_cast<const uint8_t *>(sg.ws) + eoff_s,
                                   (size_t)g.r0 * sb, (size_t)g.nr * sb, (size_t)sg.rows * sb, bar, pol, bulk);
            }
        }
        if (!bulk) mbar_arrive_expect_tx(bar, bytes);
    }
}

// ------------------------------------------------------------------ kernel
// A CTA owns T-row tiles (persistent: tile = blockIdx.x + i * gridDim.x) and
// streams each through a ring of `stages` shared-memory buffers.  Three
// warp roles run decoupled, linked only by mbarriers:
//   producer (last warp, one lane): waits for a free stage, issues its bulk
//     copies, nothing else — the copy engine is never starved by arithmetic;
//   compute warps: contract a stage into a [T][nb] term buffer (one thread
//     per (row, block)), release the stage and hand the terms on;
//   sum warp: lane r adds row slot r's terms in ascending block order — the
//     reference's sequential fp32 loop — and runs the epilogue, while the
//     compute warps already work on the next tiles (kTermBufs buffers).
// Defaults measured on B200 over the Llama-3-8B decode step (compute warps x
// CTAs per SM x tile KB): 4x3x16 252.6 tok/s, 8x2x32 275.7, 16x1x64 289.0,
// 20x1x64 285.3, 24x1x64 276.2, 16x1x96 287.6 — one wide CTA per SM with
// 64 KB tiles keeps the most bytes in flight per SM.
#ifndef OVF_GEMV_CW
#define OVF_GEMV_CW 16
#endif
static constexpr int kComputeWarps = OVF_GEMV_CW;
#ifndef OVF_GEMV_CTAS
#define OVF_GEMV_CTAS 1
#endif
static constexpr int kCtasPerSm = OVF_GEMV_CTAS;
#ifndef OVF_GEMV_TILE_KB
#define OVF_GEMV_TILE_KB 64
#endif
static constexpr int kComputeThreads = kComputeWarps * 32;
// The compute warps may form kGroups groups that take alternate tiles (a
// CTA then contracts kGroups tiles at once).  Measured on B200 the
// contraction is issue-bound rather than latency-bound, and two groups were
// slower, so one group is the default.
#ifndef OVF_GEMV_GROUPS
#define OVF_GEMV_GROUPS 1
#endif
static constexpr int kGroups = OVF_GEMV_GROUPS;
static constexpr int kGroupWarps = kComputeWarps / kGroups;
static constexpr int kGroupThreads = kGroupWarps * 32;
static_assert(kComputeWarps % kGroups == 0 && kTermBufs % kGroups == 0, "compute groups");
static constexpr int kSumWarp = kComputeWarps;
static constexpr int kProducerWarp = kComputeWarps + 1;
static constexpr int kThreads = (kComputeWarps + 2) * 32;

struct Bars {
    uint64_t *full, *empty, *tready, *tfree;
    volatile int *abort_flag;
};

__device__ __forceinline__ Bars bars_of(uint8_t *smem, int stages) {
    Bars b;
    b.full = reinterpret_cast<uint64_t *>(smem);
    b.empty = b.full + stages;
    b.tready = b.empty + stages;
    b.tfree = b.tready + kTermBufs;
    b.abort_flag = reinterpret_cast<volatile int *>(b.tfree + kTermBufs);
    return b;
}

// Bounded wait that gives up for good once any wait of the CTA has failed.
__device__ __forceinline__ void wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (*abort_flag) return;
    if (!mbar_wait_sleep_bounded(bar, parity)) *abort_flag = 1;
}

// RMSNorm of a residual output (EPI_RESIDUAL with norm_out): CTA 0 takes no
// tiles; it walks the output rows in index order and keeps the reference's
// sequential fp32 sum of squares, and the scale it leaves in norm_out spares
// every CTA of the consuming kernel a reduction and reproduces the
// reference's RmsNormalize bit for bit.  The output buffer holds the
// kNormSentinel pattern before this launch (an earlier kernel of the step
// fills it), so the norm CTA knows a row has been written when its value is
// no longer the sentinel: the tile CTAs publish nothing and pay no fences.
// The norm CTA stages 1024 squares at a time (warps 1..) while thread 0 adds
// the previous 1024 in order, so the chain trails the GEMV closely.
__device__ __noinline__ void norm_cta(const GemvParams &p, float *stage) {
    __shared__ int s_fail;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int rows = p.seg[0].rows;
    const int nchunks = (rows + 1023) / 1024;
    const float *out = p.seg[0].out;
    if (tid == 0) s_fail = 0;
    __syncthreads();
    // warps 1..: load chunk c once every row of it has been written
    auto stage_chunk = [&](int c, int buf) {
        const int r0 = 1024 * c, n = min(1024, rows - r0);
        float *dst = stage + buf * 1024;
        for (int i = tid - 32; i < n; i += nt - 32) {
            float v = __ldcg(out + r0 + i);
            for (uint32_t k = 0; __float_as_uint(v) == kNormSentinel && k < (1u << 22); ++k) {
                __nanosleep(64);
                v = __ldcg(out + r0 + i);
            }
            if (__float_as_uint(v) == kNormSentinel) s_fail = 1;
            dst[i] = fmul(v, v);
        }
    };
    if (tid >= 32) stage_chunk(0, 0);
    __syncthreads();
    float acc = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
        if (tid == 0) {
            // the reference's sequential sum over this chunk, 32 squares in
            // registers ahead of the dependent adds
            const int m = min(1024, rows - 1024 * c), m32 = m & ~31;
            const float *sv = stage + (c & 1) * 1024;
            const float4 *s4 = reinterpret_cast<const float4 *>(sv);
            float4 cur[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) cur[j] = m32 ? s4[j] : make_float4(0.f, 0.f, 0.f, 0.f);
            for (int i = 0; i < m32; i += 32) {
                float4 nxt[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) nxt[j] = i + 32 < m32 ? s4[(i + 32) / 4 + j] : cur[j];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    acc = fadd(acc, cur[j].x);
                    acc = fadd(acc, cur[j].y);
                    acc = fadd(acc, cur[j].z);
                    acc = fadd(acc, cur[j].w);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
            }
            for (int i = m32; i < m; ++i) acc = fadd(acc, sv[i]);
        } else if (tid >= 32 && c + 1 < nchunks) {
            stage_chunk(c + 1, (c + 1) & 1);
        }
        __syncthreads();
    }
    if (tid == 0) {
        if (s_fail) raise_dev_error(DEVERR_COUNTER);
        *p.norm_out = s_fail ? __int_as_float(0x7FC00000) : rms_scale(acc, rows, p.eps);
    }
}

template <bool KQ, int BPS>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const Layout L = make_layout(p);
    const Bars B = bars_of(smem, p.stages);
    uint8_t *ring = smem + L.stage_off;
    float *tbuf = reinterpret_cast<float *>(smem + L.terms_off);
    const int T = p.rows_per_group, nb = L.nb;
    // With an output RMSNorm, CTA 0 only runs the norm chain and the others
    // take the tiles: tile = tcta + i * tgrid.
    const int nfirst = p.norm_out ? 1 : 0;
    const int tgrid = (int)gridDim.x - nfirst, tcta = (int)blockIdx.x - nfirst;
    const int items = tcta >= 0 && tcta < p.total_groups ? (p.total_groups - tcta + tgrid - 1) / tgrid : 0;

    if (tid == 0) trace_mark(p.trace, TR_START);
    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&B.full[s], 1);
            mbar_init(&B.empty[s], kGroupWarps);  // stage s always serves the same group
        }
        for (int j = 0; j < kTermBufs; ++j) {
            mbar_init(&B.tready[j], kGroupWarps);
            mbar_init(&B.tfree[j], 1);
        }
        *B.abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    uint64_t pol = 0;
    // Weights do not depend on the previous kernel: start streaming now
    // (a routed expert's weights only once the routing is known).
    const bool routed = p.expert_sel != nullptr;
    if (warp == kProducerWarp && lane == 0) {
        pol = l2_evict_first_policy();
        if (!routed)
            for (int it = 0; it < p.stages && it < items; ++it)
                issue_stage(p, L, locate(p, tcta + it * tgrid), ring + (size_t)it * L.stage_bytes, &B.full[it],
                            pol);
    }

    pdl_wait();
    size_t eoff_w = 0, eoff_s = 0;
    if (routed) {
        int e = p.expert_sel[p.expert_slot];
        if (p.expert_mod > 1) {
            // expert parallel: another rank owns this expert
            if (e % p.expert_mod != p.expert_rank) {
                pdl_launch_dependents();
                if (tid == 0) trace_mark(p.trace, TR_END);
                return;
            }
            e /= p.expert_mod;
        }
        eoff_w = (size_t)e * (size_t)p.expert_wstride;
        eoff_s = (size_t)e * (size_t)p.expert_sstride;
        if (warp == kProducerWarp && lane == 0)
            for (int it = 0; it < p.stages && it < items; ++it)
                issue_stage(p, L, locate(p, tcta + it * tgrid), ring + (size_t)it * L.stage_bytes, &B.full[it],
                            pol, eoff_w, eoff_s);
    }
    if (tid == 0) trace_mark(p.trace, TR_WAITED);
    if (p.fill_sentinel) {
        // mark the buffer a later residual launch of this step will write
        // (its norm CTA waits for the marks to be overwritten)
        for (int i = blockIdx.x * blockDim.x + tid; i < p.fill_n; i += gridDim.x * blockDim.x)
            p.fill_sentinel[i] = __uint_as_float(kNormSentinel);
    }
    if (KQ) prep_q8k(p, L, smem);
    else prep_q80(p, L, smem);
    __syncthreads();
    // The dependent grid may launch once every CTA of this one has passed
    // this point, i.e. once all of them are resident: its CTAs then take
    // only the slots that finished CTAs free, stream their first weight
    // stages and wait at griddepcontrol.wait for this grid (and its norm
    // chain) to complete.
    pdl_launch_dependents();
    if (p.norm_out && blockIdx.x == 0) {
        norm_cta(p, reinterpret_cast<float *>(ring));
        if (tid == 0) trace_mark(p.trace, TR_END);
        return;
    }

    if (warp == kProducerWarp) {
        // ------------------------------------------------------- producer
        if (lane != 0) return;
        for (int it = p.stages; it < items; ++it) {
            const int s = it % p.stages;
            wait_or_abort(&B.empty[s], (uint32_t)(((it / p.stages) - 1) & 1), B.abort_flag);
            if (*B.abort_flag) break;
            fence_proxy_async_smem();
            issue_stage(p, L, locate(p, tcta + it * tgrid), ring + (size_t)s * L.stage_bytes, &B.full[s],
                        pol, eoff_w, eoff_s);
        }
        if (p.pf.n) prefetch_l2_slice(p.pf, blockIdx.x, gridDim.x);
        trace_mark(p.trace, TR_END);
        return;
    }

    const int half = p.pair ? T / 2 : T;
    if (warp == kSumWarp) {
        // ------------------------------------------------------- sum warp
        const int G = KQ ? nb : p.q8_group;
        const bool grouped = G < nb;
        const int nslots = half;  // pair mode: slot r sums gate row r and up row r
        unsigned long long best = 0ull;
        for (int it = 0; it < items; ++it) {
            const int j = it % kTermBufs;
            const GroupRef g = locate(p, tcta + it * tgrid);
            for (int slot = lane; slot < ((nslots + 31) & ~31); slot += 32) {
                int seg = 0, row = 0;
                const bool valid = slot < nslots && slot_row(p, g, slot, &seg, &row);
                // epilogue operands first: their latency overlaps the wait
                const bool hb0 = valid && p.seg[seg].bias != nullptr;
                const float b0 = hb0 ? p.seg[seg].bias[row] : 0.0f;
                const bool hb1 = valid && p.pair && p.seg[1].bias != nullptr;
                const float b1 = hb1 ? p.seg[1].bias[row] : 0.0f;
                const float res = valid && p.epi == EPI_RESIDUAL ? p.resid[row] : 0.0f;
                if (slot == lane) wait_or_abort(&B.tready[j], (uint32_t)((it / kTermBufs) & 1), B.abort_flag);
                __syncwarp();
                if (!valid) continue;
                const float *tb = tbuf + (size_t)j * T * nb;
                if (p.epi == EPI_TERMS_TP) {
                    // every block term of the row to every rank, block-major
                    const float *tr = tb + (size_t)slot * nb;
                    for (int m = 0; m < nb; ++m) {
                        const float v = tr[m];
                        const size_t o = (size_t)(p.tp_index0 + m) * p.tp_rows + row;
                        for (int w = 0; w < p.tp_world; ++w) p.tp_dst[w][o] = v;
                    }
                    continue;
                }
                float y[2] = {0.0f, 0.0f};
                for (int k = 0; k < (p.pair ? 2 : 1); ++k) {
                    const float *tr = tb + (size_t)(slot + k * half) * nb;
                    const bool hb = k == 0 ? hb0 : hb1;
                    const float bv = k == 0 ? b0 : b1;
                    if (grouped) {
                        // head-ordered sum: each group of G blocks summed in
                        // order, the group sums added in order on the bias
                        float acc = hb ? bv : 0.0f, grp = 0.0f;
                        int gp = 0, gi = 0;
                        const bool to_ranks = p.epi == EPI_GROUPS_TP;
                        int m = 0;
                        for (; m + 8 <= nb; m += 8) {
                            float v[8];
#pragma unroll
                            for (int q = 0; q < 8; ++q) v[q] = tr[m + q];
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                grp = gp == 0 ? fadd(0.0f, v[q]) : fadd(grp, v[q]);
                                if (++gp == G) {
                                    if (to_ranks) {
                                        const size_t o = (size_t)(p.tp_index0 + gi) * p.tp_rows + row;
                                        for (int w = 0; w < p.tp_world; ++w) p.tp_dst[w][o] = grp;
                                    }
                                    acc = fadd(acc, grp);
                                    gp = 0;
                                    ++gi;
                                }
                            }
                        }
                        for (; m < nb; ++m) {
                            grp = gp == 0 ? fadd(0.0f, tr[m]) : fadd(grp, tr[m]);
                            if (++gp == G) {
                                if (to_ranks) {
                                    const size_t o = (size_t)(p.tp_index0 + gi) * p.tp_rows + row;
                                    for (int w = 0; w < p.tp_world; ++w) p.tp_dst[w][o] = grp;
                                }
                                acc = fadd(acc, grp);
                                gp = 0;
                                ++gi;
                            }
                        }
                        y[k] = acc;
                    } else {
                        float sum = 0.0f;
                        int m = 0;
                        for (; m + 8 <= nb; m += 8) {
                            float v[8];
#pragma unroll
                            for (int q = 0; q < 8; ++q) v[q] = tr[m + q];
#pragma unroll
                            for (int q = 0; q < 8; ++q) sum = fadd(sum, v[q]);
                        }
                        for (; m < nb; ++m) sum = fadd(sum, tr[m]);
                        if (p.epi == EPI_GROUPS_TP) {  // one group: the whole row
                            const size_t o = (size_t)p.tp_index0 * p.tp_rows + row;
                            for (int w = 0; w < p.tp_world; ++w) p.tp_dst[w][o] = sum;
                        }
                        y[k] = hb ? fadd(bv, sum) : sum;
                    }
                }
                if (p.epi == EPI_SILU_PAIR) {
                    const float sg = fdiv(1.0f, fadd(1.0f, exp_libm(-y[0])));
                    p.seg[0].out[row] = fmul(fmul(y[0], sg), y[1]);
                } else if (p.epi == EPI_LOGITS_TP) {
                    const int grow = p.tp_index0 + row;
                    for (int w = 0; w < p.tp_world; ++w) p.tp_dst[w][grow] = y[0];
                    const unsigned long long kk = argmax_key(y[0], grow);
                    best = kk > best ? kk : best;
                } else if (p.epi == EPI_ROWS_TP) {
                    const size_t o = (size_t)p.tp_index0 * p.tp_rows + row;
                    for (int w = 0; w < p.tp_world; ++w) p.tp_dst[w][o] = y[0];
                } else if (p.epi != EPI_GROUPS_TP) {
                    float *out = p.seg[seg].out;
                    if (p.epi == EPI_RESIDUAL) out[row] = fadd(res, y[0]);
                    else out[row] = y[0];
                    if (p.epi == EPI_LOGITS_ARGMAX) {
                        const unsigned long long kk = argmax_key(y[0], row);
                        best = kk > best ? kk : best;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.tfree[j]);
        }
        if (p.epi >= EPI_GROUPS_TP) __threadfence_system();  // the peers' copies before the kernel ends
        if (p.epi == EPI_LOGITS_TP) {
            // warp max -> one global atomic per CTA; the last CTA to finish
            // publishes this rank's winning key to every rank
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best, o);
                best = other > best ? other : best;
            }
            if (lane == 0) {
                if (best) atomicMax(&p.step->argmax_key, best);
                __threadfence();
                const int ticket = atomicAdd(&p.step->done_ctas, 1);
                if (ticket == (int)gridDim.x - 1) {
                    __threadfence();
                    const unsigned long long k = atomicAdd(&p.step->argmax_key, 0ull);
                    for (int w = 0; w < p.tp_world; ++w) p.tp_keys[w][p.tp_rank] = k;
                    p.step->argmax_key = 0ull;
                    p.step->done_ctas = 0;
                    __threadfence_system();
                }
            }
        }
        if (p.epi == EPI_LOGITS_ARGMAX) {
            // warp max -> one global atomic per CTA; the last CTA to finish
            // turns the winning key into the next token.
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best, o);
                best = other > best ? other : best;
            }
            if (lane == 0) {
                if (best) atomicMax(&p.step->argmax_key, best);
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
        if (lane == 0) trace_mark(p.trace, TR_END);
        if (lane == 0) trace_mark(p.trace, TR_TILES);
        return;
    }

    // ---------------------------------------------------------- compute warps
    // Thread -> (block slot, row subset): one thread per block (K-quant
    // super-block or Q8_0 32-block).  With fewer blocks than threads the
    // threads split the tile's rows into RS subsets; with more (Q8_0 only),
    // a thread takes BPS blocks.
    constexpr int NS = kGroupThreads;
    const int grp = warp / kGroupWarps, gtid = tid - grp * kGroupThreads;
    int RS = 1, subset = 0;
    bool slot_ok = true;
    int mblk[BPS];
    bool mval[BPS];
    if (BPS == 1) {
        RS = max(1, NS / nb);
        subset = gtid / nb;
        slot_ok = gtid < RS * nb;
        mblk[0] = slot_ok ? gtid % nb : 0;
        mval[0] = slot_ok;
    } else {
#pragma unroll
        for (int b = 0; b < BPS; ++b) {
            const int m = gtid + b * NS;
            mval[b] = m < nb;
            mblk[b] = mval[b] ? m : 0;
        }
    }
    const int rps = (T + RS - 1) / RS;
    Q8Act qact[KQ ? 1 : BPS];
#pragma unroll
    for (int b = 0; b < BPS; ++b)
        if (!KQ) load_q8_act(smem + L.act_q_off + mblk[b] * kQ80ActStride, qact[KQ ? 0 : b]);
    const size_t sb = (size_t)(p.K / 8);
    for (int it = grp; it < items; it += kGroups) {
        const int s = it % p.stages, j = it % kTermBufs;
        const GroupRef g = locate(p, tcta + it * tgrid);
        const int ttype = p.seg[p.pair ? 0 : g.seg].type;  // a tile never mixes types
        const size_t rb = (size_t)row_bytes(ttype, p.K);
        const uint8_t *stage = ring + (size_t)s * L.stage_bytes;
        const uint8_t *qbase = stage + (((size_t)g.r0 * rb) & 15);
        const uint8_t *sbase = stage + L.s_region + (((size_t)g.r0 * sb) & 15);
        float *tb = tbuf + (size_t)j * T * nb;
        if (it >= kTermBufs) wait_or_abort(&B.tfree[j], (uint32_t)(((it / kTermBufs) - 1) & 1), B.abort_flag);
        wait_or_abort(&B.full[s], (uint32_t)((it / p.stages) & 1), B.abort_flag);
        for (int rr = 0; rr < rps; ++rr) {
            const int r = subset + rr * RS;
            int useg = 0, urow = 0;
            const bool rv = slot_ok && r < T && slot_row(p, g, r, &useg, &urow);
            if (!rv) continue;
            const int part = r / half, i = r - part * half;
            const uint8_t *rp = qbase + part * L.part_bytes + (size_t)i * rb;
#pragma unroll
            for (int b = 0; b < BPS; ++b) {
                if (!mval[b]) continue;
                float t;
                if (KQ) {
                    const uint8_t *aq = smem + L.act_q_off + mblk[b] * kQ8kActStride;
                    const uint8_t *am = smem + L.act_meta_off + mblk[b] * kQ8kMetaStride;
                    t = ttype == OVF_TYPE_Q4_K ? q4k_unit(rp + (size_t)mblk[b] * 144, aq, am)
                                               : q6k_unit(rp + (size_t)mblk[b] * 210, aq, am);
                } else {
                    const uint8_t *sp = sbase + part * L.s_part + (size_t)i * sb;
                    t = q80_block(rp + 32 * mblk[b], *reinterpret_cast<const float *>(sp + 4 * mblk[b]),
                                  qact[KQ ? 0 : b]);
                }
                tb[r * nb + mblk[b]] = t;
            }
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&B.empty[s]);   // the stage may be refilled
            mbar_arrive(&B.tready[j]);  // the terms may be summed (release)
        }
    }
    if (lane == 0) trace_mark(p.trace, TR_END);
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
    if (p.norm_out)
        OVF_CHECK_ARG(p.epi == EPI_RESIDUAL && p.nseg == 1,
                      "gemv: an output RMSNorm needs a single-segment residual launch");
    if (p.act_mode == ACT_F32_RMSNORM) OVF_CHECK_ARG(p.norm_scale != nullptr, "gemv: RMSNorm input without its scale");
    if (p.epi == EPI_LOGITS_ARGMAX || p.epi == EPI_LOGITS_TP)
        OVF_CHECK_ARG(p.step != nullptr, "gemv: argmax epilogue without step state");
    if (p.epi >= EPI_GROUPS_TP) {
        OVF_CHECK_ARG(p.tp_world >= 1 && p.tp_world <= 8 && p.nseg == 1 && !p.pair && !p.norm_out,
                      "gemv: tensor-parallel epilogue needs one segment and 1..8 ranks");
        for (int w = 0; w < p.tp_world; ++w)
            OVF_CHECK_ARG(p.tp_dst[w] && (p.epi != EPI_LOGITS_TP || p.tp_keys[w]), "gemv: missing exchange buffer");
        if (p.epi == EPI_GROUPS_TP) OVF_CHECK_ARG(!kq && p.q8_group > 0, "gemv: head outputs need grouped Q8_0");
    }
    if (p.expert_sel)
        OVF_CHECK_ARG(p.expert_wstride % 16 == 0 && p.expert_sstride % 16 == 0 && p.expert_slot >= 0 && !p.norm_out,
                      "gemv: routed expert weights need 16-byte strides and no output norm");

    int device = 0;
    OVF_CUDA_TRY(cudaGetDevice(&device));
    const int nsm = sm_count(device);
    const int nb = kq ? p.K / 256 : p.K / 32;
    if (!kq && p.q8_group <= 0) p.q8_group = nb;
    OVF_CHECK_ARG(kq || nb % p.q8_group == 0, "gemv: Q8_0 group must divide the block count");
    int rb = 0;  // bytes streamed per weight row (Q8_0: quants + fp32 scales)
    for (int s = 0; s < p.nseg; ++s) rb = std::max(rb, row_bytes(p.seg[s].type, p.K) + (kq ? 0 : p.K / 8));
    const int parts = p.pair ? 2 : 1;

    // Tile size: T rows (T/2 gate + T/2 up rows in pair launches), at most
    // ~40 KB of weights per stage.  Among those, take the T that minimises
    // the busiest CTA's streamed bytes plus a fixed per-tile cost (~2 KB
    // equivalent): balanced tile counts matter for the small matrices.
    const int budget = (smem_optin(device) + 1024) / kCtasPerSm - 2048;  // leaves room for static smem
    // Long rows (few blocks per row fill few compute threads) may take
    // larger tiles: each tile costs the larger of its streaming time and its
    // contraction latency, one round per kGroupThreads blocks (a round
    // weighs about as much as streaming 16 KB of Q4_K, 36 KB of Q6_K or
    // 4 KB of Q8_0 per CTA: the per-block instruction counts differ).
    int t_cap = std::max(1, std::min(64, (OVF_GEMV_TILE_KB * 1024) / (rb * parts))) * parts;
    const int t_fill = ((kGroupThreads + nb - 1) / nb + parts - 1) / parts * parts;
    while (t_cap < t_fill && (t_cap + parts) * rb * 2 <= budget - 16 * 1024) t_cap += parts;
    double round_bytes = 4096.0;
    for (int s = 0; s < p.nseg; ++s)
        round_bytes = std::max(round_bytes, p.seg[s].type == OVF_TYPE_Q6_K   ? 36864.0
                                            : p.seg[s].type == OVF_TYPE_Q4_K ? 16384.0
                                                                             : 4096.0);
    int best_T = parts;
    double best_cost = 1e300;
    for (int T = parts; T <= t_cap; T += parts) {
        const int rows_per = T / parts;
        int tiles = 0;
        if (p.pair) tiles = (p.seg[0].rows + rows_per - 1) / rows_per;
        else
            for (int s = 0; s < p.nseg; ++s) tiles += (p.seg[s].rows + rows_per - 1) / rows_per;
        if (tiles == 0) break;
        const int grid = std::min(nsm * kCtasPerSm, tiles);
        const double rounds = (double)((T * nb + kGroupThreads - 1) / kGroupThreads);
        const double cost = (double)((tiles + grid - 1) / grid) *
                            std::max((double)T * rb + 2048.0, rounds * round_bytes);
        if (cost < best_cost * 0.999) {
            best_cost = cost;
            best_T = T;
        }
    }
    int T = best_T;
    if (const char *e = getenv("OVF_GEMV_T")) T = std::max(parts, std::min(64, atoi(e) / parts * parts));
    OVF_CHECK_ARG(T * nb <= 16384, "gemv: K=%d is too long for one tile row", p.K);
    p.rows_per_group = T;
    const int rows_per = T / parts;
    int total = 0;
    for (int s = 0; s < p.nseg; ++s) {
        p.seg[s].groups = (p.seg[s].rows + rows_per - 1) / rows_per;
        if (!p.pair) total += p.seg[s].groups;
    }
    if (p.pair) total = p.seg[0].groups;
    p.total_groups = total;
    if (total == 0) return OVF_OK;

    const int grid = std::min(nsm * kCtasPerSm, total + (p.norm_out ? 1 : 0));
    const int warps = kThreads / 32;
    int stages = 0;
    size_t smem = 0;
    int s_hi = 8, s_lo = 2;
    if (const char *e = getenv("OVF_GEMV_S")) s_hi = s_lo = std::max(2, std::min(8, atoi(e)));
    for (int S = s_hi; S >= s_lo; --S) {
        if (S % kGroups) continue;  // stage s must always serve the same compute group
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
    // Blocks per compute slot: the activation slices live in registers.
    int bps = (nb + kGroupThreads - 1) / kGroupThreads;
    OVF_CHECK_ARG(bps <= (kq ? 2 : 8), "gemv: K=%d is too long (at most %d)", p.K,
                  kq ? 2 * kGroupThreads * 256 : 8 * kGroupThreads * 32);
    bps = bps <= 1 ? 1 : bps <= 2 ? 2 : bps <= 4 ? 4 : 8;
    void (*kern)(GemvParams) = kq ? (bps == 1 ? gemv_kernel<true, 1> : gemv_kernel<true, 2>)
                               : (bps == 1   ? gemv_kernel<false, 1>
                                  : bps == 2 ? gemv_kernel<false, 2>
                                  : bps == 4 ? gemv_kernel<false, 4>
                                             : gemv_kernel<false, 8>);
    const int ki = kq ? (bps == 1 ? 0 : 1) : (bps == 1 ? 2 : bps == 2 ? 3 : bps == 4 ? 4 : 5);
    static PerDeviceOnce attr_once[6];
    if (attr_once[ki].pending(device)) {
        cudaFuncAttributes fa{};
        OVF_CUDA_TRY(cudaFuncGetAttributes(&fa, kern));
        OVF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          smem_optin(device) - (int)fa.sharedSizeBytes));
        attr_once[ki].mark(device);
    }
    if (plan_out) *plan_out = GemvPlan{T, stages, warps, grid, smem};
    cudaError_t e = launch_pdl(kern, dim3(grid), dim3(warps * 32), smem, stream, pdl, p);
    if (e != cudaSuccess) return cuda_status(e, "gemv_kernel launch");
    return OVF_OK;
}

}  // namespace ovf
