// ovf_gemv.cu — quantized decode GEMV for sm_100a (see ovf_gemv.cuh).
//
// Work decomposition.  The weight matrix is cut into warp-tiles of a few
// whole rows (one K-quant super-block or 4 Q8_0 blocks per lane).  Every
// warp owns a private ring of `stages` shared-memory buffers; lane 0 streams
// its next tiles into them with cp.async.bulk (1-D TMA) while the warp
// contracts the current one, so each SM keeps ~100-200 KB of weight bytes in
// flight and no CTA-wide barrier sits on the streaming path.  The first
// `stages` tiles are requested before griddepcontrol.wait, i.e. while the
// previous kernel of the decode step is still finishing (PDL).
//
// Exactness.  Integer parts (dp4a over nibbles/6-bit quants x int8) are exact;
// the per-block fp32 tails use explicitly rounded multiplies/adds in the
// reference's operand order, and each row's block terms are summed by one
// lane in ascending block order.  The result equals the reference's
// sequential loop (Runtime/Q4KDotKernel.cs:528-552, Q6KDotKernel.cs:364-380,
// Q8DotKernel.cs:311-328) bit for bit.
#include "ovf_gemv.cuh"

#include <algorithm>
#include <cstdio>

namespace ovf {

static constexpr int kMaxTermsPerWarp = 512;  // units (blocks) per warp-tile
static constexpr int kQ8kActStride = 272;     // 256 quants + 16 pad (bank-conflict free)
static constexpr int kQ8kMetaStride = 48;     // int16 bsums[16] + f32 scale + pad
static constexpr int kQ80ActStride = 48;      // 32 quants + f32 scale + pad

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

struct Layout {
    // byte offsets inside dynamic shared memory
    int bar_off, act_q_off, act_meta_off, red_off, terms_off, vals_off, stage_off;
    int stage_bytes, q8_scale_off;  // Q8_0: scales region offset inside a stage
    int nb, row_bytes;
};

static __host__ __device__ inline int kq_block_bytes(int type) { return type == OVF_TYPE_Q4_K ? 144 : 210; }

// Bytes of one weight row of `type` (Q8_0: quants + fp32 scales).
static __host__ __device__ inline int row_bytes_of(int type, int K) {
    return is_kquant(type) ? (K / 256) * kq_block_bytes(type) : K + K / 8;
}

// Largest row of the launch's segments (K-quant segments of one launch may
// mix Q4_K and Q6_K); stage buffers are sized for it.
static __host__ __device__ inline int max_row_bytes(const GemvParams &p) {
    int m = 0;
    for (int s = 0; s < p.nseg; ++s) m = max(m, row_bytes_of(p.seg[s].type, p.K));
    return m;
}

static __host__ __device__ inline Layout make_layout(int type, int K, int rpt, int mult, int stages, int warps,
                                                     int row_bytes_max) {
    Layout L{};
    const bool kq = is_kquant(type);
    L.nb = kq ? K / 256 : K / 32;
    L.row_bytes = row_bytes_max;
    size_t off = 0;
    L.bar_off = 0;
    off = align_up(sizeof(uint64_t) * warps * stages, 128);
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
    off = align_up(off + 64 * sizeof(float) + warps * sizeof(unsigned long long), 128);
    L.terms_off = (int)off;
    off = align_up(off + (size_t)warps * kMaxTermsPerWarp * sizeof(float), 128);
    L.vals_off = (int)off;
    off = align_up(off + (size_t)warps * 32 * sizeof(float), 128);
    L.stage_off = (int)off;
    const int rows = rpt * mult;
    if (kq) {
        L.stage_bytes = (int)align_up((size_t)rows * L.row_bytes + 16, 128);
        L.q8_scale_off = 0;
    } else {
        L.q8_scale_off = (int)align_up((size_t)rows * K, 16);
        L.stage_bytes = (int)align_up((size_t)L.q8_scale_off + (size_t)rows * (K / 8) + 16, 128);
    }
    return L;
}

static __host__ __device__ inline size_t layout_smem(const Layout &L, int stages, int warps) {
    return (size_t)L.stage_off + (size_t)stages * warps * L.stage_bytes;
}

// ------------------------------------------------------------ tile helpers
struct TileRef {
    int seg, r0, nr;
};

__device__ __forceinline__ TileRef locate(const GemvParams &p, int t) {
    TileRef tr{0, 0, 0};
    int s = 0;
    if (!p.pair) {
        while (s < p.nseg - 1 && t >= p.seg[s].tiles) {
            t -= p.seg[s].tiles;
            ++s;
        }
    }
    tr.seg = s;
    tr.r0 = t * p.rows_per_tile;
    tr.nr = min(p.rows_per_tile, p.seg[s].rows - tr.r0);
    return tr;
}

// Issues the bulk copies of one warp-tile (both matrices in pair mode).  A
// ragged (<16 B) tail of a final partial tile is left to fix_tails.
__device__ __forceinline__ void issue_tile(const GemvParams &p, const Layout &L, int t, uint8_t *stage,
                                           uint64_t *bar, uint64_t pol) {
    TileRef tr = locate(p, t);
    const GemvSeg &sg = p.seg[tr.seg];
    const int K = p.K;
    if (is_kquant(sg.type)) {
        const int rb = row_bytes_of(sg.type, K);
        const uint32_t bytes = (uint32_t)(tr.nr * rb);
        const uint32_t main = bytes & ~15u;
        const int ncopy = p.pair ? 2 : 1;
        mbar_arrive_expect_tx(bar, main * ncopy);
        for (int c = 0; c < ncopy; ++c) {
            const GemvSeg &g = p.seg[p.pair ? c : tr.seg];
            uint8_t *dst = stage + (size_t)c * p.rows_per_tile * rb;
            if (main) bulk_g2s(dst, g.w + (size_t)tr.r0 * rb, main, bar, pol);
        }
    } else {
        const uint32_t qb = (uint32_t)(tr.nr * K);
        const uint32_t sb = (uint32_t)(tr.nr * (K / 8));
        const uint32_t qm = qb & ~15u, sm = sb & ~15u;
        const int ncopy = p.pair ? 2 : 1;
        mbar_arrive_expect_tx(bar, (qm + sm) * ncopy);
        for (int c = 0; c < ncopy; ++c) {
            const GemvSeg &g = p.seg[p.pair ? c : tr.seg];
            const size_t rq = (size_t)c * p.rows_per_tile;
            if (qm) bulk_g2s(stage + rq * K, g.w + (size_t)tr.r0 * K, qm, bar, pol);
            if (sm)
                bulk_g2s(stage + L.q8_scale_off + rq * (K / 8),
                         reinterpret_cast<const uint8_t *>(g.ws + (size_t)tr.r0 * (K / 32)), sm, bar, pol);
        }
    }
}

// Copies the ragged (<16 B) tails the bulk engine cannot move.  Only final
// partial tiles of unusual shapes have one.
__device__ __forceinline__ void fix_tails(const GemvParams &p, const Layout &L, int t, uint8_t *stage, int lane) {
    TileRef tr = locate(p, t);
    const GemvSeg &sg = p.seg[tr.seg];
    const int K = p.K;
    if (is_kquant(sg.type)) {
        const int rb = row_bytes_of(sg.type, K);
        const uint32_t bytes = (uint32_t)(tr.nr * rb);
        const uint32_t main = bytes & ~15u;
        if (main == bytes) return;
        const int ncopy = p.pair ? 2 : 1;
        for (int c = 0; c < ncopy; ++c) {
            const GemvSeg &g = p.seg[p.pair ? c : tr.seg];
            uint8_t *dst = stage + (size_t)c * p.rows_per_tile * rb;
            const uint8_t *src = g.w + (size_t)tr.r0 * rb;
            for (uint32_t i = main + lane; i < bytes; i += 32) dst[i] = src[i];
        }
    } else {
        const uint32_t qb = (uint32_t)(tr.nr * K), sb = (uint32_t)(tr.nr * (K / 8));
        const uint32_t qm = qb & ~15u, sm = sb & ~15u;
        const int ncopy = p.pair ? 2 : 1;
        for (int c = 0; c < ncopy; ++c) {
            const GemvSeg &g = p.seg[p.pair ? c : tr.seg];
            const size_t rq = (size_t)c * p.rows_per_tile;
            const uint8_t *qs = g.w + (size_t)tr.r0 * K;
            const uint8_t *ss = reinterpret_cast<const uint8_t *>(g.ws + (size_t)tr.r0 * (K / 32));
            for (uint32_t i = qm + lane; i < qb; i += 32) stage[rq * K + i] = qs[i];
            for (uint32_t i = sm + lane; i < sb; i += 32) stage[L.q8_scale_off + rq * (K / 8) + i] = ss[i];
        }
    }
}

__device__ __forceinline__ bool tile_has_tail(const GemvParams &p, const Layout &L, int t) {
    TileRef tr = locate(p, t);
    const GemvSeg &sg = p.seg[tr.seg];
    if (is_kquant(sg.type)) return ((tr.nr * row_bytes_of(sg.type, p.K)) & 15) != 0;
    return ((tr.nr * p.K) & 15) != 0 || ((tr.nr * (p.K / 8)) & 15) != 0;
}

// ------------------------------------------------------------- dot units
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// Q4_K x Q8_K over one super-block (Runtime/Q4KDotKernel.cs:216-256).
__device__ __forceinline__ float q4k_unit(const uint8_t *blk, const uint8_t *q8, const uint8_t *meta) {
    const uint4 h = *reinterpret_cast<const uint4 *>(blk);
    const float d = h2f_bits((uint16_t)(h.x & 0xFFFFu));
    const float dmin = h2f_bits((uint16_t)(h.x >> 16));
    int sc[8], mn[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        sc[j] = (int)(byte_of(h.y, j) & 63u);
        mn[j] = (int)(byte_of(h.z, j) & 63u);
        sc[j + 4] = (int)((byte_of(h.w, j) & 0xFu) | ((byte_of(h.y, j) >> 6) << 4));
        mn[j + 4] = (int)((byte_of(h.w, j) >> 4) | ((byte_of(h.z, j) >> 6) << 4));
    }
    int mainAcc = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * p);
        const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * p);
        const uint4 l0 = *reinterpret_cast<const uint4 *>(q8 + 64 * p);
        const uint4 l1 = *reinterpret_cast<const uint4 *>(q8 + 64 * p + 16);
        const uint4 h0 = *reinterpret_cast<const uint4 *>(q8 + 64 * p + 32);
        const uint4 h1 = *reinterpret_cast<const uint4 *>(q8 + 64 * p + 48);
        const uint32_t M = 0x0F0F0F0Fu;
        int lo = 0, hi = 0;
        lo = dp4a((int)(qa.x & M), (int)l0.x, lo);
        lo = dp4a((int)(qa.y & M), (int)l0.y, lo);
        lo = dp4a((int)(qa.z & M), (int)l0.z, lo);
        lo = dp4a((int)(qa.w & M), (int)l0.w, lo);
        lo = dp4a((int)(qb.x & M), (int)l1.x, lo);
        lo = dp4a((int)(qb.y & M), (int)l1.y, lo);
        lo = dp4a((int)(qb.z & M), (int)l1.z, lo);
        lo = dp4a((int)(qb.w & M), (int)l1.w, lo);
        hi = dp4a((int)((qa.x >> 4) & M), (int)h0.x, hi);
        hi = dp4a((int)((qa.y >> 4) & M), (int)h0.y, hi);
        hi = dp4a((int)((qa.z >> 4) & M), (int)h0.z, hi);
        hi = dp4a((int)((qa.w >> 4) & M), (int)h0.w, hi);
        hi = dp4a((int)((qb.x >> 4) & M), (int)h1.x, hi);
        hi = dp4a((int)((qb.y >> 4) & M), (int)h1.y, hi);
        hi = dp4a((int)((qb.z >> 4) & M), (int)h1.z, hi);
        hi = dp4a((int)((qb.w >> 4) & M), (int)h1.w, hi);
        mainAcc += sc[2 * p] * lo + sc[2 * p + 1] * hi;
    }
    const uint4 b0 = *reinterpret_cast<const uint4 *>(meta);
    const uint4 b1 = *reinterpret_cast<const uint4 *>(meta + 16);
    const float q8s = *reinterpret_cast<const float *>(meta + 32);
    const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    int minAcc = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const int pairsum = (int)(int16_t)(bw[s] & 0xFFFFu) + (int)(int16_t)(bw[s] >> 16);
        minAcc += mn[s] * pairsum;
    }
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
            if (lane == 0) *reinterpret_cast<float *>(meta + b * kQ8kMetaStride + 32) = p.as[b];
        }
        return;
    }
    float s = 1.0f;
    float *red = reinterpret_cast<float *>(smem + L.red_off);
    if (p.act_mode == ACT_F32_RMSNORM) s = block_rms_scale(p.x, p.K, p.eps, red);
    const bool write_out = blockIdx.x == 0 && p.aq_out != nullptr;
    for (int b = warp; b < nsb; b += nw) {
        const int e0 = b * 256 + 8 * lane;
        float v[8];
        const float4 x0 = *reinterpret_cast<const float4 *>(p.x + e0);
        const float4 x1 = *reinterpret_cast<const float4 *>(p.x + e0 + 4);
        v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
        v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
        if (p.act_mode == ACT_F32_RMSNORM) {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = p.gamma ? fmul(fmul(v[i], s), p.gamma[e0 + i]) : fmul(v[i], s);
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = warp_max(amax);
        const float scale = fdiv(amax, 127.0f);
        const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
        uint32_t w0 = 0, w1 = 0;
        int sum8 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int q = quant_elem(v[i], inv);
            sum8 += q;
            if (i < 4) w0 |= ((uint32_t)(q & 0xFF)) << (8 * i);
            else w1 |= ((uint32_t)(q & 0xFF)) << (8 * (i - 4));
        }
        const int g16 = sum8 + __shfl_xor_sync(0xFFFFFFFFu, sum8, 1);
        *reinterpret_cast<uint2 *>(aq + b * kQ8kActStride + 8 * lane) = make_uint2(w0, w1);
        if ((lane & 1) == 0) reinterpret_cast<int16_t *>(meta + b * kQ8kMetaStride)[lane >> 1] = (int16_t)g16;
        if (lane == 0) *reinterpret_cast<float *>(meta + b * kQ8kMetaStride + 32) = scale;
        if (write_out) {
            *reinterpret_cast<uint2 *>(p.aq_out + e0) = make_uint2(w0, w1);
            if ((lane & 1) == 0) p.ab_out[(size_t)b * 16 + (lane >> 1)] = (int16_t)g16;
            if (lane == 0) p.as_out[b] = scale;
        }
    }
}

__device__ void prep_q80(const GemvParams &p, const Layout &L, uint8_t *smem) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint8_t *act = smem + L.act_q_off;
    float s = 1.0f;
    float *red = reinterpret_cast<float *>(smem + L.red_off);
    if (p.act_mode == ACT_F32_RMSNORM) s = block_rms_scale(p.x, p.K, p.eps, red);
    const bool write_out = blockIdx.x == 0 && p.aq_out != nullptr;
    for (int b = warp; b < L.nb; b += nw) {
        const int e = b * 32 + lane;
        float v = p.x[e];
        if (p.act_mode == ACT_F32_RMSNORM) v = p.gamma ? fmul(fmul(v, s), p.gamma[e]) : fmul(v, s);
        const float amax = warp_max(fabsf(v));
        const float scale = fdiv(amax, 127.0f);
        const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
        const int q = quant_elem(v, inv);
        act[b * kQ80ActStride + lane] = (uint8_t)(int8_t)q;
        if (lane == 0) *reinterpret_cast<float *>(act + b * kQ80ActStride + 32) = scale;
        if (write_out) {
            p.aq_out[e] = (int8_t)q;
            if (lane == 0) p.as_out[b] = scale;
        }
    }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

// ------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(512, 1) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int type0 = p.seg[0].type;
    const int mult = p.pair ? 2 : 1;
    const Layout L = make_layout(type0, p.K, p.rows_per_tile, mult, p.stages, W, max_row_bytes(p));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off) + warp * p.stages;
    uint8_t *my_stages = smem + L.stage_off + (size_t)warp * p.stages * L.stage_bytes;
    float *terms = reinterpret_cast<float *>(smem + L.terms_off) + warp * kMaxTermsPerWarp;
    float *vals = reinterpret_cast<float *>(smem + L.vals_off) + warp * 32;

    const int gw = blockIdx.x * W + warp;
    const int nwarps = gridDim.x * W;
    uint64_t pol = l2_evict_first_policy();

    if (lane == 0) {
        for (int s = 0; s < p.stages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    // Weights do not depend on the previous kernel: start streaming now.
    if (lane == 0) {
        for (int s = 0; s < p.stages; ++s) {
            const int t = gw + s * nwarps;
            if (t >= p.total_tiles) break;
            issue_tile(p, L, t, my_stages + (size_t)s * L.stage_bytes, &bars[s], pol);
        }
    }
    pdl_wait();
    if (is_kquant(type0)) prep_q8k(p, L, smem);
    else prep_q80(p, L, smem);
    __syncthreads();
    pdl_launch_dependents();

    const uint8_t *act_q = smem + L.act_q_off;
    const uint8_t *act_meta = smem + L.act_meta_off;
    const int nb = L.nb;
    const int G = is_kquant(type0) ? nb : p.q8_group;
    unsigned long long best = 0ull;

    for (int i = 0;; ++i) {
        const int t = gw + i * nwarps;
        if (t >= p.total_tiles) break;
        const int s = i % p.stages;
        const uint32_t parity = (uint32_t)((i / p.stages) & 1);
        uint8_t *stage = my_stages + (size_t)s * L.stage_bytes;
        if (!mbar_wait_bounded(&bars[s], parity)) {
            // Give the copies still in flight (tiles i+1 .. i+stages-1) a
            // bounded chance to land, then stop streaming; the CTA still runs
            // its common exit path so no barrier is left waiting.
            for (int j = i + 1; j < i + p.stages; ++j)
                if (gw + j * nwarps < p.total_tiles)
                    mbar_wait_bounded(&bars[j % p.stages], (uint32_t)((j / p.stages) & 1));
            break;
        }
        if (tile_has_tail(p, L, t)) {
            fix_tails(p, L, t, stage, lane);
            __syncwarp();
        }
        const TileRef tr = locate(p, t);
        const int type = p.seg[tr.seg].type;
        const int nrs = tr.nr * mult;  // rows in this stage
        const int units = nrs * nb;
        for (int u = lane; u < units; u += 32) {
            const int sr = u / nb, b = u - sr * nb;
            const int srow = (p.pair && sr >= tr.nr) ? p.rows_per_tile + (sr - tr.nr) : sr;
            float term;
            if (type == OVF_TYPE_Q4_K) {
                term = q4k_unit(stage + (size_t)(srow * nb + b) * 144, act_q + b * kQ8kActStride,
                                act_meta + b * kQ8kMetaStride);
            } else if (type == OVF_TYPE_Q6_K) {
                term = q6k_unit(stage + (size_t)(srow * nb + b) * 210, act_q + b * kQ8kActStride,
                                act_meta + b * kQ8kMetaStride);
            } else {
                const float ws = reinterpret_cast<const float *>(stage + L.q8_scale_off)[srow * nb + b];
                term = q80_unit(stage + (size_t)srow * p.K + 32 * b, ws, act_q + b * kQ80ActStride);
            }
            terms[u] = term;
        }
        __syncwarp();
        // Stage s is consumed: refill it with the tile `stages` ahead.
        if (lane == 0) {
            const int tn = t + p.stages * nwarps;
            if (tn < p.total_tiles) {
                fence_proxy_async_smem();
                issue_tile(p, L, tn, stage, &bars[s], pol);
            }
        }
        // Row sums in ascending block order, one lane per row.
        if (lane < nrs) {
            const int seg = (p.pair && lane >= tr.nr) ? 1 : tr.seg;
            const int row = tr.r0 + ((p.pair && lane >= tr.nr) ? lane - tr.nr : lane);
            const float *bias = p.seg[seg].bias;
            const float *tr_terms = terms + lane * nb;
            float y;
            if (G >= nb) {
                float acc = tr_terms[0];
                for (int b = 1; b < nb; ++b) acc = fadd(acc, tr_terms[b]);
                y = bias ? fadd(bias[row], acc) : acc;
            } else {
                y = bias ? bias[row] : 0.0f;
                for (int g0 = 0; g0 < nb; g0 += G) {
                    float acc = tr_terms[g0];
                    for (int b = 1; b < G; ++b) acc = fadd(acc, tr_terms[g0 + b]);
                    y = fadd(y, acc);
                }
            }
            vals[lane] = y;
        }
        __syncwarp();
        if (p.epi == EPI_SILU_PAIR) {
            if (lane < tr.nr) {
                const float g = vals[lane], u = vals[tr.nr + lane];
                const float sg = fdiv(1.0f, fadd(1.0f, expf(-g)));
                p.seg[0].out[tr.r0 + lane] = fmul(fmul(g, sg), u);
            }
        } else if (lane < nrs) {
            const int row = tr.r0 + lane;
            const float y = vals[lane];
            float *out = p.seg[tr.seg].out;
            if (p.epi == EPI_RESIDUAL) out[row] = fadd(p.resid[row], y);
            else out[row] = y;
            if (p.epi == EPI_LOGITS_ARGMAX) {
                const unsigned long long k = argmax_key(y, row);
                best = k > best ? k : best;
            }
        }
        __syncwarp();
    }

    if (p.epi == EPI_LOGITS_ARGMAX) {
        // warp max -> CTA max -> one global atomic per CTA; the last CTA to
        // finish turns the winning key into the next token.
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best, o);
            best = other > best ? other : best;
        }
        unsigned long long *wbest = reinterpret_cast<unsigned long long *>(smem + L.red_off + 64 * sizeof(float));
        if (lane == 0) wbest[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long b = 0;
            for (int w = 0; w < W; ++w) b = wbest[w] > b ? wbest[w] : b;
            atomicMax(&p.step->argmax_key, b);
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
    OVF_CHECK_ARG(kq || p.K % 16 == 0, "gemv: Q8_0 K must be a multiple of 16");
    if (p.act_mode == ACT_PREQ_Q8K) {
        OVF_CHECK_ARG(kq, "gemv: pre-quantized Q8_K activations need K-quant weights");
        OVF_CHECK_ARG(p.aq && p.as && p.ab && aligned16(p.aq), "gemv: pre-quantized activation buffers");
    } else {
        OVF_CHECK_ARG(p.x && aligned16(p.x), "gemv: x must be non-null and 16-byte aligned");
    }
    if (p.pair)
        OVF_CHECK_ARG(p.nseg == 2 && p.seg[0].rows == p.seg[1].rows && p.seg[0].type == p.seg[1].type,
                      "gemv: pair mode needs 2 segments of equal shape and type");
    if (p.epi == EPI_RESIDUAL) OVF_CHECK_ARG(p.resid != nullptr, "gemv: residual epilogue without residual");
    if (p.epi == EPI_LOGITS_ARGMAX) OVF_CHECK_ARG(p.step != nullptr, "gemv: argmax epilogue without step state");

    int device = 0;
    OVF_CUDA_TRY(cudaGetDevice(&device));
    const int nsm = sm_count(device);
    const int nb = kq ? p.K / 256 : p.K / 32;
    const int row_bytes = max_row_bytes(p);
    // Rows per warp-tile: a multiple of the alignment step that keeps every
    // full tile's bulk copies 16-byte sized, with ~1 super-block (K-quant) or
    // ~4 blocks (Q8_0) per lane.
    int ralign = 1;
    while (ralign < 16) {
        bool ok = true;
        for (int s = 0; s < p.nseg; ++s) {
            const int rb = row_bytes_of(p.seg[s].type, p.K);
            ok = ok && (kq ? ((ralign * rb) % 16 == 0) : ((ralign * p.K) % 16 == 0 && (ralign * (p.K / 8)) % 16 == 0));
        }
        if (ok) break;
        ++ralign;
    }
    const int mult = p.pair ? 2 : 1;
    const int units_target = kq ? 32 : 128;
    int rpt = ralign * std::max(1, units_target / (ralign * nb * mult));
    while (rpt > ralign && rpt * mult * nb > kMaxTermsPerWarp) rpt -= ralign;
    OVF_CHECK_ARG(rpt * mult * nb <= kMaxTermsPerWarp && rpt * mult <= 32,
                  "gemv: K=%d too long for one warp-tile (max %d blocks per row)", p.K, kMaxTermsPerWarp);
    int total = 0;
    for (int s = 0; s < p.nseg; ++s) {
        p.seg[s].tiles = (p.seg[s].rows + rpt - 1) / rpt;
        if (!p.pair) total += p.seg[s].tiles;
    }
    if (p.pair) total = p.seg[0].tiles;
    p.total_tiles = total;
    p.rows_per_tile = rpt;
    if (!kq && p.q8_group <= 0) p.q8_group = nb;
    OVF_CHECK_ARG(kq || nb % p.q8_group == 0, "gemv: Q8_0 group must divide the block count");
    if (total == 0) return OVF_OK;

    // Warps and stages: as many bytes in flight as shared memory allows.
    const int budget = smem_optin(device) - 1024;
    int warps = 16, stages = 0;
    Layout L{};
    for (; warps >= 4; warps /= 2) {
        for (stages = 6; stages >= 2; --stages) {
            L = make_layout(type0, p.K, rpt, mult, stages, warps, row_bytes);
            if (layout_smem(L, stages, warps) <= (size_t)budget) break;
        }
        if (stages >= 3 || (warps == 4 && stages >= 2)) break;
    }
    OVF_CHECK_ARG(stages >= 2, "gemv: K=%d does not fit shared memory", p.K);
    p.stages = stages;
    const size_t smem = layout_smem(L, stages, warps);
    int grid = std::min(nsm, (total + warps - 1) / warps);
    static bool attr_done[64] = {false};
    if (device < 64 && !attr_done[device]) {
        OVF_CUDA_TRY(cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          smem_optin(device)));
        attr_done[device] = true;
    }
    if (plan_out) *plan_out = GemvPlan{rpt, stages, warps, grid, smem};
    cudaError_t e = launch_pdl(gemv_kernel, dim3(grid), dim3(warps * 32), smem, stream, pdl, p);
    if (e != cudaSuccess) return cuda_status(e, "gemv_kernel launch");
    return OVF_OK;
}

}  // namespace ovf
