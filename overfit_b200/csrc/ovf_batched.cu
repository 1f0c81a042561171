// ovf_batched.cu — weight-stationary batched projection (prefill rows).
//
// Runtime/Q4KDotKernel.cs:819-955 (ProjectBatchedWeightStationary),
// Q6KDotKernel.cs:403-525 and Q8DotKernel.cs:352-445 (ProjectBatched): every
// activation row is quantized on its own (Q8_K or Q8_0) and contracted with
// every weight row exactly as the single-row projection does, so row m of
// the result is bit-identical to a single-row call on x[m].  The reference
// decodes each weight tile once and applies it to many activation rows;
// here one CTA stages a tile of kBatRows weight rows x one K chunk in
// shared memory and applies it to kBatActs activation rows, one thread
// per (weight row, activation row) pair.  Each thread adds its block terms
// in ascending block order into one fp32 accumulator — the reference's
// sequential loop — so no cross-thread reduction touches the fp32 sum.
//
// CTAs with adjacent blockIdx.x share a weight tile (x = activation tile,
// y = weight tile), so a tile is read from HBM once and from L2 by the
// other activation tiles.
//
// Work per output is integer dp4a plus a short fp32 tail; for M >= 16 this
// is bounded by the dp4a issue rate, not by HBM.
#include "ovf_common.cuh"
#include "ovf_internal.cuh"

namespace ovf {

static constexpr int kBatRows = 32;   // weight rows per CTA (one per lane)
static constexpr int kBatActs = 8;    // activation rows per CTA (one per warp)
static constexpr int kBatThreads = kBatRows * kBatActs;
static constexpr int kBatKqBlocks = 4;   // K-quant super-blocks per chunk
static constexpr int kBatQ80Blocks = 32; // Q8_0 blocks per chunk

// Shared-memory row strides of the staged weight chunk.  Q4_K: 4 x 144 + 16
// (148 words, a multiple of 4 that is 20 mod 32: the 16-byte loads of eight
// consecutive rows hit distinct bank quads).  Q6_K: a 4 x 210 span copied
// from the 16-byte boundary below it needs 872 bytes; 876 = 219 words (odd,
// so the unit's 4-byte loads of 32 rows are conflict-free).  Q8_0: 32 x 32 +
// 16 = 260 words.
template <int TYPE>
struct BatCfg;
template <>
struct BatCfg<OVF_TYPE_Q4_K> {
    static constexpr int kBlocks = kBatKqBlocks, kBlockBytes = 144, kStride = 592;
};
template <>
struct BatCfg<OVF_TYPE_Q6_K> {
    static constexpr int kBlocks = kBatKqBlocks, kBlockBytes = 210, kStride = 876;
};
template <>
struct BatCfg<OVF_TYPE_Q8_0> {
    static constexpr int kBlocks = kBatQ80Blocks, kBlockBytes = 32, kStride = 1040;
};

static constexpr int kBatQ8kAct = 272;   // Q8_K quants of one super-block (+16 pad)
static constexpr int kBatQ8kMeta = 64;   // int16 bsums[16] | f32 scale | pad | int16 pair sums[8]
static constexpr int kBatQ80Act = 1040;  // Q8_0 quants of one chunk (+16 pad)

struct BatParams {
    const uint8_t *w;      // K-quant rows, or Q8_0 int8 quants [n x K]
    const float *ws;       // Q8_0 scales [n x K/32]
    const float *bias;     // [n] or null
    const int8_t *aq;      // [M x K]
    const float *as;       // Q8_K [M x K/256] or Q8_0 [M x K/32]
    const int16_t *ab;     // Q8_K bsums [M x K/16]
    float *y;              // [M x n]
    const float *resid;    // [M x n] residual added after the bias (or null)
    size_t w_bytes;        // size of the weight buffer (bounds the aligned-down copies)
    int n, K, M;
    int group;             // Q8_0: blocks per head-ordered summation group (0 = one sequential sum)
};

// Copy `len` bytes from `src` into shared memory at `dst`, starting at the
// 16-byte boundary at or below `src`; returns the offset of `src` within
// the copy.  Whole 16-byte units inside [base, end) are loaded as uint4; a
// unit that would cross `end` is loaded byte by byte.  Stores are 4-byte
// (the Q6_K row stride is not a multiple of 16).  `part`/`nparts` split the
// units among the threads working on this row.
__device__ __forceinline__ int bat_copy(uint8_t *dst, const uint8_t *src, int len, const uint8_t *end, int part,
                                        int nparts) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(src);
    const uint8_t *base = reinterpret_cast<const uint8_t *>(a & ~uintptr_t(15));
    const int off = (int)(a & 15u);
    const int units = (off + len + 15) >> 4;
    for (int u = part; u < units; u += nparts) {
        const uint8_t *g = base + 16 * u;
        uint32_t v[4];
        if (g + 16 <= end) {
            const uint4 q = __ldg(reinterpret_cast<const uint4 *>(g));
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t wv = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (g + 4 * j + i < end) wv |= (uint32_t)g[4 * j + i] << (8 * i);
                v[j] = wv;
            }
        }
        uint32_t *d = reinterpret_cast<uint32_t *>(dst + 16 * u);
        d[0] = v[0]; d[1] = v[1]; d[2] = v[2]; d[3] = v[3];
    }
    return off;
}

template <int TYPE>
__global__ void __launch_bounds__(kBatThreads) batched_project_kernel(const __grid_constant__ BatParams p) {
    using C = BatCfg<TYPE>;
    constexpr bool KQ = TYPE != OVF_TYPE_Q8_0;
    constexpr int KB = C::kBlocks, BB = C::kBlockBytes, WS = C::kStride;
    __shared__ __align__(16) uint8_t s_w[kBatRows * WS];
    __shared__ __align__(16) uint8_t s_act[KQ ? kBatActs * KB * kBatQ8kAct : kBatActs * kBatQ80Act];
    __shared__ __align__(16) uint8_t s_meta[KQ ? kBatActs * KB * kBatQ8kMeta : 16];
    __shared__ float s_ws[KQ ? 1 : kBatRows * KB];
    __shared__ float s_as[KQ ? 1 : kBatActs * KB];
    __shared__ int s_off[kBatRows];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m0 = blockIdx.x * kBatActs, o0 = blockIdx.y * kBatRows;
    const int nb = KQ ? p.K / 256 : p.K / 32;
    const size_t rb = KQ ? (size_t)nb * BB : (size_t)p.K;
    const uint8_t *wend = p.w + p.w_bytes;
    const int o = o0 + lane, m = m0 + warp;
    const bool active = o < p.n && m < p.M;
    // Grouped (Wo per head, CachedMultiHeadAttention head-ordered sum): each
    // group of G blocks is summed from zero, and the group sums are added in
    // order on top of the bias.  Ungrouped: one sum, the bias added last.
    const int G = KQ ? 0 : p.group;
    const float bo = active && p.bias ? p.bias[o] : 0.0f;
    float acc = G ? bo : 0.0f, grp = 0.0f;
    int gp = 0;

    for (int c0 = 0; c0 < nb; c0 += KB) {
        const int cb = min(KB, nb - c0);
        // ---- stage the weight chunk: 8 threads per row, 32 rows
        {
            const int r = tid >> 3, part = tid & 7;
            if (o0 + r < p.n) {
                const uint8_t *src = p.w + (size_t)(o0 + r) * rb + (size_t)c0 * BB;
                const int off = bat_copy(s_w + r * WS, src, cb * BB, wend, part, 8);
                if (part == 0) s_off[r] = off;
            }
            if (!KQ) {
                for (int i = tid; i < kBatRows * KB; i += kBatThreads) {
                    const int rr = i / KB, b = i - rr * KB;
                    if (o0 + rr < p.n && b < cb) s_ws[i] = p.ws[(size_t)(o0 + rr) * nb + c0 + b];
                }
            }
        }
        // ---- stage the activation chunk
        if (KQ) {
            // one warp per (activation row, super-block): 8 bytes per lane
            for (int i = warp; i < kBatActs * KB; i += kBatThreads / 32) {
                const int a = i / KB, b = i - a * KB;
                if (m0 + a >= p.M || b >= cb) continue;
                const size_t blk = (size_t)(m0 + a) * nb + c0 + b;
                *reinterpret_cast<uint2 *>(s_act + i * kBatQ8kAct + 8 * lane) =
                    *reinterpret_cast<const uint2 *>(p.aq + blk * 256 + 8 * lane);
                uint8_t *meta = s_meta + i * kBatQ8kMeta;
                if (lane < 16) reinterpret_cast<int16_t *>(meta)[lane] = p.ab[blk * 16 + lane];
                if (lane < 8)
                    reinterpret_cast<int16_t *>(meta + 48)[lane] =
                        (int16_t)(p.ab[blk * 16 + 2 * lane] + p.ab[blk * 16 + 2 * lane + 1]);
                if (lane == 0) *reinterpret_cast<float *>(meta + 32) = p.as[blk];
            }
        } else {
            // one warp per activation row: 1024 quants + 32 scales
            const int a = warp;
            if (m0 + a < p.M) {
                const int8_t *src = p.aq + (size_t)(m0 + a) * p.K + (size_t)c0 * 32;
                for (int u = lane; u < cb * 2; u += 32)
                    *reinterpret_cast<uint4 *>(s_act + a * kBatQ80Act + 16 * u) =
                        *reinterpret_cast<const uint4 *>(src + 16 * u);
                if (lane < cb) s_as[a * KB + lane] = p.as[(size_t)(m0 + a) * nb + c0 + lane];
            }
        }
        __syncthreads();
        // ---- contract: ascending blocks into the thread's accumulator
        if (active) {
            const uint8_t *wr = s_w + lane * WS + s_off[lane];
            for (int b = 0; b < cb; ++b) {
                float t;
                if (TYPE == OVF_TYPE_Q4_K) {
                    const int i = warp * KB + b;
                    t = q4k_unit(wr + b * BB, s_act + i * kBatQ8kAct, s_meta + i * kBatQ8kMeta);
                } else if (TYPE == OVF_TYPE_Q6_K) {
                    const int i = warp * KB + b;
                    t = q6k_unit(wr + b * BB, s_act + i * kBatQ8kAct, s_meta + i * kBatQ8kMeta);
                } else {
                    Q8Act qa;
                    load_q8_act(s_act + warp * kBatQ80Act + 32 * b, qa);  // scale word replaced below
                    qa.s = s_as[warp * KB + b];
                    t = q80_block(wr + 32 * b, s_ws[lane * KB + b], qa);
                }
                if (G) {
                    grp = gp == 0 ? fadd(0.0f, t) : fadd(grp, t);
                    if (++gp == G) {
                        acc = fadd(acc, grp);
                        gp = 0;
                    }
                } else {
                    acc = fadd(acc, t);
                }
            }
        }
        __syncthreads();
    }
    if (active) {
        float y = G || !p.bias ? acc : fadd(bo, acc);
        if (p.resid) y = fadd(p.resid[(size_t)m * p.n + o], y);
        p.y[(size_t)m * p.n + o] = y;
    }
}

ovf_status launch_batched_project(int type, const void *w, const float *ws, size_t w_bytes, const float *bias,
                                  const int8_t *aq, const float *as, const int16_t *ab, float *y, int64_t n,
                                  int64_t k, int64_t rows, cudaStream_t st, int group, const float *resid) {
    if (n == 0 || rows == 0) return OVF_OK;
    OVF_CHECK_ARG(group >= 0 && (group == 0 || type == OVF_TYPE_Q8_0), "batched projection: bad group");
    BatParams p{};
    p.w = (const uint8_t *)w;
    p.ws = ws;
    p.bias = bias;
    p.aq = aq;
    p.as = as;
    p.ab = ab;
    p.y = y;
    p.w_bytes = w_bytes;
    p.n = (int)n;
    p.K = (int)k;
    p.M = (int)rows;
    p.group = group;
    p.resid = resid;
    const dim3 grid((unsigned)((rows + kBatActs - 1) / kBatActs), (unsigned)((n + kBatRows - 1) / kBatRows));
    OVF_CHECK_ARG(grid.y <= 65535u, "batched projection: %lld output rows is too many", (long long)n);
    switch (type) {
        case OVF_TYPE_Q4_K: batched_project_kernel<OVF_TYPE_Q4_K><<<grid, kBatThreads, 0, st>>>(p); break;
        case OVF_TYPE_Q6_K: batched_project_kernel<OVF_TYPE_Q6_K><<<grid, kBatThreads, 0, st>>>(p); break;
        case OVF_TYPE_Q8_0: batched_project_kernel<OVF_TYPE_Q8_0><<<grid, kBatThreads, 0, st>>>(p); break;
        default: OVF_CHECK_ARG(false, "batched projection: bad type %d", type);
    }
    return cuda_status(cudaGetLastError(), "batched_project");
}

}  // namespace ovf
