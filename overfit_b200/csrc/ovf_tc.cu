// ovf_tc.cu — the prefill projection of Q4_K weights on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM), bit-identical to the
// reference's per-row dot (Runtime/Q4KDotKernel.cs:216-256 via
// ProjectBatchedWeightStationary :819-955) and so to batched_project_kernel.
//
// Exactness.  Per weight row n, token m and super-block b the reference
// forms two integers, mainAcc = sum_s sc[s] * sum_{k in s} q4[k] q8[k] and
// minAcc = sum_s m[s] * bsum_s, then term = xs * (d * mainAcc - dmin *
// minAcc) in fp32 and adds the terms in ascending b.  The tensor cores
// compute both integers exactly in fp32 accumulators:
//   * A = q4 * sc as fp16 integers (0..945), B = the Q8_K activation as fp16
//     integers; mainAcc is split over two accumulators by K half (sub-blocks
//     0-3 and 4-7).  Each half is a sum of 128 products below 945 * 128, so
//     every partial sum stays below 2^24 and is exact in any order; the fp32
//     add of the two halves is then the correctly rounded (float)mainAcc.
//   * minAcc = sum_j m[j/2] * bsum16_j over the 16 Q8_K 16-element sums
//     (|bsum16| <= 2048, exact in fp16): one K=16 MMA.
// The epilogue runs the reference's fp32 tail and the ascending-b sum.
//
// Weights are expanded in shared memory with the fp16 magic-number trick
// (0x6400 | nibble = 1024 + nibble, then one fma by the 6-bit scale), which
// yields the elements of an 8-group in the order 0,2,1,3,4,6,5,7; the
// activation tiles are packed in the same K order, so the products pair up.
//
// Layout.  A CTA owns 128 weight rows x 64 tokens; per super-block four
// K-chunks of 64 flow through rings of fp16 operand tiles in the UMMA
// no-swizzle K-major layout (8x16-byte core matrices; K-adjacent core
// matrices 128 B apart, 8-row groups 1024 B apart).  Warp roles, linked by
// mbarriers:
//   warp 0      producer: a 2-D tensor copy of the 128 rows' 144-byte blocks
//               per super-block, the packed activation chunks, the bsum16
//               tile and the tokens' scales;
//   warp 1      TMEM allocation (256 columns) and the single MMA-issuing
//               thread: per chunk four MMAs (M=128, N=64, K=16) into the
//               chunk's K-half accumulator, plus the minAcc MMA with chunk 0;
//               tcgen05.commit releases operand stages and publishes the
//               accumulator set;
//   warps 2-5   converters: thread = weight row; they also hand d / dmin and
//               the token scales to the epilogue through a small ring;
//   warps 6-9   epilogue: warp w reads TMEM lanes 32*(w%4).., all 64 tokens,
//               and keeps the running per-(row, token) sums in TMEM.
// Two CTAs per SM overlap each other's pipeline hand-offs.  The operands live
// in this GPU's shared memory only; no cluster, no multicast.  Every mbarrier
// wait is bounded (the device error word is set and the kernel drains
// instead of hanging).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "ovf_internal.cuh"

namespace ovf {

static constexpr int kTcRows = 128;     // weight rows per CTA (MMA M, TMEM lanes)
static constexpr int kTcToks = 64;      // tokens per CTA (MMA N)
static constexpr int kTcKc = 64;        // K per operand chunk
// Ring depths cover the ~350-cycle mbarrier round trip between warps: a
// chunk's four MMAs take ~130 cycles, so a stage comes back to its
// producer only after several chunks.
static constexpr int kTcAStages = 2;    // A ring (chunks; filled in shared memory by the converters)
static constexpr int kTcBStages = 3;    // B ring (chunks; copied from L2)
static constexpr int kTcRaw = 2;        // per-super-block ring: raw blocks, m tile, bsum tile, token scales
static constexpr int kTcE = 2;          // epilogue ring: per-row d / dmin and the token scales
static constexpr int kTcThreads = 320;  // 10 warps; two CTAs per SM
static constexpr int kTcATile = kTcRows * kTcKc * 2;    // 16 KB
static constexpr int kTcAMin = kTcRows * 16 * 2;        // 4 KB: m[j/2], K = 16
static constexpr int kTcBTile = kTcToks * kTcKc * 2;    // 8 KB
static constexpr int kTcBBs = kTcToks * 16 * 2;         // 2 KB: bsum16, K = 16
static constexpr int kTcAStage = kTcATile;
static constexpr int kTcBStage = kTcBTile;
static constexpr int kTcXsBytes = kTcToks * 4;          // token scales per super-block
static constexpr int kTcEBytes = kTcRows * 8 + kTcXsBytes;  // float2 (d, dmin) per row + token scales
// TMEM columns: per accumulator set [lo half | hi half | minAcc], two sets,
// then the running sums
static constexpr int kTcSetCols = 3 * kTcToks;
static constexpr int kTcOutCol = kTcSetCols;  // one accumulator set, then the running sums
static constexpr int kTcTmemCols = 256;       // half of TMEM: two CTAs per SM
static_assert(kTcOutCol + kTcToks <= kTcTmemCols, "TMEM budget");

// shared memory map (bytes from a 1024-aligned base)
struct TcSmem {
    static constexpr int a_off = 0;                                        // [stages] A tiles (+ min tile)
    static constexpr int b_off = a_off + kTcAStages * kTcAStage;            // [stages] B tiles
    static constexpr int raw_off = b_off + kTcBStages * kTcBStage;          // [raw] Q4_K blocks [128][144]
    static constexpr int amin_off = raw_off + kTcRaw * kTcRows * 144;       // [raw] m[j/2] tiles
    static constexpr int bs_off = amin_off + kTcRaw * kTcAMin;              // [raw] bsum16 tiles
    static constexpr int xs_off = bs_off + kTcRaw * kTcBBs;                 // [raw] token scales
    static constexpr int e_off = xs_off + kTcRaw * kTcXsBytes;              // [E] epilogue slots
    static constexpr int bar_off = e_off + kTcE * kTcEBytes;                // mbarriers
    static constexpr int total = bar_off + 512 + 128;                       // + alignment slack
};
static_assert(TcSmem::total <= 113 * 1024, "shared memory budget: two CTAs per SM");

// no-swizzle K-major descriptor: LBO = K-adjacent core matrices, SBO =
// 8-row groups, descriptor version 1
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// kind::f16, fp16 A and B (K-major), fp32 accumulator, M = 128, N = 64
static constexpr uint32_t kTcIdesc = (1u << 4) | ((uint32_t)(kTcToks >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive columns of this warp's 32 TMEM lanes (one value per thread
// and column); the wait is left to the caller so several loads overlap.
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// element order inside an 8-group of the operand tiles (see the header)
__device__ __forceinline__ int tc_perm8(int j) { return (j & 4) | ((j & 1) << 1) | ((j >> 1) & 1); }

// Activation packing: the Q8_K rows of a batch as fp16 operand tiles in the
// UMMA layout, x16 [token tile][K chunk][64 x 64]; per (token tile, super-
// block) the bsum16 tile bs16 [64 x 16] (same layout) and the token scales
// xs [64].  Tokens past `rows` are zero.
__global__ void tc_pack_kernel(const int8_t *__restrict__ aq, const float *__restrict__ as,
                               const int16_t *__restrict__ ab, int rows, int K, __half *__restrict__ x16,
                               __half *__restrict__ bs16, float *__restrict__ xs) {
    const int mt = blockIdx.y, kc = blockIdx.x;  // token tile, K chunk
    const int nkc = K / kTcKc, nb = K / 256;
    __half *dst = x16 + ((size_t)mt * nkc + kc) * (kTcToks * kTcKc);
    for (int i = threadIdx.x; i < kTcToks * 8; i += blockDim.x) {
        // one 8-element (16-byte) core-matrix row: token t, k group g
        const int t = i >> 3, g = i & 7, m = mt * kTcToks + t;
        __align__(16) __half h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int v = m < rows ? aq[(size_t)m * K + kc * kTcKc + 8 * g + tc_perm8(j)] : 0;
            h[j] = __int2half_rn(v);
        }
        *reinterpret_cast<uint4 *>(dst + (t >> 3) * 512 + g * 64 + (t & 7) * 8) = *reinterpret_cast<const uint4 *>(h);
    }
    if ((kc & 3) == 0) {
        const int b = kc >> 2;
        __half *bd = bs16 + ((size_t)mt * nb + b) * (kTcToks * 16);
        for (int i = threadIdx.x; i < kTcToks * 2; i += blockDim.x) {
            const int t = i >> 1, g = i & 1, m = mt * kTcToks + t;
            __align__(16) __half h[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) h[j] = __int2half_rn(m < rows ? (int)ab[(size_t)m * (K / 16) + b * 16 + 8 * g + j] : 0);
            *reinterpret_cast<uint4 *>(bd + (t >> 3) * 128 + g * 64 + (t & 7) * 8) = *reinterpret_cast<const uint4 *>(h);
        }
        for (int t = threadIdx.x; t < kTcToks; t += blockDim.x) {
            const int m = mt * kTcToks + t;
            xs[((size_t)mt * nb + b) * kTcToks + t] = m < rows ? as[(size_t)m * nb + b] : 0.0f;
        }
    }
}

struct TcParams {
    const uint8_t *w;      // Q4_K [n][K/256] blocks
    const __half *x16;     // packed activation tiles
    const __half *bs16;    // packed bsum16 tiles
    const float *xs;       // packed token scales
    const float *bias;     // [n] or null
    const float *resid;    // [rows][n] or null
    float *y;              // [rows][n]
    int n, K, rows;
};

// A Q4_K block's d, dmin and 6-bit scales / mins
// (GgmlDequant.UnpackQ4_KScalesMins, Loading/GgmlDequant.cs:49-77); zeros for
// a row past the matrix.
__device__ __forceinline__ void tc_unpack_scales(const uint8_t *blk, bool valid, int *sc, int *mn, float *d,
                                                 float *dmin) {
    if (!valid) {
#pragma unroll
        for (int j = 0; j < 8; ++j) sc[j] = mn[j] = 0;
        *d = *dmin = 0.0f;
        return;
    }
    const uint4 hv = *reinterpret_cast<const uint4 *>(blk);
    const uint32_t w0 = hv.x, w1 = hv.y, w2 = hv.z, w3 = hv.w;
    *d = __half2float(__ushort_as_half((unsigned short)(w0 & 0xFFFF)));
    *dmin = __half2float(__ushort_as_half((unsigned short)(w0 >> 16)));
    uint8_t q[12];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        q[j] = (uint8_t)(w1 >> (8 * j));
        q[4 + j] = (uint8_t)(w2 >> (8 * j));
        q[8 + j] = (uint8_t)(w3 >> (8 * j));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        sc[j] = q[j] & 63;
        mn[j] = q[j + 4] & 63;
    }
#pragma unroll
    for (int j = 4; j < 8; ++j) {
        sc[j] = (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4);
        mn[j] = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// 2-D tiled tensor copy global -> shared (no multicast); x in bytes, a
// multiple of 16.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// one arrival per warp (after every lane's prior work)
__device__ __forceinline__ void warp_arrive(uint64_t *bar, int lane) {
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
}

__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity) { return mbar_wait_bounded(bar, parity); }

// 4 packed bytes -> 8 fp16 values nibble * sc: {lo 0,2}, {lo 1,3}, {hi 0,2}, {hi 1,3}
__device__ __forceinline__ void tc_expand4(uint32_t w, __half2 lo_sc, __half2 lo_off, __half2 hi_sc, __half2 hi_off,
                                           uint32_t *lo, uint32_t *hi) {
    const uint32_t m = 0x000F000Fu, mg = 0x64006400u;
    uint32_t a = (w & m) | mg, b = ((w >> 8) & m) | mg, c = ((w >> 4) & m) | mg, e = ((w >> 12) & m) | mg;
    const __half2 ra = __hfma2(*reinterpret_cast<__half2 *>(&a), lo_sc, lo_off);
    const __half2 rb = __hfma2(*reinterpret_cast<__half2 *>(&b), lo_sc, lo_off);
    const __half2 rc = __hfma2(*reinterpret_cast<__half2 *>(&c), hi_sc, hi_off);
    const __half2 re = __hfma2(*reinterpret_cast<__half2 *>(&e), hi_sc, hi_off);
    lo[0] = *reinterpret_cast<const uint32_t *>(&ra);
    lo[1] = *reinterpret_cast<const uint32_t *>(&rb);
    hi[0] = *reinterpret_cast<const uint32_t *>(&rc);
    hi[1] = *reinterpret_cast<const uint32_t *>(&re);
}

__global__ void __launch_bounds__(kTcThreads, 2)
    tc_q4k_project_kernel(const __grid_constant__ CUtensorMap wmap, const TcParams p) {
    extern __shared__ uint8_t tc_raw_smem[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_raw_smem) + 127) & ~uintptr_t(127));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kTcRows, mt = blockIdx.y, m0 = mt * kTcToks;
    const int nb = p.K / 256, nkc = p.K / kTcKc;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + TcSmem::bar_off);
    uint64_t *raw_full = bars, *raw_empty = raw_full + kTcRaw;
    uint64_t *b_full = raw_empty + kTcRaw, *b_empty = b_full + kTcBStages;
    uint64_t *a_full = b_empty + kTcBStages, *a_empty = a_full + kTcAStages;
    uint64_t *acc_full = a_empty + kTcAStages, *acc_empty = acc_full + 2;
    uint64_t *e_full = acc_empty + 2, *e_empty = e_full + kTcE;
    uint64_t *mma_done = e_empty + kTcE;  // every MMA of this CTA retired (before dealloc)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    static_assert(2 * (kTcRaw + kTcBStages + kTcAStages + 2 + kTcE) + 2 < 512 / 8, "barrier area");
    if (tid == 0) {
        for (int i = 0; i < kTcRaw; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 4 + 1);  // converter warps + the MMA commit after the min tile
        }
        for (int i = 0; i < kTcBStages; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < kTcAStages; ++i) {
            mbar_init(&a_full[i], 4);  // converter warps
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);  // epilogue warps
        }
        for (int i = 0; i < kTcE; ++i) {
            mbar_init(&e_full[i], 4);
            mbar_init(&e_empty[i], 4);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTcTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int nrows = min(kTcRows, p.n - n0);

    if (warp == 0) {
        // ------------------------------------------------------- producer
        const uint64_t pol = l2_evict_first_policy();
        int c = 0;           // operand chunks issued
        int raw_issued = 0;  // super-blocks issued
        bool ok = true;
        for (int b = 0; b < nb && ok; ++b) {
            const int r = b % kTcRaw;
            if (b >= kTcRaw && !tc_wait(&raw_empty[r], ((b / kTcRaw) - 1) & 1)) break;
            raw_issued = b + 1;
            if (lane == 0) {
                // one 2-D tensor copy: 128 rows x the 144-byte block b (rows
                // past the matrix read as zeros), the bsum16 tile, the scales
                mbar_arrive_expect_tx(&raw_full[r], (uint32_t)(kTcRows * 144 + kTcBBs + kTcXsBytes));
                tma_load_2d(sm + TcSmem::raw_off + r * kTcRows * 144, &wmap, b * 144, n0, &raw_full[r], pol);
                bulk_g2s(sm + TcSmem::bs_off + r * kTcBBs, p.bs16 + ((size_t)mt * nb + b) * (kTcToks * 16), kTcBBs,
                         &raw_full[r], pol);
                bulk_g2s(sm + TcSmem::xs_off + r * kTcXsBytes, p.xs + ((size_t)mt * nb + b) * kTcToks, kTcXsBytes,
                         &raw_full[r], pol);
            }
            __syncwarp();
            for (int q = 0; q < 4; ++q, ++c) {
                const int s = c % kTcBStages;
                if (c >= kTcBStages && !tc_wait(&b_empty[s], ((c / kTcBStages) - 1) & 1)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&b_full[s], kTcBTile);
                    bulk_g2s(sm + TcSmem::b_off + s * kTcBStage,
                             p.x16 + ((size_t)mt * nkc + (size_t)b * 4 + q) * (kTcToks * kTcKc), kTcBTile, &b_full[s],
                             pol);
                }
                __syncwarp();
            }
        }
        // drain: the last copy issued into every stage has landed before the
        // CTA can exit (a consumer that gave up no longer waits for it)
        for (int r = 0; r < kTcRaw; ++r) {
            int last = -1;
            for (int b = r; b < raw_issued; b += kTcRaw) last = b;
            if (last >= 0) tc_wait(&raw_full[r], (last / kTcRaw) & 1);
        }
        for (int s = 0; s < kTcBStages; ++s) {
            int last = -1;
            for (int i = s; i < c; i += kTcBStages) last = i;
            if (last >= 0) tc_wait(&b_full[s], (last / kTcBStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            int c = 0;
            bool ok = true;
            for (int b = 0; b < nb && ok; ++b) {
                const int r = b % kTcRaw;
                const uint32_t set = tmem;
                if (b >= 1) ok = tc_wait(&acc_empty[0], (b - 1) & 1);
                ok = ok && tc_wait(&raw_full[r], (b / kTcRaw) & 1);  // the bsum16 tile has landed
                tc_fence_after();
                for (int q = 0; q < 4 && ok; ++q, ++c) {
                    const int sa = c % kTcAStages, sb = c % kTcBStages;
                    ok = tc_wait(&b_full[sb], (c / kTcBStages) & 1) && tc_wait(&a_full[sa], (c / kTcAStages) & 1);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t abase = smem_u32(sm + TcSmem::a_off + sa * kTcAStage);
                    const uint32_t bbase = smem_u32(sm + TcSmem::b_off + sb * kTcBStage);
                    const uint32_t acc = set + (q >> 1) * kTcToks;  // K half: chunks 0-1 / 2-3
#pragma unroll
                    for (int k = 0; k < kTcKc / 16; ++k)
                        tc_mma(acc, umma_desc(abase + k * 256, 128, 1024), umma_desc(bbase + k * 256, 128, 1024),
                               ((q & 1) || k > 0) ? 1u : 0u);
                    if (q == 0) {
                        // minAcc: m[j/2] x bsum16_j, K = 16, from this super-block's ring slot,
                        // which is released once these MMAs have read it
                        tc_mma(set + 2 * kTcToks, umma_desc(smem_u32(sm + TcSmem::amin_off + r * kTcAMin), 128, 256),
                               umma_desc(smem_u32(sm + TcSmem::bs_off + r * kTcBBs), 128, 256), 0u);
                        tc_commit(&raw_empty[r]);
                    }
                    tc_commit(&a_empty[sa]);  // the stages are free once these MMAs have read them
                    tc_commit(&b_empty[sb]);
                }
                if (ok) tc_commit(&acc_full[0]);  // super-block b's integer sums are in TMEM
            }
            // every MMA issued has retired before TMEM is released
            tc_commit(mma_done);
            tc_wait(mma_done, 0);
        }
        __syncwarp();
    } else if (warp < 6) {
        // ---------------------------------------------------- converters
        const int row = tid - 64;  // 0..127
        const bool valid = row < nrows;
        int c = 0;
        bool ok = true;
        for (int b = 0; b < nb && ok; ++b) {
            const int r = b % kTcRaw, e = b % kTcE;
            if (!tc_wait(&raw_full[r], (b / kTcRaw) & 1)) break;
            const uint8_t *blk = sm + TcSmem::raw_off + (r * kTcRows + row) * 144;
            int sc[8], mn[8];
            float d = 0.0f, dmin = 0.0f;
            tc_unpack_scales(blk, valid, sc, mn, &d, &dmin);
            // the epilogue's share of the block: d, dmin per row and the token scales
            if (b >= kTcE && !tc_wait(&e_empty[e], ((b / kTcE) - 1) & 1)) break;
            uint8_t *es = sm + TcSmem::e_off + e * kTcEBytes;
            reinterpret_cast<float2 *>(es)[row] = make_float2(d, dmin);
            if (row < kTcToks)
                reinterpret_cast<float *>(es + kTcRows * 8)[row] =
                    reinterpret_cast<const float *>(sm + TcSmem::xs_off + r * kTcXsBytes)[row];
            warp_arrive(&e_full[e], lane);
#pragma unroll
            for (int q = 0; q < 4; ++q, ++c) {
                const int s = c % kTcAStages;
                // this chunk's 32 packed bytes (low nibbles: sub-block 2q, high: 2q+1)
                uint4 wv[2];
                wv[0] = valid ? reinterpret_cast<const uint4 *>(blk + 16 + 32 * q)[0] : make_uint4(0, 0, 0, 0);
                wv[1] = valid ? reinterpret_cast<const uint4 *>(blk + 16 + 32 * q)[1] : make_uint4(0, 0, 0, 0);
                if (c >= kTcAStages && !tc_wait(&a_empty[s], ((c / kTcAStages) - 1) & 1)) {
                    ok = false;
                    break;
                }
                const __half lsc = __int2half_rn(sc[2 * q]), hsc = __int2half_rn(sc[2 * q + 1]);
                const __half2 lo_sc = __halves2half2(lsc, lsc), hi_sc = __halves2half2(hsc, hsc);
                const __half lof = __int2half_rn(-1024 * sc[2 * q]), hof = __int2half_rn(-1024 * sc[2 * q + 1]);
                const __half2 lo_off = __halves2half2(lof, lof), hi_off = __halves2half2(hof, hof);
                uint8_t *a = sm + TcSmem::a_off + s * kTcAStage + (row >> 3) * 1024 + (row & 7) * 16;
                const uint32_t *wd = reinterpret_cast<const uint32_t *>(wv);
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    uint32_t lo[4], hi[4];
                    tc_expand4(wd[2 * g], lo_sc, lo_off, hi_sc, hi_off, lo, hi);
                    tc_expand4(wd[2 * g + 1], lo_sc, lo_off, hi_sc, hi_off, lo + 2, hi + 2);
                    *reinterpret_cast<uint4 *>(a + g * 128) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    *reinterpret_cast<uint4 *>(a + (g + 4) * 128) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                }
                if (q == 0) {
                    // the minAcc operand: m[j/2] for K = 0..15
                    uint8_t *am = sm + TcSmem::amin_off + r * kTcAMin + (row >> 3) * 256 + (row & 7) * 16;
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        uint32_t h[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const __half v = __int2half_rn(mn[4 * g + j]);
                            const __half2 v2 = __halves2half2(v, v);
                            h[j] = *reinterpret_cast<const uint32_t *>(&v2);
                        }
                        *reinterpret_cast<uint4 *>(am + g * 128) = make_uint4(h[0], h[1], h[2], h[3]);
                    }
                }
                fence_proxy_async_smem();
                warp_arrive(&a_full[s], lane);
            }
            warp_arrive(&raw_empty[r], lane);
        }
    } else {
        // ------------------------------------------------------ epilogue
        const int lane_base = 32 * (warp & 3);   // TMEM lanes this warp may read
        const int row = lane_base + lane;        // weight row in the tile; all 64 token columns
        const uint32_t lane_addr = tmem + ((uint32_t)lane_base << 16);
        for (int b = 0; b < nb; ++b) {
            const int e = b % kTcE;
            if (!tc_wait(&e_full[e], (b / kTcE) & 1) || !tc_wait(&acc_full[0], b & 1)) break;
            tc_fence_after();
            const uint8_t *es = sm + TcSmem::e_off + e * kTcEBytes;
            const float2 ddm = reinterpret_cast<const float2 *>(es)[row];
            const float d = ddm.x, dmin = ddm.y;
            const float *xs = reinterpret_cast<const float *>(es + kTcRows * 8);
            const uint32_t set = lane_addr;
#pragma unroll 1
            for (int piece = 0; piece < 4; ++piece) {
                const int cb = 16 * piece;
                uint32_t lo[16], hi[16], mi[16], ov[16];
                tmem_ld16_nowait(set + cb, lo);
                tmem_ld16_nowait(set + kTcToks + cb, hi);
                tmem_ld16_nowait(set + 2 * kTcToks + cb, mi);
                if (b > 0) tmem_ld16_nowait(lane_addr + kTcOutCol + cb, ov);
                tmem_ld_wait();
                if (piece == 3) {
                    // every accumulator value is in registers or already folded in
                    tc_fence_before();
                    warp_arrive(&acc_empty[0], lane);
                }
                float out[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    // (float)mainAcc: the exact halves added with one rounding
                    const float mainf = fadd(__uint_as_float(lo[j]), __uint_as_float(hi[j]));
                    const float term =
                        fmul(xs[cb + j], fsub(fmul(d, mainf), fmul(dmin, __uint_as_float(mi[j]))));
                    out[j] = b > 0 ? fadd(__uint_as_float(ov[j]), term) : fadd(0.0f, term);
                }
                tmem_st16(lane_addr + kTcOutCol + cb, out);
            }
            tmem_st_wait();
            warp_arrive(&e_empty[e], lane);
        }
        // the row's outputs: bias after the sum, then the residual
        const int n = n0 + row;
#pragma unroll 1
        for (int piece = 0; piece < 4; ++piece) {
            uint32_t ov[16];
            tmem_ld16_nowait(lane_addr + kTcOutCol + 16 * piece, ov);
            tmem_ld_wait();
            if (row < nrows) {
                const float bv = p.bias ? p.bias[n] : 0.0f;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = m0 + 16 * piece + j;
                    if (m < p.rows) {
                        float y = p.bias ? fadd(bv, __uint_as_float(ov[j])) : __uint_as_float(ov[j]);
                        if (p.resid) y = fadd(p.resid[(size_t)m * p.n + n], y);
                        p.y[(size_t)m * p.n + n] = y;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
    }
}

static int64_t tc_mtiles(int64_t rows) { return (rows + kTcToks - 1) / kTcToks; }

int64_t tc_scratch_bytes(int64_t rows, int64_t k) {
    const int64_t mt = tc_mtiles(rows), nb = k / 256;
    return mt * kTcToks * k * 2 + mt * nb * (kTcBBs + kTcXsBytes) + 256;
}

bool tc_project_supported(int type, int64_t n, int64_t k, int64_t rows) {
    return type == OVF_TYPE_Q4_K && k % 256 == 0 && k >= 256 && n >= 1 && rows >= 1 && n <= 0x7FFFFFFF;
}

// The packed operands of a batch of Q8_K rows in `scratch`
// (tc_scratch_bytes(rows, k)): fp16 activation tiles, bsum16 tiles and token
// scales (tc_pack_kernel); the tiles' and scales' addresses are returned.
static ovf_status launch_tc_pack(const int8_t *aq, const float *as, const int16_t *ab, int64_t rows, int64_t k,
                                 void *scratch, cudaStream_t st, const __half **x16_out, const float **xs_out) {
    const int64_t mtiles = tc_mtiles(rows), nb = k / 256;
    uint8_t *base = static_cast<uint8_t *>(scratch);
    __half *x16 = reinterpret_cast<__half *>(base);
    __half *bs16 = reinterpret_cast<__half *>(base + mtiles * kTcToks * k * 2);
    float *xs = reinterpret_cast<float *>(base + mtiles * kTcToks * k * 2 + mtiles * nb * kTcBBs);
    tc_pack_kernel<<<dim3((unsigned)(k / kTcKc), (unsigned)mtiles), 256, 0, st>>>(aq, as, ab, (int)rows, (int)k, x16,
                                                                                  bs16, xs);
    if (x16_out) *x16_out = x16;
    if (xs_out) *xs_out = xs;
    return cuda_status(cudaGetLastError(), "tc_pack");
}

// A 2-D tiled tensor map over a byte matrix [rows][inner] (row stride in
// bytes, a multiple of 16), box `box_rows` x `box_inner` bytes (box_inner a
// multiple of 16, at most 256), no swizzle, zero fill past the edges.
static ovf_status encode_bytes_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t rows,
                                  uint64_t row_stride, uint32_t box_inner, uint32_t box_rows) {
    // resolved once, thread-safely (function-local static initialisation)
    static const PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        return e == cudaSuccess && q == cudaDriverEntryPointSuccess ? reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn)
                                                                    : nullptr;
    }();
    if (!encode) {
        set_error("tensor map: cuTensorMapEncodeTiled unavailable");
        return OVF_ECUDA;
    }
    const cuuint64_t gdim[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)row_stride};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult cr = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), gdim, gstride, box,
                               estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) {
        set_error("tensor map encode failed (CUresult %d)", (int)cr);
        return OVF_EINVAL;
    }
    return OVF_OK;
}

// y [rows x n] (+ bias, + resid) from the Q8_K rows (aq, as, ab) and Q4_K
// weights; scratch holds tc_scratch_bytes(rows, k).
ovf_status launch_tc_project(int type, const void *w, const float *bias, const int8_t *aq, const float *as,
                             const int16_t *ab, float *y, int64_t n, int64_t k, int64_t rows, void *scratch,
                             cudaStream_t st, const float *resid) {
    OVF_CHECK_ARG(tc_project_supported(type, n, k, rows), "tensor-core projection: unsupported shape/type");
    OVF_CHECK_ARG(aligned16(w) && scratch && aligned16(scratch), "tensor-core projection: alignment");
    const int64_t mtiles = tc_mtiles(rows), ntiles = (n + kTcRows - 1) / kTcRows, nb = k / 256;
    OVF_CHECK_ARG(mtiles <= 65535, "tensor-core projection: too many rows");
    uint8_t *base = static_cast<uint8_t *>(scratch);
    const __half *bs16 = reinterpret_cast<const __half *>(base + mtiles * kTcToks * k * 2);
    const __half *x16 = nullptr;
    const float *xs = nullptr;
    if (ovf_status r = launch_tc_pack(aq, as, ab, rows, k, scratch, st, &x16, &xs)) return r;
    cudaError_t e = cudaSuccess;
    static PerDeviceOnce attr_once;
    const int dev = current_device();
    if (attr_once.pending(dev)) {
        e = cudaFuncSetAttribute(tc_q4k_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TcSmem::total);
        if (e != cudaSuccess) return cuda_status(e, "tc attribute");
        attr_once.mark(dev);
    }
    // the weight matrix as a 2-D byte tensor [n][nb * 144], box 128 x 144
    CUtensorMap wmap;
    if (ovf_status r = encode_bytes_2d(&wmap, w, (uint64_t)nb * 144, (uint64_t)n, (uint64_t)nb * 144, 144,
                                       (uint32_t)kTcRows))
        return r;
    TcParams p{};
    p.w = static_cast<const uint8_t *>(w);
    p.x16 = x16;
    p.bs16 = bs16;
    p.xs = xs;
    p.bias = bias;
    p.resid = resid;
    p.y = y;
    p.n = (int)n;
    p.K = (int)k;
    p.rows = (int)rows;
    tc_q4k_project_kernel<<<dim3((unsigned)ntiles, (unsigned)mtiles), kTcThreads, TcSmem::total, st>>>(wmap, p);
    return cuda_status(cudaGetLastError(), "tc_q4k_project");
}

}  // namespace ovf
