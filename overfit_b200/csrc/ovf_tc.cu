// ovf_tc.cu — the prefill projection of Q4_K weights on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM), bit-identical to the
// reference's per-row dot (Runtime/Q4KDotKernel.cs:216-256 via
// ProjectBatchedWeightStationary :819-955) and so to batched_project_kernel.
//
// Exactness.  Per row n, token m and super-block b the reference forms two
// integers, mainAcc = sum_s sc[s] * sum_{k in s} q4[k] q8[k] and minAcc =
// sum_s m[s] * bsum_s, then term = xs * (d * mainAcc - dmin * minAcc) in fp32
// and adds the terms in ascending b.  The tensor cores compute the integer
// part: A = the weights as fp16 integers (q4 - 8) * sc in [-504, 441], B =
// the Q8_K activation as fp16 integers in [-127, 127], fp32 accumulation over
// the 256 products of one super-block.  Every product and partial sum is an
// integer below 504 * 127 * 256 < 2^24 in magnitude, so the fp32 sum is exact
// in any order; mainAcc = acc + 8 * sum_s sc[s] * bsum_s restores the
// uncentered value.  The epilogue then runs the reference's fp32 tail and
// the ascending-b sum per (n, m).
//
// Layout.  A CTA owns 128 weight rows x 128 tokens; per super-block four
// K-chunks of 64 flow through a 4-deep ring of fp16 operand tiles in the
// UMMA no-swizzle K-major layout (8x16-byte core matrices; K-adjacent core
// matrices 128 B apart, 8-row groups 1024 B apart).  Warp roles, linked by
// mbarriers:
//   warp 0      producer: 1-D bulk copies of the raw Q4_K blocks (128 rows of
//               144 B per super-block), the pre-packed fp16 activation chunks
//               and the per-token metadata (bsum pairs, scales);
//   warp 1      TMEM allocation and the single MMA-issuing thread: 4 MMAs
//               (M=128, N=128, K=16) per chunk into one of two TMEM
//               accumulators (one per super-block parity), tcgen05.commit to
//               release the operand stage and to publish the accumulator;
//   warps 2-5   converters: thread = weight row; unpack the row's nibbles and
//               6-bit scales, write (q4 - 8) * sc as fp16 into the A tile;
//   warps 6-13  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//               lanes 32*(w%4).., 64 token columns), the fp32 tail, the
//               running per-(row, token) sum (kept in a third TMEM region).
// The operands live in this GPU's shared memory only; no cluster, no
// multicast.  Every mbarrier wait is bounded (the device error word is set
// and the kernel drains instead of hanging).
#include "ovf_internal.cuh"

namespace ovf {

static constexpr int kTcRows = 128;     // weight rows per CTA (MMA M, TMEM lanes)
static constexpr int kTcToks = 128;     // tokens per CTA (MMA N, TMEM columns per accumulator)
static constexpr int kTcKc = 64;        // K per operand chunk
static constexpr int kTcStages = 4;     // operand ring depth (chunks)
static constexpr int kTcRaw = 3;        // raw super-block ring depth
static constexpr int kTcThreads = 448;  // 14 warps
static constexpr int kTcTileBytes = kTcRows * kTcKc * 2;  // 16 KB per operand tile
static constexpr int kTcMetaBytes = kTcToks * 16 + kTcToks * 4;  // bsum pairs [128][8] int16 + scales [128]
// TMEM columns: two accumulators [0, 256) and the running sums [256, 384)
static constexpr int kTcOutCol = 2 * kTcToks;
static constexpr int kTcTmemCols = 512;

// shared memory map (bytes from a 1024-aligned base)
struct TcSmem {
    static constexpr int a_off = 0;                                        // [stages] A tiles
    static constexpr int b_off = a_off + kTcStages * kTcTileBytes;          // [stages] B tiles
    static constexpr int raw_off = b_off + kTcStages * kTcTileBytes;        // [raw] Q4_K blocks [128][144]
    static constexpr int meta_off = raw_off + kTcRaw * kTcRows * 144;       // [raw] token metadata
    static constexpr int bar_off = meta_off + kTcRaw * kTcMetaBytes;        // mbarriers
    static constexpr int total = bar_off + 256 + 1024;                      // + alignment slack
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    // no-swizzle K-major: LBO = 128 B (K-adjacent core matrices), SBO = 1024 B
    // (8-row groups), descriptor version 1
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)(128 >> 4) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// kind::f16, fp16 A and B (K-major), fp32 accumulator, M = 128, N = 128
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

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
        "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Activation packing: the Q8_K rows of a batch as fp16 operand tiles in the
// UMMA layout, [token tile][K chunk][128 x 64], and per (token tile, super-
// block) the tokens' bsum pairs (bsum[2s] + bsum[2s+1], int16 [128][8]) and
// scales (float [128]).  Tokens past `rows` are zero.
__global__ void tc_pack_kernel(const int8_t *__restrict__ aq, const float *__restrict__ as,
                               const int16_t *__restrict__ ab, int rows, int K, __half *__restrict__ x16,
                               uint8_t *__restrict__ meta) {
    const int mt = blockIdx.y, kc = blockIdx.x;  // token tile, K chunk
    const int nkc = K / kTcKc;
    __half *dst = x16 + ((size_t)mt * nkc + kc) * (kTcToks * kTcKc);
    for (int i = threadIdx.x; i < kTcToks * 8; i += blockDim.x) {
        // one 8-element (16-byte) core-matrix row: token t, k group g
        const int t = i >> 3, g = i & 7, m = mt * kTcToks + t;
        __align__(16) __half h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int v = m < rows ? aq[(size_t)m * K + kc * kTcKc + 8 * g + j] : 0;
            h[j] = __int2half_rn(v);
        }
        *reinterpret_cast<uint4 *>(dst + (t >> 3) * 512 + g * 64 + (t & 7) * 8) = *reinterpret_cast<const uint4 *>(h);
    }
    if ((kc & 3) == 0) {
        const int b = kc >> 2, nb = K / 256;
        uint8_t *mb = meta + ((size_t)mt * nb + b) * kTcMetaBytes;
        for (int t = threadIdx.x; t < kTcToks; t += blockDim.x) {
            const int m = mt * kTcToks + t;
            int16_t *bs = reinterpret_cast<int16_t *>(mb) + t * 8;
#pragma unroll
            for (int s = 0; s < 8; ++s)
                bs[s] = m < rows ? (int16_t)(ab[(size_t)m * (K / 16) + b * 16 + 2 * s] +
                                             ab[(size_t)m * (K / 16) + b * 16 + 2 * s + 1])
                                 : (int16_t)0;
            reinterpret_cast<float *>(mb + kTcToks * 16)[t] = m < rows ? as[(size_t)m * nb + b] : 0.0f;
        }
    }
}

struct TcParams {
    const uint8_t *w;      // Q4_K [n][K/256] blocks
    const __half *x16;     // packed activation tiles
    const uint8_t *meta;   // packed token metadata
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
    *d = __half2float(*reinterpret_cast<const __half *>(blk));
    *dmin = __half2float(*reinterpret_cast<const __half *>(blk + 2));
    const uint8_t *q = blk + 4;
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

__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity) { return mbar_wait_sleep_bounded(bar, parity); }

__global__ void __launch_bounds__(kTcThreads, 1) tc_q4k_project_kernel(const TcParams p) {
    extern __shared__ uint8_t tc_raw_smem[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_raw_smem) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kTcRows, mt = blockIdx.y, m0 = mt * kTcToks;
    const int nb = p.K / 256, nkc = p.K / kTcKc;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + TcSmem::bar_off);
    uint64_t *raw_full = bars, *raw_empty = bars + kTcRaw;            // raw super-block stages
    uint64_t *b_full = bars + 2 * kTcRaw, *a_full = b_full + kTcStages, *op_empty = a_full + kTcStages;
    uint64_t *acc_full = op_empty + kTcStages, *acc_empty = acc_full + 2;
    uint64_t *mma_done = acc_empty + 2;  // every MMA of this CTA retired (before dealloc)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 3);
    if (tid == 0) {
        for (int i = 0; i < kTcRaw; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 128 + 256);  // converters + epilogue threads
        }
        for (int i = 0; i < kTcStages; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&a_full[i], 128);
            mbar_init(&op_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 256);
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
    const size_t row_stride = (size_t)nb * 144;
    const int nrows = min(kTcRows, p.n - n0);

    if (warp == 0) {
        // ------------------------------------------------------- producer
        const uint64_t pol = l2_evict_first_policy();
        int c = 0;           // B chunks issued
        int raw_issued = 0;  // raw super-blocks issued
        bool ok = true;
        for (int b = 0; b < nb && ok; ++b) {
            const int r = b % kTcRaw;
            if (b >= kTcRaw && !tc_wait(&raw_empty[r], ((b / kTcRaw) - 1) & 1)) break;
            raw_issued = b + 1;
            if (lane == 0) mbar_arrive_expect_tx(&raw_full[r], (uint32_t)(nrows * 144 + kTcMetaBytes));
            __syncwarp();
            uint8_t *raw = sm + TcSmem::raw_off + r * kTcRows * 144;
            for (int i = lane; i < nrows; i += 32)
                bulk_g2s(raw + i * 144, p.w + (size_t)(n0 + i) * row_stride + (size_t)b * 144, 144, &raw_full[r], pol);
            if (lane == 0)
                bulk_g2s(sm + TcSmem::meta_off + r * kTcMetaBytes, p.meta + ((size_t)mt * nb + b) * kTcMetaBytes,
                         kTcMetaBytes, &raw_full[r], pol);
            for (int q = 0; q < 4; ++q, ++c) {
                const int s = c % kTcStages;
                if (c >= kTcStages && !tc_wait(&op_empty[s], ((c / kTcStages) - 1) & 1)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&b_full[s], kTcTileBytes);
                    bulk_g2s(sm + TcSmem::b_off + s * kTcTileBytes,
                             p.x16 + ((size_t)mt * nkc + (size_t)b * 4 + q) * (kTcToks * kTcKc), kTcTileBytes,
                             &b_full[s], pol);
                }
                __syncwarp();
            }
        }
        // drain: the last copy issued into every stage has landed before the
        // CTA can exit (a consumer that gave up no longer waits for it)
        const int braw = raw_issued;
        for (int r = 0; r < kTcRaw; ++r) {
            int last = -1;
            for (int b = r; b < braw; b += kTcRaw) last = b;
            if (last >= 0) tc_wait(&raw_full[r], (last / kTcRaw) & 1);
        }
        for (int s = 0; s < kTcStages; ++s) {
            int last = -1;
            for (int i = s; i < c; i += kTcStages) last = i;
            if (last >= 0) tc_wait(&b_full[s], (last / kTcStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            int c = 0;
            bool ok = true;
            for (int b = 0; b < nb && ok; ++b) {
                const int buf = b & 1;
                if (b >= 2) ok = tc_wait(&acc_empty[buf], ((b >> 1) - 1) & 1);
                tc_fence_after();
                for (int q = 0; q < 4 && ok; ++q, ++c) {
                    const int s = c % kTcStages;
                    ok = tc_wait(&a_full[s], (c / kTcStages) & 1) && tc_wait(&b_full[s], (c / kTcStages) & 1);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t abase = smem_u32(sm + TcSmem::a_off + s * kTcTileBytes);
                    const uint32_t bbase = smem_u32(sm + TcSmem::b_off + s * kTcTileBytes);
#pragma unroll
                    for (int k = 0; k < kTcKc / 16; ++k)
                        tc_mma(tmem + buf * kTcToks, umma_desc(abase + k * 256), umma_desc(bbase + k * 256),
                               (q > 0 || k > 0) ? 1u : 0u);
                    tc_commit(&op_empty[s]);  // the stage is free once these MMAs have read it
                }
                if (ok) tc_commit(&acc_full[buf]);  // super-block b's integer sums are in TMEM
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
            const int r = b % kTcRaw;
            if (!tc_wait(&raw_full[r], (b / kTcRaw) & 1)) break;
            const uint8_t *blk = sm + TcSmem::raw_off + (r * kTcRows + row) * 144;
            int sc[8], mn[8];
            float d = 0.0f, dmin = 0.0f;
            tc_unpack_scales(blk, valid, sc, mn, &d, &dmin);
            for (int q = 0; q < 4; ++q, ++c) {
                const int s = c % kTcStages;
                if (c >= kTcStages && !tc_wait(&op_empty[s], ((c / kTcStages) - 1) & 1)) {
                    ok = false;
                    break;
                }
                // chunk q = elements 64q .. 64q+63: low nibbles of qs[32q..] (sub-block
                // 2q), then high nibbles (sub-block 2q+1)
                uint8_t *a = sm + TcSmem::a_off + s * kTcTileBytes + (row >> 3) * 1024 + (row & 7) * 16;
                const uint8_t *qs = blk + 16 + 32 * q;
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const int hi = g >> 2;  // core matrices 0-3: low nibbles, 4-7: high
                    const int scv = valid ? sc[2 * q + hi] : 0;
                    __align__(16) __half h[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int byte = valid ? qs[(g & 3) * 8 + j] : 8;
                        const int nib = hi ? (byte >> 4) : (byte & 15);
                        h[j] = __int2half_rn((nib - 8) * scv);
                    }
                    *reinterpret_cast<uint4 *>(a + g * 128) = *reinterpret_cast<const uint4 *>(h);
                }
                fence_proxy_async_smem();
                mbar_arrive(&a_full[s]);
            }
            mbar_arrive(&raw_empty[r]);
        }
    } else {
        // ------------------------------------------------------ epilogue
        const int ew = warp - 6;                 // 0..7
        const int lane_base = 32 * (warp & 3);   // TMEM lanes this warp may read
        const int row = lane_base + lane;        // weight row in the tile
        const int col0 = 64 * (ew >> 2);         // token columns [col0, col0 + 64)
        const uint32_t lane_addr = tmem + ((uint32_t)lane_base << 16);
        for (int b = 0; b < nb; ++b) {
            const int r = b % kTcRaw, buf = b & 1;
            if (!tc_wait(&raw_full[r], (b / kTcRaw) & 1) || !tc_wait(&acc_full[buf], (b >> 1) & 1)) break;
            tc_fence_after();
            int sc8[8], mn8[8];
            float d, dmin;
            tc_unpack_scales(sm + TcSmem::raw_off + (r * kTcRows + row) * 144, row < nrows, sc8, mn8, &d, &dmin);
            const uint8_t *meta = sm + TcSmem::meta_off + r * kTcMetaBytes;
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                float acc[32], out[32];
                const int cb = col0 + 32 * half;
                tmem_ld32(lane_addr + buf * kTcToks + cb, acc);
                if (b > 0) {
                    tmem_ld32(lane_addr + kTcOutCol + cb, out);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) out[j] = 0.0f;
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int t = cb + j;
                    const int4 bsv = *reinterpret_cast<const int4 *>(meta + t * 16);
                    const int16_t *bs = reinterpret_cast<const int16_t *>(&bsv);
                    int corr = 0, mins = 0;
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        corr += sc8[s] * (int)bs[s];
                        mins += mn8[s] * (int)bs[s];
                    }
                    const int main_acc = __float2int_rn(acc[j]) + 8 * corr;
                    const float xs = reinterpret_cast<const float *>(meta + kTcToks * 16)[t];
                    const float term = fmul(xs, fsub(fmul(d, (float)main_acc), fmul(dmin, (float)mins)));
                    out[j] = fadd(out[j], term);
                }
                tmem_st32(lane_addr + kTcOutCol + cb, out);
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[buf]);
            mbar_arrive(&raw_empty[r]);
        }
        // the row's outputs: bias after the sum, then the residual
        const int n = n0 + row;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
            float out[32];
            tmem_ld32(lane_addr + kTcOutCol + col0 + 32 * half, out);
            if (row < nrows) {
                const float bv = p.bias ? p.bias[n] : 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int m = m0 + col0 + 32 * half + j;
                    if (m < p.rows) {
                        float y = p.bias ? fadd(bv, out[j]) : out[j];
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

int64_t tc_scratch_bytes(int64_t rows, int64_t k) {
    const int64_t mtiles = (rows + kTcToks - 1) / kTcToks;
    return mtiles * kTcToks * k * 2 + mtiles * (k / 256) * kTcMetaBytes + 256;
}

bool tc_project_supported(int type, int64_t n, int64_t k, int64_t rows) {
    return type == OVF_TYPE_Q4_K && k % 256 == 0 && k >= 256 && n >= 1 && rows >= 1 && n <= 0x7FFFFFFF;
}

// y [rows x n] (+ bias, + resid) from the Q8_K rows (aq, as, ab) and Q4_K
// weights; scratch holds tc_scratch_bytes(rows, k).
ovf_status launch_tc_project(int type, const void *w, const float *bias, const int8_t *aq, const float *as,
                             const int16_t *ab, float *y, int64_t n, int64_t k, int64_t rows, void *scratch,
                             cudaStream_t st, const float *resid) {
    OVF_CHECK_ARG(tc_project_supported(type, n, k, rows), "tensor-core projection: unsupported shape/type");
    OVF_CHECK_ARG(aligned16(w) && scratch && aligned16(scratch), "tensor-core projection: alignment");
    const int64_t mtiles = (rows + kTcToks - 1) / kTcToks, ntiles = (n + kTcRows - 1) / kTcRows;
    OVF_CHECK_ARG(mtiles <= 65535, "tensor-core projection: too many rows");
    __half *x16 = static_cast<__half *>(scratch);
    uint8_t *meta = static_cast<uint8_t *>(scratch) + mtiles * kTcToks * k * 2;
    tc_pack_kernel<<<dim3((unsigned)(k / kTcKc), (unsigned)mtiles), 256, 0, st>>>(aq, as, ab, (int)rows, (int)k, x16,
                                                                                  meta);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "tc_pack");
    static PerDeviceOnce attr_once;
    const int dev = current_device();
    if (attr_once.pending(dev)) {
        e = cudaFuncSetAttribute(tc_q4k_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TcSmem::total);
        if (e != cudaSuccess) return cuda_status(e, "tc attribute");
        attr_once.mark(dev);
    }
    TcParams p{};
    p.w = static_cast<const uint8_t *>(w);
    p.x16 = x16;
    p.meta = meta;
    p.bias = bias;
    p.resid = resid;
    p.y = y;
    p.n = (int)n;
    p.K = (int)k;
    p.rows = (int)rows;
    tc_q4k_project_kernel<<<dim3((unsigned)ntiles, (unsigned)mtiles), kTcThreads, TcSmem::total, st>>>(p);
    return cuda_status(cudaGetLastError(), "tc_q4k_project");
}

}  // namespace ovf
