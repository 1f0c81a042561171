// ovf_tc6.cu — the prefill projection of Q6_K weights on the 5th-generation
// tensor cores (tcgen05.mma kind::f16, fp32 accumulators in TMEM),
// bit-identical to the reference's per-row Q6_K dot (Runtime/Q6KDotKernel.cs:
// 77-225 via ProjectBatched :403-525) and so to batched_project_kernel.
//
// Exactness.  Per weight row n, token m and super-block b the reference forms
// the integer mainAcc = sum_s sc[s] * sum_{k in s} (q6[k] - 32) * q8[k] over
// sixteen 16-element sub-blocks with signed 8-bit scales, then the term
// (d * q8scale) * (float)mainAcc, added in ascending b.  The scale is split
// as sc = 16 * sh + sl (sl in 0..15, sh in -8..7); the tensor cores compute
// lo = sum (q6 - 32) * sl * q8 and hi = sum (q6 - 32) * sh * q8 with fp16
// integer operands (|(q6 - 32) * sl| <= 480, |(q6 - 32) * sh| <= 256) and
// fp32 accumulation over the 256 products of the block: every partial sum is
// an integer below 2^24, so both are exact, and mainAcc = lo + 16 * hi is
// formed in int32 before the reference's fp32 tail.
//
// The 6-bit values are expanded with the fp16 magic-number trick
// (0x6400 | q = 1024 + q, then one fma per scale half), which yields the
// elements of an 8-group in the order 0,2,1,3,4,6,5,7 — the order
// tc_pack_kernel gives the activation tiles, which are shared with the Q4_K
// kernel.
//
// Layout.  A CTA owns 128 weight rows x 64 tokens.  Per super-block a 2-D
// tensor copy brings the 128 rows' 210-byte blocks (a 224-byte box at the
// 16-byte boundary below the block; the converters read it with aligned
// words and funnel shifts).  A operand chunks of K = 32 (a lo and a hi tile)
// and B chunks of K = 64 flow through 2-deep rings; one accumulator set
// (lo, hi) and the running sums live in TMEM (192 of 256 columns).  Warp
// roles as in tc_q4k_project_kernel: producer, MMA issuer, 4 converter warps
// (thread = weight row), 4 epilogue warps (thread = weight row, 64 tokens).
// Two CTAs per SM.  No cluster, no multicast; every wait is bounded.
#include "ovf_internal.cuh"

namespace ovf {

static constexpr int kT6Rows = 128, kT6Toks = 64;
static constexpr int kT6Threads = 320;                      // 10 warps
static constexpr int kT6Box = 224;                          // raw bytes per row per super-block
static constexpr int kT6RawBytes = kT6Rows * kT6Box;        // 28 KB
static constexpr int kT6XsBytes = kT6Toks * 4;
static constexpr int kT6ATile = kT6Rows * 32 * 2;           // 8 KB: 128 rows x K 32, fp16
static constexpr int kT6AStage = 2 * kT6ATile;              // lo and hi tiles
static constexpr int kT6BStage = kT6Toks * 64 * 2;          // 8 KB: 64 tokens x K 64, fp16
static constexpr int kT6EBytes = kT6Rows * 4 + kT6XsBytes;  // d per row + token scales
static constexpr int kT6Raw = 2, kT6AStages = 2, kT6BStages = 2, kT6E = 2;
static constexpr int kT6OutCol = 2 * kT6Toks;               // TMEM: lo [0,64) | hi [64,128) | out [128,192)
static constexpr int kT6TmemCols = 256;

struct T6Smem {
    static constexpr int raw_off = 0;
    static constexpr int xs_off = raw_off + kT6Raw * kT6RawBytes;
    static constexpr int a_off = xs_off + kT6Raw * kT6XsBytes;
    static constexpr int b_off = a_off + kT6AStages * kT6AStage;
    static constexpr int e_off = b_off + kT6BStages * kT6BStage;
    static constexpr int bar_off = e_off + kT6E * kT6EBytes;
    static constexpr int total = bar_off + 512 + 128;
};
static_assert(T6Smem::total <= 113 * 1024, "two CTAs per SM");
static_assert(T6Smem::xs_off % 128 == 0 && T6Smem::a_off % 128 == 0 && T6Smem::b_off % 128 == 0, "alignment");

// kind::f16, fp16 A and B (K-major), fp32 accumulator, M = 128, N = 64
static constexpr uint32_t kT6Idesc = (1u << 4) | ((uint32_t)(kT6Toks >> 3) << 17) | ((uint32_t)(kT6Rows >> 4) << 24);

__device__ __forceinline__ void t6_mma(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(adesc), "l"(bdesc), "r"(kT6Idesc), "r"(accumulate)
        : "memory");
}

// Four 6-bit values (one per byte of v) -> (q - 32) * s for the two scale
// halves: lo[0..1] / hi[0..1] hold the elements {0, 2} and {1, 3}.
__device__ __forceinline__ void t6_expand4(uint32_t v, __half2 sl, __half2 ol, __half2 sh, __half2 oh, uint32_t *lo,
                                           uint32_t *hi) {
    uint32_t a = (v & 0x00FF00FFu) | 0x64006400u, b = ((v >> 8) & 0x00FF00FFu) | 0x64006400u;
    const __half2 la = __hfma2(*reinterpret_cast<__half2 *>(&a), sl, ol);
    const __half2 lb = __hfma2(*reinterpret_cast<__half2 *>(&b), sl, ol);
    const __half2 ha = __hfma2(*reinterpret_cast<__half2 *>(&a), sh, oh);
    const __half2 hb = __hfma2(*reinterpret_cast<__half2 *>(&b), sh, oh);
    lo[0] = *reinterpret_cast<const uint32_t *>(&la);
    lo[1] = *reinterpret_cast<const uint32_t *>(&lb);
    hi[0] = *reinterpret_cast<const uint32_t *>(&ha);
    hi[1] = *reinterpret_cast<const uint32_t *>(&hb);
}

// The scale halves of a signed 8-bit sub-block scale as fp16 pairs with the
// matching offsets: x = 1024 + q gives x * s - 1056 * s = (q - 32) * s,
// exact (1056 * s = 33 * s * 32 needs 11 significant bits at most).
__device__ __forceinline__ void t6_scale_pairs(int sc, __half2 *sl, __half2 *ol, __half2 *sh, __half2 *oh) {
    const int l = sc & 15, h = sc >> 4;  // sc = 16 * h + l
    const __half hl = __int2half_rn(l), hh = __int2half_rn(h);
    const __half fl = __int2half_rn(-1056 * l), fh = __int2half_rn(-1056 * h);
    *sl = __halves2half2(hl, hl);
    *ol = __halves2half2(fl, fl);
    *sh = __halves2half2(hh, hh);
    *oh = __halves2half2(fh, fh);
}

struct T6Params {
    const __half *x16;  // packed activation tiles (tc_pack_kernel)
    const float *xs;    // packed token scales (tc_pack_kernel)
    const float *bias;  // [n] or null
    const float *resid; // [rows][n] or null
    float *y;           // [rows][n]
    int n, K, rows;
};

__global__ void __launch_bounds__(kT6Threads, 2)
    tc_q6k_project_kernel(const __grid_constant__ CUtensorMap wmap, const T6Params p) {
    extern __shared__ uint8_t t6_raw_smem[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(t6_raw_smem) + 127) & ~uintptr_t(127));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kT6Rows, mt = blockIdx.y, m0 = mt * kT6Toks;
    const int nb = p.K / 256, nkc = p.K / 64;  // super-blocks, B chunks (K = 64)
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + T6Smem::bar_off);
    uint64_t *raw_full = bars, *raw_empty = raw_full + kT6Raw;
    uint64_t *a_full = raw_empty + kT6Raw, *a_empty = a_full + kT6AStages;
    uint64_t *b_full = a_empty + kT6AStages, *b_empty = b_full + kT6BStages;
    uint64_t *e_full = b_empty + kT6BStages, *e_empty = e_full + kT6E;
    uint64_t *acc_full = e_empty + kT6E, *acc_empty = acc_full + 1, *mma_done = acc_empty + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    if (tid == 0) {
        for (int i = 0; i < kT6Raw; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 4);  // converter warps
        }
        for (int i = 0; i < kT6AStages; ++i) {
            mbar_init(&a_full[i], 4);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < kT6BStages; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < kT6E; ++i) {
            mbar_init(&e_full[i], 4);
            mbar_init(&e_empty[i], 4);  // epilogue warps
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 4);
        mbar_init(mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kT6TmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int nrows = min(kT6Rows, p.n - n0);

    if (warp == 0) {
        // ------------------------------------------------------- producer
        const uint64_t pol = l2_evict_first_policy();
        int raw_issued = 0, kc = 0;
        bool ok = true;
        for (int b = 0; b < nb && ok; ++b) {
            const int r = b % kT6Raw;
            if (b >= kT6Raw && !tc_wait(&raw_empty[r], ((b / kT6Raw) - 1) & 1)) break;
            raw_issued = b + 1;
            if (lane == 0) {
                // the rows' block b: a 224-byte box from the 16-byte boundary
                // at or below byte 210 * b (past the row end reads as zeros)
                mbar_arrive_expect_tx(&raw_full[r], (uint32_t)(kT6RawBytes + kT6XsBytes));
                tma_load_2d(sm + T6Smem::raw_off + r * kT6RawBytes, &wmap, (b * 210) & ~15, n0, &raw_full[r], pol);
                bulk_g2s(sm + T6Smem::xs_off + r * kT6XsBytes, p.xs + ((size_t)mt * nb + b) * kT6Toks, kT6XsBytes,
                         &raw_full[r], pol);
            }
            __syncwarp();
            for (int q = 0; q < 4; ++q, ++kc) {
                const int s = kc % kT6BStages;
                if (kc >= kT6BStages && !tc_wait(&b_empty[s], ((kc / kT6BStages) - 1) & 1)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&b_full[s], kT6BStage);
                    bulk_g2s(sm + T6Smem::b_off + s * kT6BStage, p.x16 + ((size_t)mt * nkc + kc) * (kT6Toks * 64),
                             kT6BStage, &b_full[s], pol);
                }
                __syncwarp();
            }
        }
        // drain: the last copy issued into every stage has landed before exit
        for (int r = 0; r < kT6Raw; ++r) {
            int last = -1;
            for (int b = r; b < raw_issued; b += kT6Raw) last = b;
            if (last >= 0) tc_wait(&raw_full[r], (last / kT6Raw) & 1);
        }
        for (int s = 0; s < kT6BStages; ++s) {
            int last = -1;
            for (int i = s; i < kc; i += kT6BStages) last = i;
            if (last >= 0) tc_wait(&b_full[s], (last / kT6BStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            bool ok = true;
            for (int b = 0; b < nb && ok; ++b) {
                if (b >= 1) ok = tc_wait(acc_empty, (b - 1) & 1);
                tc_fence_after();
                for (int cc = 0; cc < 8 && ok; ++cc) {
                    const int c = 8 * b + cc, sa = c % kT6AStages, kcg = c >> 1, sb = kcg % kT6BStages;
                    ok = tc_wait(&a_full[sa], (c / kT6AStages) & 1);
                    if (ok && (cc & 1) == 0) ok = tc_wait(&b_full[sb], (kcg / kT6BStages) & 1);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t alo = smem_u32(sm + T6Smem::a_off + sa * kT6AStage);
                    const uint32_t bbase = smem_u32(sm + T6Smem::b_off + sb * kT6BStage) + (cc & 1) * 512;
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const uint32_t acc = (cc > 0 || k > 0) ? 1u : 0u;
                        const uint64_t bd = umma_desc(bbase + k * 256, 128, 1024);
                        t6_mma(tmem, umma_desc(alo + k * 256, 128, 512), bd, acc);
                        t6_mma(tmem + kT6Toks, umma_desc(alo + kT6ATile + k * 256, 128, 512), bd, acc);
                    }
                    tc_commit(&a_empty[sa]);               // the A stage is free once these MMAs have read it
                    if (cc & 1) tc_commit(&b_empty[sb]);   // both halves of the B chunk are read
                }
                if (ok) tc_commit(acc_full);  // super-block b's integer sums are in TMEM
            }
            tc_commit(mma_done);
            tc_wait(mma_done, 0);
        }
        __syncwarp();
    } else if (warp < 6) {
        // ---------------------------------------------------- converters
        const int row = tid - 64;  // 0..127
        const bool valid = row < nrows;
        bool ok = true;
        for (int b = 0; b < nb && ok; ++b) {
            const int r = b % kT6Raw, e = b % kT6E;
            if (!tc_wait(&raw_full[r], (b / kT6Raw) & 1)) break;
            // the block starts (210 b) mod 16 bytes into the row's box; read it
            // as aligned words, funnel-shifted into place
            const uintptr_t bp = reinterpret_cast<uintptr_t>(sm + T6Smem::raw_off + r * kT6RawBytes + row * kT6Box +
                                                             ((b * 210) & 15));
            const uint32_t *wb = reinterpret_cast<const uint32_t *>(bp & ~uintptr_t(3));
            const int shb = (int)(bp & 3u) * 8;
            const float d = valid ? __half2float(__ushort_as_half((unsigned short)(ldw_shifted(wb, 52, shb) & 0xFFFFu)))
                                  : 0.0f;
            if (b >= kT6E && !tc_wait(&e_empty[e], ((b / kT6E) - 1) & 1)) break;
            uint8_t *es = sm + T6Smem::e_off + e * kT6EBytes;
            reinterpret_cast<float *>(es)[row] = d;
            if (row < kT6Toks)
                reinterpret_cast<float *>(es + kT6Rows * 4)[row] =
                    reinterpret_cast<const float *>(sm + T6Smem::xs_off + r * kT6XsBytes)[row];
            warp_arrive(&e_full[e], lane);
            for (int cc = 0; cc < 8; ++cc) {
                const int c = 8 * b + cc, sa = c % kT6AStages;
                const int hf = cc >> 2, k = cc & 3;  // half of the block, quarter within it
                // this chunk's two sub-block scales (elements 32 cc .. 32 cc + 31)
                const uint32_t scw = valid ? ldw_shifted(wb, 48 + (cc >> 1), shb) : 0u;
                const int sc0 = (int)(int8_t)byte_of(scw, 2 * (cc & 1)), sc1 = (int)(int8_t)byte_of(scw, 2 * (cc & 1) + 1);
                if (c >= kT6AStages && !tc_wait(&a_empty[sa], ((c / kT6AStages) - 1) & 1)) {
                    ok = false;
                    break;
                }
                uint8_t *alo = sm + T6Smem::a_off + sa * kT6AStage + (row >> 3) * 512 + (row & 7) * 16;
                uint8_t *ahi = alo + kT6ATile;
#pragma unroll
                for (int sub = 0; sub < 2; ++sub) {
                    __half2 sl, ol, sh, oh;
                    t6_scale_pairs(sub ? sc1 : sc0, &sl, &ol, &sh, &oh);
#pragma unroll
                    for (int g2 = 0; g2 < 2; ++g2) {
                        // core-matrix column g = 2 sub + g2: elements l = 8 g .. 8 g + 7
                        const int g = 2 * sub + g2;
                        uint32_t lo[4], hi[4];
#pragma unroll
                        for (int wi = 0; wi < 2; ++wi) {
                            const int l4 = 2 * g + wi;  // word of 4 elements: l = 4 l4 .. 4 l4 + 3
                            uint32_t v = 0;
                            if (valid) {
                                const uint32_t qlw = ldw_shifted(wb, 16 * hf + 8 * (k & 1) + l4, shb);
                                const uint32_t qhw = ldw_shifted(wb, 32 + 8 * hf + l4, shb);
                                v = ((qlw >> (4 * (k >> 1))) & 0x0F0F0F0Fu) | (((qhw >> (2 * k)) & 0x03030303u) << 4);
                            } else {
                                v = 0x20202020u;  // q = 32: a zero weight under any scale
                            }
                            t6_expand4(v, sl, ol, sh, oh, lo + 2 * wi, hi + 2 * wi);
                        }
                        *reinterpret_cast<uint4 *>(alo + g * 128) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        *reinterpret_cast<uint4 *>(ahi + g * 128) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    }
                }
                fence_proxy_async_smem();
                warp_arrive(&a_full[sa], lane);
            }
            warp_arrive(&raw_empty[r], lane);
        }
    } else {
        // ------------------------------------------------------ epilogue
        const int lane_base = 32 * (warp & 3);
        const int row = lane_base + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)lane_base << 16);
        for (int b = 0; b < nb; ++b) {
            const int e = b % kT6E;
            if (!tc_wait(&e_full[e], (b / kT6E) & 1) || !tc_wait(acc_full, b & 1)) break;
            tc_fence_after();
            const uint8_t *es = sm + T6Smem::e_off + e * kT6EBytes;
            const float d = reinterpret_cast<const float *>(es)[row];
            const float *xs = reinterpret_cast<const float *>(es + kT6Rows * 4);
#pragma unroll 1
            for (int piece = 0; piece < 4; ++piece) {
                const int cb = 16 * piece;
                uint32_t lo[16], hi[16], ov[16];
                tmem_ld16_nowait(lane_addr + cb, lo);
                tmem_ld16_nowait(lane_addr + kT6Toks + cb, hi);
                if (b > 0) tmem_ld16_nowait(lane_addr + kT6OutCol + cb, ov);
                tmem_ld_wait();
                if (piece == 3) {
                    tc_fence_before();
                    warp_arrive(acc_empty, lane);
                }
                float out[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int main_acc =
                        __float2int_rn(__uint_as_float(lo[j])) + 16 * __float2int_rn(__uint_as_float(hi[j]));
                    const float term = fmul(fmul(d, xs[cb + j]), i2f(main_acc));
                    out[j] = b > 0 ? fadd(__uint_as_float(ov[j]), term) : fadd(0.0f, term);
                }
                tmem_st16(lane_addr + kT6OutCol + cb, out);
            }
            tmem_st_wait();
            warp_arrive(&e_empty[e], lane);
        }
        // the row's outputs: bias after the sum, then the residual
        const int n = n0 + row;
#pragma unroll 1
        for (int piece = 0; piece < 4; ++piece) {
            uint32_t ov[16];
            tmem_ld16_nowait(lane_addr + kT6OutCol + 16 * piece, ov);
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kT6TmemCols) : "memory");
    }
}

bool tc6_project_supported(int64_t n, int64_t k, int64_t rows) {
    // the weight rows (k / 256 blocks of 210 bytes) must be whole 16-byte units
    return k % 2048 == 0 && n >= 1 && rows >= 1 && n <= 0x7FFFFFFF;
}

// y [rows x n] (+ bias, + resid) from the Q8_K rows (aq, as, ab) and Q6_K
// weights; scratch holds tc_scratch_bytes(rows, k) (the Q4_K kernel's packed
// operands, of which the bsum tiles are unused here).
ovf_status launch_tc6_project(const void *w, const float *bias, const int8_t *aq, const float *as, const int16_t *ab,
                              float *y, int64_t n, int64_t k, int64_t rows, void *scratch, cudaStream_t st,
                              const float *resid) {
    OVF_CHECK_ARG(tc6_project_supported(n, k, rows), "tensor-core Q6_K projection: unsupported shape");
    OVF_CHECK_ARG(aligned16(w) && scratch && aligned16(scratch), "tensor-core Q6_K projection: alignment");
    const int64_t mtiles = (rows + kT6Toks - 1) / kT6Toks, ntiles = (n + kT6Rows - 1) / kT6Rows, nb = k / 256;
    OVF_CHECK_ARG(mtiles <= 65535, "tensor-core Q6_K projection: too many rows");
    const __half *x16 = nullptr;
    const float *xs = nullptr;
    ovf_status r = launch_tc_pack(aq, as, ab, rows, k, scratch, st, &x16, &xs);
    if (r) return r;
    static PerDeviceOnce attr_once;
    const int dev = current_device();
    if (attr_once.pending(dev)) {
        const cudaError_t e =
            cudaFuncSetAttribute(tc_q6k_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, T6Smem::total);
        if (e != cudaSuccess) return cuda_status(e, "tc6 attribute");
        attr_once.mark(dev);
    }
    CUtensorMap wmap;
    if ((r = encode_bytes_2d(&wmap, w, (uint64_t)nb * 210, (uint64_t)n, (uint64_t)nb * 210, kT6Box, kT6Rows)))
        return r;
    T6Params p{};
    p.x16 = x16;
    p.xs = xs;
    p.bias = bias;
    p.resid = resid;
    p.y = y;
    p.n = (int)n;
    p.K = (int)k;
    p.rows = (int)rows;
    tc_q6k_project_kernel<<<dim3((unsigned)ntiles, (unsigned)mtiles), kT6Threads, T6Smem::total, st>>>(wmap, p);
    return cuda_status(cudaGetLastError(), "tc_q6k_project");
}

}  // namespace ovf
