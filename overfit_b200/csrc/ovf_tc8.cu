// ovf_tc8.cu — the prefill projection of Q8_0 weights on the 5th-generation
// tensor cores (tcgen05.mma kind::i8, exact int32 accumulators in TMEM),
// bit-identical to the reference's per-row Q8_0 dot (Runtime/Q8DotKernel.cs:
// 99-140 via ProjectBatched :352-445) and so to batched_project_kernel.
//
// Exactness.  Per weight row n, token m and 32-element block j the reference
// forms the integer dot_j = sum q_w * q_x (|dot| <= 127 * 128 * 32) and the
// term (ws_j * xs_j) * (float)dot_j in fp32, then adds the terms in ascending
// j (or, for Wo, sums each head's group of blocks from zero and adds the
// group sums in order on top of the bias).  One MMA of K = 32 (signed int8 x
// signed int8, s32 accumulator) gives dot_j exactly; every block has its own
// TMEM accumulator, and the epilogue runs the fp32 tail in the reference's
// order with the running sums in registers.
//
// Layout.  A CTA owns 128 weight rows x 64 tokens; K flows in stages of 64
// (two blocks) through a 4-deep ring:
//   warp 0      producer: a 2-D tensor copy of the 128 rows' 64 quant bytes,
//               the pre-packed activation tile and the tokens' block scales;
//   warp 1      TMEM allocation (256 columns: four block slots of 64) and the
//               MMA-issuing thread: one M=128 N=64 K=32 MMA per block;
//   warp 2      converter: moves the row-major quant tile into the UMMA
//               no-swizzle K-major layout (8-row x 16-byte core matrices);
//   warps 3-10  epilogue: warp w reads TMEM lanes 32*(w%4).., 32 tokens.
// Two CTAs per SM.  No cluster, no multicast; every wait is bounded.
#include "ovf_internal.cuh"

namespace ovf {

static constexpr int kT8Rows = 128, kT8Toks = 64, kT8Kc = 64, kT8Stages = 4, kT8Slots = 4;
static constexpr int kT8Threads = 352;                      // 11 warps
static constexpr int kT8Raw = kT8Rows * kT8Kc;              // 8 KB: quants as copied [row][64]
static constexpr int kT8Conv = kT8Rows * kT8Kc;             // 8 KB: [kgroup 0..3][row][16 B]
static constexpr int kT8B = kT8Toks * kT8Kc;                // 4 KB: [kgroup][token][16 B]
static constexpr int kT8Xs = 2 * kT8Toks * 4;               // token scales of the stage's two blocks
static constexpr int kT8Stage = kT8Raw + kT8Conv + kT8B + kT8Xs;
static constexpr int kT8Bars = 512;
static constexpr int kT8Smem = kT8Stages * kT8Stage + kT8Bars + 128;
static_assert(kT8Smem <= 113 * 1024, "two CTAs per SM");
static_assert(kT8Stage % 128 == 0, "stage alignment");

// kind::i8, signed A and B (K-major), s32 accumulator, M = 128, N = 64
static constexpr uint32_t kT8Idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kT8Toks >> 3) << 17) |
                                     ((uint32_t)(kT8Rows >> 4) << 24);

__device__ __forceinline__ void t8_mma(uint32_t tmem, uint64_t adesc, uint64_t bdesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, 0, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(adesc), "l"(bdesc), "r"(kT8Idesc)
        : "memory");
}

// Activation packing: the Q8_0 rows of a batch as int8 operand tiles,
// x8 [token tile][stage][kgroup 0..3][64 tokens][16 B], and the tokens' block
// scales xs [token tile][stage][2][64].  Tokens past `rows` are zero.
__global__ void t8_pack_kernel(const int8_t *__restrict__ aq, const float *__restrict__ as, int rows, int K,
                               int8_t *__restrict__ x8, float *__restrict__ xs) {
    const int mt = blockIdx.y, c = blockIdx.x, nkc = K / kT8Kc;
    const int tid = threadIdx.x;  // 256 threads: (kgroup, token)
    const int kg = tid >> 6, t = tid & 63, m = mt * kT8Toks + t;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (m < rows) v = *reinterpret_cast<const uint4 *>(aq + (size_t)m * K + c * kT8Kc + 16 * kg);
    reinterpret_cast<uint4 *>(x8 + ((size_t)mt * nkc + c) * kT8B)[kg * kT8Toks + t] = v;
    if (tid < 2 * kT8Toks) {
        const int j = tid >> 6;
        xs[((size_t)mt * nkc + c) * (2 * kT8Toks) + tid] = m < rows ? as[(size_t)m * (K / 32) + 2 * c + j] : 0.0f;
    }
}

struct T8Params {
    const int8_t *x8;     // packed activation tiles
    const float *xs;      // packed token scales
    const float *ws;      // weight block scales [n][K/32]
    const float *bias;    // [n] or null
    const float *resid;   // [rows][n] or null
    float *y;             // [rows][n]
    int n, K, rows, group;
};

template <bool GROUPED>
__global__ void __launch_bounds__(kT8Threads, 2)
    tc_q80_project_kernel(const __grid_constant__ CUtensorMap wmap, const T8Params p) {
    extern __shared__ uint8_t t8_raw_smem[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(t8_raw_smem) + 127) & ~uintptr_t(127));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kT8Rows, mt = blockIdx.y, m0 = mt * kT8Toks;
    const int nkc = p.K / kT8Kc, nbk = p.K / 32;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kT8Stages * kT8Stage);
    uint64_t *full = bars, *conv = full + kT8Stages, *empty = conv + kT8Stages;
    uint64_t *acc_full = empty + kT8Stages, *acc_empty = acc_full + kT8Slots, *mma_done = acc_empty + kT8Slots;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    static_assert((3 * kT8Stages + 2 * kT8Slots + 2) * 8 <= kT8Bars, "barrier area");
    if (tid == 0) {
        for (int i = 0; i < kT8Stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&conv[i], 1);
            mbar_init(&empty[i], 8);  // epilogue warps
        }
        for (int i = 0; i < kT8Slots; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 8);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kT8Slots * kT8Toks)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto stage_ptr = [&](int s) { return sm + (size_t)s * kT8Stage; };

    if (warp == 0) {
        // ------------------------------------------------------- producer
        const uint64_t pol = l2_evict_first_policy();
        int issued = 0;
        for (int c = 0; c < nkc; ++c) {
            const int s = c % kT8Stages;
            if (c >= kT8Stages && !tc_wait(&empty[s], ((c / kT8Stages) - 1) & 1)) break;
            if (lane == 0) {
                uint8_t *st = stage_ptr(s);
                mbar_arrive_expect_tx(&full[s], (uint32_t)(kT8Raw + kT8B + kT8Xs));
                tma_load_2d(st, &wmap, c * kT8Kc, n0, &full[s], pol);
                bulk_g2s(st + kT8Raw + kT8Conv, p.x8 + ((size_t)mt * nkc + c) * kT8B, kT8B, &full[s], pol);
                bulk_g2s(st + kT8Raw + kT8Conv + kT8B, p.xs + ((size_t)mt * nkc + c) * (2 * kT8Toks), kT8Xs,
                         &full[s], pol);
            }
            issued = c + 1;
            __syncwarp();
        }
        // drain: the last copy issued into every stage has landed before exit
        for (int s = 0; s < kT8Stages; ++s) {
            int last = -1;
            for (int c = s; c < issued; c += kT8Stages) last = c;
            if (last >= 0) tc_wait(&full[s], (last / kT8Stages) & 1);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            bool ok = true;
            for (int c = 0; c < nkc && ok; ++c) {
                const int s = c % kT8Stages;
                ok = tc_wait(&full[s], (c / kT8Stages) & 1) && tc_wait(&conv[s], (c / kT8Stages) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t abase = smem_u32(stage_ptr(s) + kT8Raw);
                const uint32_t bbase = smem_u32(stage_ptr(s) + kT8Raw + kT8Conv);
                for (int j = 0; j < 2 && ok; ++j) {
                    const int g = 2 * c + j, slot = g % kT8Slots;
                    if (g >= kT8Slots) ok = tc_wait(&acc_empty[slot], ((g / kT8Slots) - 1) & 1);
                    if (!ok) break;
                    tc_fence_after();
                    // block j: core-matrix columns 2j, 2j+1 (K-adjacent 2048 B apart in A,
                    // 1024 B in B; 8-row groups 128 B apart in both)
                    t8_mma(tmem + slot * kT8Toks, umma_desc(abase + 2 * j * 2048, 2048, 128),
                           umma_desc(bbase + 2 * j * 1024, 1024, 128));
                    tc_commit(&acc_full[slot]);
                }
            }
            tc_commit(mma_done);
            tc_wait(mma_done, 0);
        }
        __syncwarp();
    } else if (warp == 2) {
        // ---------------------------------------------------- converter
        for (int c = 0; c < nkc; ++c) {
            const int s = c % kT8Stages;
            if (!tc_wait(&full[s], (c / kT8Stages) & 1)) break;
            const uint8_t *raw = stage_ptr(s);
            uint8_t *cv = stage_ptr(s) + kT8Raw;
#pragma unroll 4
            for (int i = lane; i < kT8Rows * 4; i += 32) {
                const int row = i & (kT8Rows - 1), kg = i >> 7;
                reinterpret_cast<uint4 *>(cv)[kg * kT8Rows + row] =
                    reinterpret_cast<const uint4 *>(raw)[row * 4 + kg];
            }
            fence_proxy_async_smem();
            warp_arrive(&conv[s], lane);
        }
    } else {
        // ------------------------------------------------------ epilogue
        const int lane_base = 32 * (warp & 3);
        const int row = lane_base + lane, n = n0 + row;
        const int t0 = 32 * ((warp - 3) >> 2);
        const bool rvalid = n < p.n;
        const uint32_t lane_addr = tmem + ((uint32_t)lane_base << 16);
        const int G = GROUPED ? p.group : 0;
        const float bo = rvalid && p.bias ? p.bias[n] : 0.0f;
        float acc[32];
        float grp[GROUPED ? 32 : 1];
#pragma unroll
        for (int t = 0; t < 32; ++t) acc[t] = GROUPED ? bo : 0.0f;
        int gp = 0;
        const float *wsr = p.ws + (size_t)(rvalid ? n : 0) * nbk;
        float wsn = rvalid ? __ldg(wsr) : 0.0f;
        bool ok = true;
        for (int c = 0; c < nkc && ok; ++c) {
            const int s = c % kT8Stages;
            // the stage's token scales were written by the copy engine
            if (!tc_wait(&full[s], (c / kT8Stages) & 1)) break;
            const float *xs = reinterpret_cast<const float *>(stage_ptr(s) + kT8Raw + kT8Conv + kT8B);
            for (int j = 0; j < 2; ++j) {
                const int g = 2 * c + j, slot = g % kT8Slots;
                const float wsv = wsn;
                if (g + 1 < nbk) wsn = rvalid ? __ldg(wsr + g + 1) : 0.0f;
                if (!tc_wait(&acc_full[slot], (g / kT8Slots) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const bool close = GROUPED && gp + 1 == G;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t d[16];
                    tmem_ld16_nowait(lane_addr + slot * kT8Toks + t0 + 16 * h, d);
                    tmem_ld_wait();
                    if (h == 1) {
                        tc_fence_before();
                        warp_arrive(&acc_empty[slot], lane);
                    }
                    const float4 *x4 = reinterpret_cast<const float4 *>(xs + j * kT8Toks + t0 + 16 * h);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 xv = x4[q];
                        const float xq[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int i = 4 * q + e, t = 16 * h + i;
                            const float term = fmul(fmul(wsv, xq[e]), __int2float_rn((int)d[i]));
                            if (GROUPED) {
                                grp[t] = gp == 0 ? fadd(0.0f, term) : fadd(grp[t], term);
                                if (close) acc[t] = fadd(acc[t], grp[t]);
                            } else {
                                acc[t] = fadd(acc[t], term);
                            }
                        }
                    }
                }
                if (GROUPED) gp = close ? 0 : gp + 1;
            }
            warp_arrive(&empty[s], lane);
        }
        if (rvalid) {
#pragma unroll
            for (int t = 0; t < 32; ++t) {
                const int m = m0 + t0 + t;
                if (m < p.rows) {
                    float y = GROUPED || !p.bias ? acc[t] : fadd(bo, acc[t]);
                    if (p.resid) y = fadd(p.resid[(size_t)m * p.n + n], y);
                    p.y[(size_t)m * p.n + n] = y;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kT8Slots * kT8Toks)
                     : "memory");
    }
}

bool tc8_project_supported(int64_t n, int64_t k, int64_t rows, int group) {
    return k % kT8Kc == 0 && k >= kT8Kc && n >= 1 && rows >= 1 && n <= 0x7FFFFFFF && group >= 0 &&
           (group == 0 || (k / 32) % group == 0);
}

int64_t tc8_scratch_bytes(int64_t rows, int64_t k) {
    const int64_t mt = (rows + kT8Toks - 1) / kT8Toks;
    return mt * kT8Toks * k + mt * (k / 32) * kT8Toks * 4 + 256;
}

// y [rows x n] (+ bias, + resid) from the Q8_0 activation rows (aq, as) and
// de-interleaved Q8_0 weights (wq [n][k] int8, ws [n][k/32] fp32); scratch
// holds tc8_scratch_bytes(rows, k).  group > 0: head-ordered sums of `group`
// blocks (Wo).
ovf_status launch_tc8_project(const int8_t *wq, const float *ws, const float *bias, const int8_t *aq,
                              const float *as, float *y, int64_t n, int64_t k, int64_t rows, int group,
                              void *scratch, cudaStream_t st, const float *resid) {
    OVF_CHECK_ARG(tc8_project_supported(n, k, rows, group), "tensor-core Q8_0 projection: unsupported shape");
    OVF_CHECK_ARG(aligned16(wq) && aligned16(aq) && scratch && aligned16(scratch),
                  "tensor-core Q8_0 projection: alignment");
    const int64_t mtiles = (rows + kT8Toks - 1) / kT8Toks, ntiles = (n + kT8Rows - 1) / kT8Rows;
    OVF_CHECK_ARG(mtiles <= 65535, "tensor-core Q8_0 projection: too many rows");
    int8_t *x8 = static_cast<int8_t *>(scratch);
    float *xs = reinterpret_cast<float *>(static_cast<uint8_t *>(scratch) + mtiles * kT8Toks * k);
    t8_pack_kernel<<<dim3((unsigned)(k / kT8Kc), (unsigned)mtiles), 256, 0, st>>>(aq, as, (int)rows, (int)k, x8, xs);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "t8_pack");
    static PerDeviceOnce attr_once;
    const int dev = current_device();
    if (attr_once.pending(dev)) {
        e = cudaFuncSetAttribute(tc_q80_project_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kT8Smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(tc_q80_project_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kT8Smem);
        if (e != cudaSuccess) return cuda_status(e, "tc8 attribute");
        attr_once.mark(dev);
    }
    CUtensorMap wmap;
    if (ovf_status r = encode_bytes_2d(&wmap, wq, (uint64_t)k, (uint64_t)n, (uint64_t)k, kT8Kc, kT8Rows)) return r;
    T8Params p{};
    p.x8 = x8;
    p.xs = xs;
    p.ws = ws;
    p.bias = bias;
    p.resid = resid;
    p.y = y;
    p.n = (int)n;
    p.K = (int)k;
    p.rows = (int)rows;
    p.group = group;
    const dim3 grid((unsigned)ntiles, (unsigned)mtiles);
    if (group > 0) tc_q80_project_kernel<true><<<grid, kT8Threads, kT8Smem, st>>>(wmap, p);
    else tc_q80_project_kernel<false><<<grid, kT8Threads, kT8Smem, st>>>(wmap, p);
    return cuda_status(cudaGetLastError(), "tc_q80_project");
}

}  // namespace ovf
