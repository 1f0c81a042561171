// ovf_common.cuh — shared device helpers for the sm_100a kernels:
// status plumbing, mbarrier + bulk-copy (TMA 1-D) wrappers with bounded
// waits, and IEEE-exact float helpers (no FMA contraction) for the parts of
// the path that must reproduce the reference's fp32 arithmetic bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>

#include <atomic>

#include "../../include/ovf.h"

namespace ovf {

// A per-device "already done" flag for one-time per-device set-up
// (cudaFuncSetAttribute applies to the current device only).
struct PerDeviceOnce {
    std::atomic<bool> done[64] = {};
    // True when the set-up still has to run on `dev`.
    bool pending(int dev) const { return dev < 0 || dev >= 64 || !done[dev].load(std::memory_order_acquire); }
    void mark(int dev) {
        if (dev >= 0 && dev < 64) done[dev].store(true, std::memory_order_release);
    }
};

inline int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}


// ------------------------------------------------------------ host status
void set_error(const char *fmt, ...);
ovf_status cuda_status(cudaError_t e, const char *what);

#define OVF_CHECK_ARG(cond, ...)          \
    do {                                  \
        if (!(cond)) {                    \
            ::ovf::set_error(__VA_ARGS__); \
            return OVF_EINVAL;            \
        }                                 \
    } while (0)

#define OVF_CUDA_TRY(expr)                                              \
    do {                                                                \
        cudaError_t _e = (expr);                                        \
        if (_e != cudaSuccess) return ::ovf::cuda_status(_e, #expr);    \
    } while (0)

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device-side error word (per device, per library instance).  Kernels set it
// when a bounded wait gives up; the host reads it with ovf_device_error.
enum : int { DEVERR_NONE = 0, DEVERR_MBAR_TIMEOUT = 1, DEVERR_COUNTER = 2, DEVERR_TP_TIMEOUT = 3 };
// Defined once: the library is a single translation unit (csrc/ovf_lib.cu).
__device__ int g_dev_error = 0;

__device__ __forceinline__ void raise_dev_error(int code) { atomicCAS(&g_dev_error, 0, code); }

// --------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 1-D bulk copy global -> shared (the TMA engine, no tensor map): dst and src
// 16-byte aligned, bytes a non-zero multiple of 16.  Completion is signalled
// on the mbarrier as transaction bytes.  Evict-first L2 policy: weights are
// streamed once per token and must not push activations out of L2.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

// 1-D bulk copy from this CTA's shared memory to a CTA of the cluster
// (addresses from mapa_shared), completion signalled on that CTA's mbarrier.
// 16-byte aligned addresses, bytes a non-zero multiple of 16.
__device__ __forceinline__ void bulk_s2cluster(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst),
                 "r"(smem_u32(src)), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or `ns` nanoseconds pass, instead of spinning on issue slots
// that the CTA's other warps need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Sleeping bounded wait: gives up after 2^20 suspensions of at most 2 us
// (about two seconds), raises the device error word and returns false.
__device__ __forceinline__ bool mbar_wait_sleep_bounded(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 20); ++i)
        if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
    raise_dev_error(DEVERR_MBAR_TIMEOUT);
    return false;
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Polling wait (non-blocking test_wait): gives up after 2^28 polls (well
// over a second), raises the device error word and returns false.
__device__ __forceinline__ bool mbar_poll_bounded(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 28); ++i)
        if (mbar_test_wait(bar, parity)) return true;
    raise_dev_error(DEVERR_MBAR_TIMEOUT);
    return false;
}

// Bounded wait: gives up after ~2^26 polls (each try_wait itself suspends
// for a while), raises the device error word and returns false.  A correct
// program never gets near the limit.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 26); ++i)
        if (mbar_try_wait(bar, parity)) return true;
    raise_dev_error(DEVERR_MBAR_TIMEOUT);
    return false;
}

// Programmatic dependent launch: wait until the preceding grid's memory is
// visible / allow the next grid to start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------ numerics
// Explicitly rounded single ops so nvcc cannot contract a*b+c into an FMA:
// the reference's fp32 tails are separate multiplies and adds.
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float i2f(int v) { return __int2float_rn(v); }

__device__ __forceinline__ float h2f_bits(uint16_t u) { return __half2float(__ushort_as_half(u)); }

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Running fp32 sum of squares over x[0..n) in index order — the
// reference's sequential RMSNorm loop (Runtime/CachedTransformerBlock.cs:
// 532-536), bit for bit — computed by one warp.  The lanes hold 512
// elements at a time in registers (the next 512 are loaded meanwhile, so
// the loads hide behind the chain), square them, and the running sum takes
// them in order through shuffles: about one dependent add per element.
// Every lane returns the same sum.
__device__ __forceinline__ float warp_seq_sumsq(const float *x, int n, float acc) {
    constexpr int V = 16;  // elements per lane per batch
    const int lane = threadIdx.x & 31;
    float cur[V], nxt[V];
#pragma unroll
    for (int j = 0; j < V; ++j) cur[j] = 32 * j + lane < n ? __ldcg(x + 32 * j + lane) : 0.0f;
    for (int b = 0; b < n; b += 32 * V) {
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int i = b + 32 * V + 32 * j + lane;
            nxt[j] = i < n ? __ldcg(x + i) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int m = min(32, n - (b + 32 * j));
            if (m <= 0) break;
            const float sq = fmul(cur[j], cur[j]);
            if (m == 32) {
#pragma unroll
                for (int l = 0; l < 32; ++l) acc = fadd(acc, __shfl_sync(0xFFFFFFFFu, sq, l));
            } else {
                for (int l = 0; l < m; ++l) acc = fadd(acc, __shfl_sync(0xFFFFFFFFu, sq, l));
            }
        }
#pragma unroll
        for (int j = 0; j < V; ++j) cur[j] = nxt[j];
    }
    return acc;
}

// The same running sum formed by a whole CTA: the threads square 1024
// elements at a time into shared memory (`stage`, 2 x 1024 floats, double
// buffered) while thread 0 adds the previous 1024 in order, four per
// shared-memory load — one dependent add per element.  Called by every
// thread of the CTA; every thread returns the sum.
__device__ __forceinline__ float cta_seq_sumsq(const float *x, int n, float acc, float *stage) {
    __shared__ float s_acc;
    const int tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) s_acc = acc;
    for (int i = tid; i < 1024 && i < n; i += nt) stage[i] = fmul(__ldcg(x + i), __ldcg(x + i));
    __syncthreads();
    for (int b = 0, buf = 0; b < n; b += 1024, buf ^= 1) {
        const int m = min(1024, n - b);
        if (tid == 0) {
            const float4 *sv = reinterpret_cast<const float4 *>(stage + buf * 1024);
            float a = s_acc;
            const int m32 = m & ~31;
            // 32 elements in registers ahead of the chain
            float4 cur[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) cur[j] = m32 ? sv[j] : make_float4(0.f, 0.f, 0.f, 0.f);
            for (int i = 0; i < m32; i += 32) {
                float4 nxt[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) nxt[j] = i + 32 < m32 ? sv[(i + 32) / 4 + j] : cur[j];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    a = fadd(a, cur[j].x);
                    a = fadd(a, cur[j].y);
                    a = fadd(a, cur[j].z);
                    a = fadd(a, cur[j].w);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
            }
            for (int i = m32; i < m; ++i) a = fadd(a, stage[buf * 1024 + i]);
            s_acc = a;
        } else {
            float *nx = stage + (buf ^ 1) * 1024;
            for (int i = tid - 1; i < 1024 && b + 1024 + i < n; i += nt - 1) {
                const float v = __ldcg(x + b + 1024 + i);
                nx[i] = fmul(v, v);
            }
        }
        __syncthreads();
    }
    const float r = s_acc;
    __syncthreads();
    return r;
}

// RMSNorm scale from the sum of squares: 1 / sqrt(sumSq / d + eps).
__device__ __forceinline__ float rms_scale(float sumsq, int d, float eps) {
    return fdiv(1.0f, sqrtf(fadd(fdiv(sumsq, (float)d), eps)));
}

// cp.async (Ampere-style asynchronous copies into shared memory).
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// e^x for a float argument with the bits of the host C library's expf, which
// is what the reference's MathF.Exp calls on Linux.  glibc (2.27 onwards)
// and musl use the ARM optimized-routines single-precision exp (Szabolcs
// Nagy, MIT / Apache-2.0 licence: glibc sysdeps/ieee754/flt-32/e_expf.c,
// e_exp2f_data.c): in double precision, x*32/ln2 = k + r with k an integer
// found by the round-to-nearest shift 1.5*2^52, 2^(k/32) built from a
// 32-entry table tab[i] = bits(2^(i/32)) - (i << 47) plus k << 47, and
// 2^(r/32) ~= C0 r^3 + C1 r^2 + C2 r + 1 with the published degree-3
// coefficients; the double result is rounded to float once.  On x86-64 hosts
// with FMA, glibc selects a build of that code compiled with FMA contraction,
// so every a*b+c below is one fused multiply-add; compared over every float
// with |x| < 88 this equals that host expf bit for bit (the unfused build
// differs on two inputs), and the range tails follow the same code's
// special cases (overflow to +inf above 0x1.62e42ep6, zero below
// -0x1.9fe368p6, NaN propagated).
// Read through the L1 data cache: lanes index it divergently, which the
// constant cache would serialize.
__device__ const unsigned long long kExp2Tab32[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

// `tab`: the 32-entry table above, or a copy of it in shared memory (a
// kernel that exponentiates on its critical path copies it at its start: the
// global table's first read costs an L2 round trip).
__device__ __forceinline__ float exp_libm(float x, const unsigned long long *tab) {
    if (!(fabsf(x) < 88.0f)) {
        if (x != x) return x + x;
        if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0, c1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0,
                 c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double xd = (double)x;
    double kd = __fma_rn(inv_ln2_n, xd, shift);
    const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
    kd = __dsub_rn(kd, shift);
    const double r = __fma_rn(inv_ln2_n, xd, -kd);
    unsigned long long t = tab[ki & 31];
    t += ki << 47;
    const double s = __longlong_as_double((long long)t);
    const double z = __fma_rn(c0, r, c1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(c2, r, 1.0);
    y = __fma_rn(z, r2, y);
    y = __dmul_rn(y, s);
    return __double2float_rn(y);
}

__device__ __forceinline__ float exp_libm(float x) { return exp_libm(x, kExp2Tab32); }

// Q8_K / Q8_0 element quantizer: clamp(round_half_even(x * inv), -127, 127).
__device__ __forceinline__ int quant_elem(float x, float inv) {
    float r = rintf(fmul(x, inv));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    return static_cast<int>(r);
}

// Launch helper: launches with the programmatic-stream-serialization
// attribute so consecutive kernels overlap their prologues (PDL).
template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    static const bool no_pdl = [] {
        const char *v = getenv("OVF_NO_PDL");
        return v && v[0] == '1';
    }();
    attr[0].val.programmaticStreamSerializationAllowed = (pdl && !no_pdl) ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Upcoming weights to pull into L2 while a kernel runs: the next
// projection's bytes during a latency-bound phase (attention chains, a
// GEMV's drain and norm tail), so the next launch streams from L2.
struct L2Prefetch {
    const void *ptr[4];
    int64_t bytes[4];
    int n;
};

// CTA `cta` of `ncta` issues its slice of every range (bulk L2 prefetches of
// at most 64 KB, 16-byte granules; no shared memory, no completion wait).
__device__ __forceinline__ void prefetch_l2_slice(const L2Prefetch &pf, int cta, int ncta) {
    for (int r = 0; r < pf.n; ++r) {
        const int64_t per = ((pf.bytes[r] + ncta - 1) / ncta + 15) & ~int64_t(15);
        const int64_t a = per * cta, e = pf.bytes[r] < a + per ? pf.bytes[r] : a + per;
        const char *base = static_cast<const char *>(pf.ptr[r]);
        for (int64_t o = a; o < e; o += 65536) {
            const int64_t left = e - o;
            const uint32_t n = (uint32_t)(left < 65536 ? left : 65536) & ~15u;
            if (!n) break;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + o), "r"(n) : "memory");
        }
    }
}

// Per-launch timeline for OVF_TRACE (debugging): first CTA start, last
// griddepcontrol.wait return and last exit, in %globaltimer nanoseconds;
// start is kept as its complement so that every field is an atomicMax.
struct TraceSlot {
    unsigned long long start_c, waited, end, tiles;
};

__device__ __forceinline__ unsigned long long gtime_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// TR_TILES: a GEMV's tile CTAs (not its norm CTA) are done.
enum : int { TR_START = 0, TR_WAITED = 1, TR_END = 2, TR_TILES = 3 };
__device__ __forceinline__ void trace_mark(TraceSlot *t, int what) {
    if (!t) return;
    const unsigned long long v = gtime_ns();
    if (what == TR_START) atomicMax(&t->start_c, ~v);
    else if (what == TR_WAITED) atomicMax(&t->waited, v);
    else if (what == TR_TILES) atomicMax(&t->tiles, v);
    else atomicMax(&t->end, v);
}

int sm_count(int device);

}  // namespace ovf
