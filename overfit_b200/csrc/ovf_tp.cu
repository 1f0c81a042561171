// ovf_tp.cu — the exchange side of tensor parallelism (one process per GPU,
// peers' buffers mapped with CUDA IPC over NVLink).
//
// The split follows the reference's per-head structure
// (CachedMultiHeadAttention.cs:221-298) and keeps its arithmetic exactly:
//   * Q/K/V rows of a rank's heads, and gate/up rows of its FFN slice, are
//     computed whole on that rank (rows are independent);
//   * Wo: the rank's heads' per-head outputs y_h (the Q8_0 per-head groups,
//     CachedSingleHeadAttention.cs:450-481) are stored by the producing GEMV
//     straight into every rank's exchange buffer; each rank then forms
//     after = hidden + (((bias + y_0) + y_1) + ... + y_{H-1}), the
//     reference's head-ordered sum (:294-297), and the next RMSNorm;
//   * down: the rank's super-block terms of every output row are stored into
//     every rank's buffer, block-major; each rank adds all blocks' terms in
//     ascending order (the reference's sequential fp32 loop) and the residual;
//   * LM head: vocabulary rows split; logits go to every rank's buffer and
//     each rank's first-maximum key is published, the maximum of the keys
//     being TokenSampler.ArgMax over the whole vocabulary.
// So a TP run is bit-identical to one GPU.  The producing GEMV's remote
// stores end with a system-scope fence; the combine kernel (the next launch
// on the stream) then publishes this rank's epoch in every rank's flag
// table with a release store and waits, with a bound, for every rank's.
#include "ovf_internal.cuh"

namespace ovf {

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Thread 0 only: publishes this rank's epoch for the slot on every rank and
// waits for every rank's (about a second at most; then the error word is
// set and the data read afterwards is whatever arrived).
__device__ bool tp_signal_and_wait(const TpExchange &x) {
    const unsigned e = *x.epoch;
    __threadfence_system();
    for (int w = 0; w < x.world; ++w) st_release_sys(x.flags_peer[w] + (size_t)x.slot * x.world + x.rank, e);
    for (int w = 0; w < x.world; ++w) {
        const unsigned *f = x.flags_own + (size_t)x.slot * x.world + w;
        uint32_t it = 0;
        while ((int)(ld_acquire_sys(f) - e) < 0) {
            if (++it > (1u << 22)) {
                raise_dev_error(DEVERR_TP_TIMEOUT);
                return false;
            }
            __nanosleep(128);
        }
    }
    return true;
}

// out[i] = resid[i] + (((init + recv[0][i]) + recv[1][i]) + ... ), init =
// bias[i] or 0, then the RMSNorm scale of out (the reference's sequential
// sum of squares) in norm_out.  One CTA.
__global__ void tp_sum_combine_kernel(const TpExchange x, const float *__restrict__ recv, int n,
                                      const float *__restrict__ bias, const float *__restrict__ resid,
                                      float *__restrict__ out, float *norm_out, int D, float eps) {
    pdl_wait();
    if (threadIdx.x == 0) tp_signal_and_wait(x);
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v = bias ? bias[i] : 0.0f;
        int j = 0;
        for (; j + 8 <= n; j += 8) {
            float t[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) t[q] = __ldcg(recv + (size_t)(j + q) * D + i);
#pragma unroll
            for (int q = 0; q < 8; ++q) v = fadd(v, t[q]);
        }
        for (; j < n; ++j) v = fadd(v, __ldcg(recv + (size_t)j * D + i));
        out[i] = fadd(resid[i], v);
    }
    __syncthreads();
    __shared__ __align__(16) float stage[2048];
    const float ss = cta_seq_sumsq(out, D, 0.0f, stage);
    if (threadIdx.x == 0 && norm_out) *norm_out = rms_scale(ss, D, eps);
    pdl_launch_dependents();
}

ovf_status launch_tp_sum_combine(const TpExchange &x, const float *recv, int n, const float *bias, const float *resid,
                                 float *out, float *norm_out, int D, float eps, cudaStream_t st, bool pdl) {
    cudaError_t e = launch_pdl(tp_sum_combine_kernel, dim3(1), dim3(1024), 0, st, pdl, x, recv, n, bias, resid, out,
                               norm_out, D, eps);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "tp_sum_combine");
}

// Expert parallel combine: every rank's selected experts' outputs y_j
// (written by their owners) in top-k order, hidden = after + (((0 + w_0 y_0)
// + w_1 y_1) + ...), then the next RMSNorm's scale (MoeFeedForwardBlock.Decode
// :121-137 and the residual).  One CTA.
__global__ void tp_moe_combine_kernel(const TpExchange x, const float *__restrict__ recv, const float *__restrict__ w,
                                      int K, const float *__restrict__ resid, float *__restrict__ out, float *norm_out,
                                      int D, float eps) {
    pdl_wait();
    if (threadIdx.x == 0) tp_signal_and_wait(x);
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float f = 0.0f;
        for (int j = 0; j < K; ++j) f = fadd(f, fmul(w[j], __ldcg(recv + (size_t)j * D + i)));
        out[i] = fadd(resid[i], f);
    }
    __syncthreads();
    __shared__ __align__(16) float stage[2048];
    const float ss = cta_seq_sumsq(out, D, 0.0f, stage);
    if (threadIdx.x == 0 && norm_out) *norm_out = rms_scale(ss, D, eps);
    pdl_launch_dependents();
}

ovf_status launch_tp_moe_combine(const TpExchange &x, const float *recv, const float *w, int K, const float *resid,
                                 float *out, float *norm_out, int D, float eps, cudaStream_t st, bool pdl) {
    cudaError_t e = launch_pdl(tp_moe_combine_kernel, dim3(1), dim3(1024), 0, st, pdl, x, recv, w, K, resid, out,
                               norm_out, D, eps);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "tp_moe_combine");
}

// The greedy token from every rank's first-maximum key: the largest key
// (orderable logit, then the lower index) is the whole vocabulary's.
__global__ void tp_lm_finish_kernel(const TpExchange x, const unsigned long long *keys, DevStep *step,
                                    int32_t *tokens_log) {
    pdl_wait();
    if (threadIdx.x == 0) {
        tp_signal_and_wait(x);
        unsigned long long k = 0ull;
        for (int w = 0; w < x.world; ++w) {
            const unsigned long long v = __ldcg(keys + w);
            k = v > k ? v : k;
        }
        const int idx = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        step->token = idx;
        if (tokens_log) tokens_log[step->n_generated] = idx;
        step->n_generated += 1;
    }
    pdl_launch_dependents();
}

ovf_status launch_tp_lm_finish(const TpExchange &x, const unsigned long long *keys, DevStep *step, int32_t *tokens_log,
                               cudaStream_t st, bool pdl) {
    cudaError_t e = launch_pdl(tp_lm_finish_kernel, dim3(1), dim3(32), 0, st, pdl, x, keys, step, tokens_log);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "tp_lm_finish");
}

}  // namespace ovf
