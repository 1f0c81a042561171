// ovf_moe.cu — mixture-of-experts feed-forward (Mixtral style) on the device:
// the router (Runtime/MoeRouter.cs:40-128 over the F32 input-major gate
// projection, Runtime/SingleTokenProjectionKernel.cs:229-275), the weighted
// combine of the selected experts' SwiGLU outputs in top-k order
// (Runtime/MoeFeedForwardBlock.cs:79-138), and the row gather / scatter of
// the batched form that groups rows per expert (:140-243).  The experts
// themselves run through the quantized GEMV (decode: the expert index is
// read on the device, ovf_gemv.cu) or the weight-stationary batched
// projection (rows).
#include "ovf_internal.cuh"

namespace ovf {

static constexpr int kMoeMaxExperts = 64;
static constexpr int kMoeMaxUsed = 8;

// One CTA per row.  x: the row's normalized FFN input, or (norm_scale
// given) the residual stream that is normalized here as (x * s) * gamma, the
// same operations the GEMV prologue applies, so the router sees the bits the
// experts' activation quantizer sees.  logits[e] = sum_i x_i * R[i][e] in
// ascending i from zero, skipping x_i == 0 (TensorPrimitives.MultiplyAdd per
// input row, SingleTokenProjectionKernel.ProjectChunk); then the reference's
// top-k insertion (ties keep the lower index) and the softmax over the k
// selected (normalize) or over all experts.
__global__ void moe_route_kernel(const float *__restrict__ x, int ld_x, const float *__restrict__ gamma,
                                 const float *__restrict__ norm_scale, const float *__restrict__ R, int D, int E,
                                 int K, int normalize, int32_t *__restrict__ sel, float *__restrict__ wout) {
    extern __shared__ __align__(16) float xs[];  // [D]
    __shared__ float lg[kMoeMaxExperts];
    pdl_wait();
    const int row = blockIdx.x, tid = threadIdx.x;
    const float *xr = x + (size_t)row * ld_x;
    const float s = norm_scale ? *norm_scale : 1.0f;
    for (int i = tid; i < D; i += blockDim.x) {
        float v = xr[i];
        if (norm_scale) v = gamma ? fmul(fmul(v, s), gamma[i]) : fmul(v, s);
        xs[i] = v;
    }
    __syncthreads();
    if (tid < E) {
        float y = 0.0f;
        int i = 0;
        for (; i + 8 <= D; i += 8) {
            float r[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) r[j] = R[(size_t)(i + j) * E + tid];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float xv = xs[i + j];
                if (xv != 0.0f) y = fadd(y, fmul(r[j], xv));
            }
        }
        for (; i < D; ++i) {
            const float xv = xs[i];
            if (xv != 0.0f) y = fadd(y, fmul(R[(size_t)i * E + tid], xv));
        }
        lg[tid] = y;
    }
    __syncthreads();
    if (tid == 0) {
        const int k = K < E ? K : E;
        int idx[kMoeMaxUsed];
        float wv[kMoeMaxUsed];
        for (int i = 0; i < k; ++i) {
            idx[i] = -1;
            wv[i] = -INFINITY;
        }
        int filled = 0;
        for (int e = 0; e < E; ++e) {
            const float l = lg[e];
            if (filled == k && l <= wv[k - 1]) continue;
            int pos = filled < k ? filled : k - 1;
            while (pos > 0 && wv[pos - 1] < l) {
                wv[pos] = wv[pos - 1];
                idx[pos] = idx[pos - 1];
                --pos;
            }
            wv[pos] = l;
            idx[pos] = e;
            if (filled < k) ++filled;
        }
        const float mx = wv[0];
        if (normalize) {
            float sum = 0.0f;
            for (int i = 0; i < k; ++i) {
                const float w = exp_libm(fsub(wv[i], mx));
                wv[i] = w;
                sum = fadd(sum, w);
            }
            const float inv = sum > 0.0f ? fdiv(1.0f, sum) : 0.0f;
            for (int i = 0; i < k; ++i) wv[i] = fmul(wv[i], inv);
        } else {
            float total = 0.0f;
            for (int e = 0; e < E; ++e) total = fadd(total, exp_libm(fsub(lg[e], mx)));
            const float inv = total > 0.0f ? fdiv(1.0f, total) : 0.0f;
            for (int i = 0; i < k; ++i) wv[i] = fmul(exp_libm(fsub(wv[i], mx)), inv);
        }
        for (int i = 0; i < k; ++i) {
            sel[(size_t)row * K + i] = idx[i];
            wout[(size_t)row * K + i] = wv[i];
        }
    }
    pdl_launch_dependents();
}

ovf_status launch_moe_route(const float *x, int ld_x, const float *gamma, const float *norm_scale, const float *R,
                            int rows, int D, int E, int K, int normalize, int32_t *sel, float *w, cudaStream_t st,
                            bool pdl) {
    OVF_CHECK_ARG(E >= 1 && E <= kMoeMaxExperts && K >= 1 && K <= kMoeMaxUsed && K <= E,
                  "moe: %d experts, %d used (at most %d / %d)", E, K, kMoeMaxExperts, kMoeMaxUsed);
    if (rows == 0) return OVF_OK;
    const size_t smem = (size_t)D * 4;
    OVF_CHECK_ARG(smem <= 48 * 1024, "moe: d_model %d too large for the router", D);
    cudaError_t e = launch_pdl(moe_route_kernel, dim3(rows), dim3(256), smem, st, pdl, x, ld_x, gamma, norm_scale, R,
                               D, E, K, normalize, sel, w);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "moe_route");
}

// Decode combine (MoeFeedForwardBlock.Decode :121-137 then the residual,
// CachedTransformerBlock): hidden = after + (((0 + w0*y0) + w1*y1) + ...),
// experts in top-k order; then the next RMSNorm's sequential sum of squares
// of hidden, left as a scale in norm_out (one CTA).
__global__ void moe_combine_kernel(const float *__restrict__ after, const float *__restrict__ y, const float *__restrict__ w,
                                   int K, int D, float *__restrict__ hidden, float *norm_out, float eps) {
    pdl_wait();
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float f = 0.0f;
        for (int j = 0; j < K; ++j) f = fadd(f, fmul(w[j], y[(size_t)j * D + i]));
        hidden[i] = fadd(after[i], f);
    }
    __syncthreads();
    __shared__ __align__(16) float stage[2048];
    const float ss = cta_seq_sumsq(hidden, D, 0.0f, stage);
    if (threadIdx.x == 0 && norm_out) *norm_out = rms_scale(ss, D, eps);
    pdl_launch_dependents();
}

ovf_status launch_moe_combine(const float *after, const float *y, const float *w, int K, int D, float *hidden,
                              float *norm_out, float eps, cudaStream_t st, bool pdl) {
    cudaError_t e = launch_pdl(moe_combine_kernel, dim3(1), dim3(1024), 0, st, pdl, after, y, w, K, D, hidden, norm_out,
                               eps);
    return e == cudaSuccess ? OVF_OK : cuda_status(e, "moe_combine");
}

// Rows form of the combine: out[m] = a[m] + sum_j w[m][j] * slot[m][j] in
// top-k order (DecodeBatched step 3, :229-242, then the residual).
__global__ void moe_combine_rows_kernel(const float *__restrict__ a, const float *__restrict__ slot,
                                        const float *__restrict__ w, int K, int D, float *__restrict__ out) {
    const int m = blockIdx.x;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float f = 0.0f;
        for (int j = 0; j < K; ++j) f = fadd(f, fmul(w[(size_t)m * K + j], slot[((size_t)m * K + j) * D + i]));
        out[(size_t)m * D + i] = fadd(a[(size_t)m * D + i], f);
    }
}

ovf_status launch_moe_combine_rows(const float *a, const float *slot, const float *w, int K, int rows, int D, float *out,
                                   cudaStream_t st) {
    if (rows == 0) return OVF_OK;
    moe_combine_rows_kernel<<<rows, 256, 0, st>>>(a, slot, w, K, D, out);
    return cuda_status(cudaGetLastError(), "moe_combine_rows");
}

// dst[i] = src[rows[i]] (width floats per row).
__global__ void gather_rows_kernel(const float *__restrict__ src, const int32_t *__restrict__ rows, int width,
                                   float *__restrict__ dst) {
    const int i = blockIdx.x;
    const float *s = src + (size_t)rows[i] * width;
    for (int c = threadIdx.x; c < width; c += blockDim.x) dst[(size_t)i * width + c] = s[c];
}

// dst[(rows[i] * K + slots[i])] = src[i] (width floats per row).
__global__ void scatter_slots_kernel(const float *__restrict__ src, const int32_t *__restrict__ rows,
                                     const int32_t *__restrict__ slots, int K, int width, float *__restrict__ dst) {
    const int i = blockIdx.x;
    float *d = dst + ((size_t)rows[i] * K + slots[i]) * width;
    for (int c = threadIdx.x; c < width; c += blockDim.x) d[c] = src[(size_t)i * width + c];
}

ovf_status launch_gather_rows(const float *src, const int32_t *rows, int n, int width, float *dst, cudaStream_t st) {
    if (n == 0) return OVF_OK;
    gather_rows_kernel<<<n, 256, 0, st>>>(src, rows, width, dst);
    return cuda_status(cudaGetLastError(), "gather_rows");
}

ovf_status launch_scatter_slots(const float *src, const int32_t *rows, const int32_t *slots, int n, int K, int width,
                                float *dst, cudaStream_t st) {
    if (n == 0) return OVF_OK;
    scatter_slots_kernel<<<n, 256, 0, st>>>(src, rows, slots, K, width, dst);
    return cuda_status(cudaGetLastError(), "scatter_slots");
}

}  // namespace ovf
