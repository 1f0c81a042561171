// ovf_quant.cu — activation quantizers and weight codecs on the device.
//
// All of these are byte/integer work bounded by HBM: one thread (or one warp)
// per block, coalesced where the block layout allows.  Every routine
// reproduces the reference's fp32 arithmetic with explicitly rounded ops, so
// its output bytes equal the CPU restatement's (tests/test_gpu_codecs.py).
#include "ovf_common.cuh"
#include "ovf_internal.cuh"

namespace ovf {

// ------------------------------------------------------------ activations
// Runtime/Q4KDotKernel.cs:71-136 (QuantizeActivationQ8K).  One warp per
// 256-element block, 8 consecutive elements per lane.
__global__ void quantize_q8k_kernel(const float *__restrict__ x, int64_t nblocks, int8_t *__restrict__ q,
                                    float *__restrict__ scales, int16_t *__restrict__ bsums) {
    // a dependent GEMV may launch at once and stream its weights while the
    // activation is quantized (it reads the activation after its
    // griddepcontrol.wait, i.e. after this grid has completed)
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    const float *xb = x + b * 256 + 8 * lane;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = xb[i];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float scale = fdiv(amax, 127.0f);
    const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
    int sum8 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int qi = quant_elem(v[i], inv);
        q[b * 256 + 8 * lane + i] = (int8_t)qi;
        sum8 += qi;
    }
    const int g16 = sum8 + __shfl_xor_sync(0xFFFFFFFFu, sum8, 1);
    if ((lane & 1) == 0) bsums[b * 16 + (lane >> 1)] = (int16_t)g16;
    if (lane == 0) scales[b] = scale;
}

// Runtime/Q8DotKernel.cs:42-91 (Quantize): one warp per 32-element block.
__global__ void quantize_q8_0_kernel(const float *__restrict__ x, int64_t nblocks, int8_t *__restrict__ q,
                                     float *__restrict__ scales) {
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    const float v = x[b * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float scale = fdiv(amax, 127.0f);
    const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
    q[b * 32 + lane] = (int8_t)quant_elem(v, inv);
    if (lane == 0) scales[b] = scale;
}

// ---------------------------------------------------------------- encoders
__device__ __forceinline__ uint16_t half_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

// fp16 store at a 2-byte aligned address (GGUF block headers are little endian).
__device__ __forceinline__ void store_half(uint8_t *p, float v) { *reinterpret_cast<uint16_t *>(p) = half_bits(v); }

// Loading/GgmlQuant.cs:31-135 (EncodeQ4_KBlock), one thread per super-block.
__global__ void encode_q4k_kernel(const float *__restrict__ w, int64_t nsb_total, uint8_t *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nsb_total) return;
    const float *src = w + i * 256;
    uint8_t *blk = out + i * 144;
    float subScale[8], subMin[8];
    for (int j = 0; j < 8; ++j) {
        float lo = INFINITY, hi = -INFINITY;
        for (int e = 0; e < 32; ++e) {
            const float v = src[j * 32 + e];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (lo > 0.0f) lo = 0.0f;
        subScale[j] = fdiv(fsub(hi, lo), 15.0f);
        subMin[j] = -lo;
    }
    float maxScale = 0.0f, maxMin = 0.0f;
    for (int j = 0; j < 8; ++j) {
        if (subScale[j] > maxScale) maxScale = subScale[j];
        if (subMin[j] > maxMin) maxMin = subMin[j];
    }
    const float invScale = maxScale > 0.0f ? fdiv(63.0f, maxScale) : 0.0f;
    const float invMin = maxMin > 0.0f ? fdiv(63.0f, maxMin) : 0.0f;
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = min(63, (int)rintf(fmul(invScale, subScale[j])));
        m[j] = min(63, (int)rintf(fmul(invMin, subMin[j])));
    }
    const float d = fdiv(maxScale, 63.0f), dmin = fdiv(maxMin, 63.0f);
    *reinterpret_cast<uint32_t *>(blk) = (uint32_t)half_bits(d) | ((uint32_t)half_bits(dmin) << 16);
    // Loading/GgmlQuant.cs:164-172 (PackScalesMins)
    for (int j = 0; j < 4; ++j) {
        blk[4 + j] = (uint8_t)((sc[j] & 0x3F) | ((sc[j + 4] >> 4) << 6));
        blk[8 + j] = (uint8_t)((m[j] & 0x3F) | ((m[j + 4] >> 4) << 6));
        blk[12 + j] = (uint8_t)((sc[j + 4] & 0x0F) | ((m[j + 4] & 0x0F) << 4));
    }
    for (int p = 0; p < 4; ++p) {
        const float es0 = fmul(d, (float)sc[2 * p]), em0 = fmul(dmin, (float)m[2 * p]);
        const float es1 = fmul(d, (float)sc[2 * p + 1]), em1 = fmul(dmin, (float)m[2 * p + 1]);
        for (int e = 0; e < 32; ++e) {
            int l0 = es0 > 0.0f ? (int)rintf(fdiv(fadd(src[64 * p + e], em0), es0)) : 0;
            int l1 = es1 > 0.0f ? (int)rintf(fdiv(fadd(src[64 * p + 32 + e], em1), es1)) : 0;
            l0 = max(0, min(15, l0));
            l1 = max(0, min(15, l1));
            blk[16 + 32 * p + e] = (uint8_t)(l0 | (l1 << 4));
        }
    }
}

// Q6_K encoder for the layout Loading/GgmlDequant.cs:159-209 decodes (the
// reference has no Q6_K encoder): symmetric per-16 absmax, int8 sub-scales
// under an fp16 d, quants computed with the fp32 d.  Same bytes as the CPU
// restatement's orc_encode_q6k_block.
__global__ void encode_q6k_kernel(const float *__restrict__ w, int64_t nsb_total, uint8_t *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nsb_total) return;
    const float *src = w + i * 256;
    uint8_t *blk = out + i * 210;
    float sf[16];
    float maxsf = 0.0f;
    for (int s = 0; s < 16; ++s) {
        float amax = 0.0f;
        for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(src[s * 16 + e]));
        sf[s] = fdiv(amax, 31.0f);
        if (sf[s] > maxsf) maxsf = sf[s];
    }
    const float d = fdiv(maxsf, 127.0f);
    const float inv = maxsf > 0.0f ? fdiv(127.0f, maxsf) : 0.0f;
    int sc[16];
    for (int s = 0; s < 16; ++s) sc[s] = min(127, (int)rintf(fmul(inv, sf[s])));
    for (int h = 0; h < 2; ++h) {
        for (int l = 0; l < 32; ++l) {
            int u[4];
            for (int k = 0; k < 4; ++k) {
                const int e = 128 * h + l + 32 * k;
                const int s = e / 16;
                const float es = fmul(d, (float)sc[s]);
                int q = es > 0.0f ? (int)rintf(fdiv(src[e], es)) : 0;
                q = max(-32, min(31, q));
                u[k] = q + 32;
            }
            blk[64 * h + l] = (uint8_t)((u[0] & 15) | ((u[2] & 15) << 4));
            blk[64 * h + l + 32] = (uint8_t)((u[1] & 15) | ((u[3] & 15) << 4));
            blk[128 + 32 * h + l] = (uint8_t)((u[0] >> 4) | ((u[1] >> 4) << 2) | ((u[2] >> 4) << 4) | ((u[3] >> 4) << 6));
        }
    }
    for (int s = 0; s < 16; ++s) blk[192 + s] = (uint8_t)(int8_t)sc[s];
    store_half(blk + 208, d);
}

// GGUF Q8_0 encoder: fp16 scale + 32 int8 (quants as Runtime/Q8DotKernel.cs:42-91).
__global__ void encode_q8_0_gguf_kernel(const float *__restrict__ w, int64_t nblocks, uint8_t *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    const float v = w[b * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float d = fdiv(amax, 127.0f);
    const float id = d > 0.0f ? fdiv(1.0f, d) : 0.0f;
    uint8_t *o = out + b * 34;
    o[2 + lane] = (uint8_t)(int8_t)quant_elem(v, id);
    if (lane == 0) store_half(o, d);
}

// Loading/GgufReader.cs:198-266 (LoadTensorQ8_0Raw): one warp per block.
__global__ void q8_0_deinterleave_kernel(const uint8_t *__restrict__ g, int64_t nblocks, int8_t *__restrict__ q,
                                         float *__restrict__ s) {
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    const uint8_t *blk = g + b * 34;
    q[b * 32 + lane] = (int8_t)blk[2 + lane];
    if (lane == 0) s[b] = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
}

// ---------------------------------------------------------------- decoders
__global__ void dequant_rows_kernel(int type, const uint8_t *__restrict__ w, const float *__restrict__ q8s,
                                    int64_t row0, int64_t nrows, int64_t k, float *__restrict__ dst) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nrows * k) return;
    const int64_t r = row0 + i / k, c = i % k;
    float v;
    if (type == OVF_TYPE_Q4_K) {
        v = q4k_elem(w + (r * (k / 256) + c / 256) * 144, (int)(c % 256));
    } else if (type == OVF_TYPE_Q6_K) {
        v = q6k_elem(w + (r * (k / 256) + c / 256) * 210, (int)(c % 256));
    } else if (type == OVF_TYPE_Q8_0) {
        v = fmul(q8s[r * (k / 32) + c / 32], (float)reinterpret_cast<const int8_t *>(w)[r * k + c]);
    } else {
        v = reinterpret_cast<const float *>(w)[r * k + c];
    }
    dst[i] = v;
}

// Loading/GgufLlamaLoader.cs:977-995,1298-1336: decode to fp32, then
// Q8Weight.QuantizeRows (Runtime/Q8Weight.cs:115-158 -> Q8DotKernel.Quantize)
// per 32-block.  One warp per block.
__global__ void requant_q8_0_kernel(int type, const uint8_t *__restrict__ w, int64_t rows, int64_t k,
                                    int8_t *__restrict__ q, float *__restrict__ s) {
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= rows * (k / 32)) return;
    const int64_t r = b / (k / 32), c = (b % (k / 32)) * 32 + lane;
    float v;
    if (type == OVF_TYPE_Q4_K) v = q4k_elem(w + (r * (k / 256) + c / 256) * 144, (int)(c % 256));
    else if (type == OVF_TYPE_Q6_K) v = q6k_elem(w + (r * (k / 256) + c / 256) * 210, (int)(c % 256));
    else v = reinterpret_cast<const float *>(w)[r * k + c];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float scale = fdiv(amax, 127.0f);
    const float inv = scale > 0.0f ? fdiv(1.0f, scale) : 0.0f;
    q[r * k + c] = (int8_t)quant_elem(v, inv);
    if (lane == 0) s[b] = scale;
}

// ------------------------------------------------------------- launchers
static inline unsigned blocks_for(int64_t n, int per) { return (unsigned)((n + per - 1) / per); }

ovf_status launch_quantize_q8k(const float *x, int64_t k, int8_t *q, float *s, int16_t *b, cudaStream_t st) {
    const int64_t nb = k / 256;
    if (nb == 0) return OVF_OK;
    quantize_q8k_kernel<<<blocks_for(nb, 8), 256, 0, st>>>(x, nb, q, s, b);
    return cuda_status(cudaGetLastError(), "quantize_q8k");
}

ovf_status launch_quantize_q8_0(const float *x, int64_t k, int8_t *q, float *s, cudaStream_t st) {
    const int64_t nb = k / 32;
    if (nb == 0) return OVF_OK;
    quantize_q8_0_kernel<<<blocks_for(nb, 8), 256, 0, st>>>(x, nb, q, s);
    return cuda_status(cudaGetLastError(), "quantize_q8_0");
}

ovf_status launch_encode(int type, const float *w, int64_t rows, int64_t k, void *out, cudaStream_t st) {
    const int64_t n = rows * k;
    if (n == 0) return OVF_OK;
    if (type == OVF_TYPE_Q4_K) {
        encode_q4k_kernel<<<blocks_for(n / 256, 128), 128, 0, st>>>(w, n / 256, (uint8_t *)out);
    } else if (type == OVF_TYPE_Q6_K) {
        encode_q6k_kernel<<<blocks_for(n / 256, 128), 128, 0, st>>>(w, n / 256, (uint8_t *)out);
    } else {
        encode_q8_0_gguf_kernel<<<blocks_for(n / 32, 8), 256, 0, st>>>(w, n / 32, (uint8_t *)out);
    }
    return cuda_status(cudaGetLastError(), "encode");
}

ovf_status launch_q8_0_deinterleave(const void *g, int64_t n, int8_t *q, float *s, cudaStream_t st) {
    if (n == 0) return OVF_OK;
    q8_0_deinterleave_kernel<<<blocks_for(n / 32, 8), 256, 0, st>>>((const uint8_t *)g, n / 32, q, s);
    return cuda_status(cudaGetLastError(), "q8_0_deinterleave");
}

ovf_status launch_dequant_rows(int type, const void *w, const float *q8s, int64_t row0, int64_t nrows, int64_t k,
                               float *dst, cudaStream_t st) {
    const int64_t n = nrows * k;
    if (n == 0) return OVF_OK;
    dequant_rows_kernel<<<blocks_for(n, 256), 256, 0, st>>>(type, (const uint8_t *)w, q8s, row0, nrows, k, dst);
    return cuda_status(cudaGetLastError(), "dequant_rows");
}

ovf_status launch_requant_q8_0(int type, const void *w, int64_t rows, int64_t k, int8_t *q, float *s,
                               cudaStream_t st) {
    const int64_t nb = rows * (k / 32);
    if (nb == 0) return OVF_OK;
    requant_q8_0_kernel<<<blocks_for(nb, 8), 256, 0, st>>>(type, (const uint8_t *)w, rows, k, q, s);
    return cuda_status(cudaGetLastError(), "requant_q8_0");
}

}  // namespace ovf
