/*
 * ovf_oracle.c — CPU restatement of Overfit's quantized-projection decode path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker + timed CPU baseline); see
 * ovf_oracle.h for the contract.  Reference paths are relative to
 * Sources/Main/LanguageModels/ of DevOnBike/Overfit.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off, no fast-math).
 */
#include "ovf_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* fp16 helpers (BitConverter.UInt16BitsToHalf / (Half)x: IEEE RNE)     */
/* ------------------------------------------------------------------ */
static inline float h2f(const uint8_t *p) {
    uint16_t u = (uint16_t)(p[0] | (p[1] << 8));
    _Float16 h;
    memcpy(&h, &u, 2);
    return (float)h;
}
static inline void f2h(float f, uint8_t *p) {
    _Float16 h = (_Float16)f;
    uint16_t u;
    memcpy(&u, &h, 2);
    p[0] = (uint8_t)(u & 0xFF);
    p[1] = (uint8_t)(u >> 8);
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------ */
/* Codecs                                                              */
/* ------------------------------------------------------------------ */

/* Loading/GgmlDequant.cs:49-77 (UnpackQ4_KScalesMins). */
void orc_unpack_q4k_scales_mins(const uint8_t *q, uint8_t *sc, uint8_t *m) {
    for (int j = 0; j < 4; j++) {
        sc[j] = (uint8_t)(q[j] & 0x3F);
        m[j] = (uint8_t)(q[j + 4] & 0x3F);
    }
    for (int j = 4; j < 8; j++) {
        sc[j] = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
        m[j] = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* Loading/GgmlDequant.cs:95-141 (DecodeQ4_KBlock). */
void orc_decode_q4k_block(const uint8_t *b, float *dst) {
    float d = h2f(b), dmin = h2f(b + 2);
    uint8_t sc[8], m[8];
    orc_unpack_q4k_scales_mins(b + 4, sc, m);
    const uint8_t *qs = b + 16;
    for (int p = 0; p < 4; p++) {
        float s1 = d * (float)sc[2 * p], m1 = dmin * (float)m[2 * p];
        float s2 = d * (float)sc[2 * p + 1], m2 = dmin * (float)m[2 * p + 1];
        for (int i = 0; i < 32; i++) dst[64 * p + i] = s1 * (float)(qs[32 * p + i] & 0x0F) - m1;
        for (int i = 0; i < 32; i++) dst[64 * p + 32 + i] = s2 * (float)(qs[32 * p + i] >> 4) - m2;
    }
}

/* Loading/GgmlDequant.cs:159-209 (DecodeQ6_KBlock).  C# evaluates
 * d * s1 * (q1 - 32) left to right: (d*s1)*(q1-32). */
void orc_decode_q6k_block(const uint8_t *b, float *dst) {
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    float d = h2f(b + 208);
    for (int h = 0; h < 2; h++) {
        for (int l = 0; l < 32; l++) {
            uint8_t qhb = qh[32 * h + l];
            int is = l / 16;
            int q1 = (ql[64 * h + l] & 0x0F) | (((qhb >> 0) & 3) << 4);
            int q2 = (ql[64 * h + l + 32] & 0x0F) | (((qhb >> 2) & 3) << 4);
            int q3 = (ql[64 * h + l] >> 4) | (((qhb >> 4) & 3) << 4);
            int q4 = (ql[64 * h + l + 32] >> 4) | (((qhb >> 6) & 3) << 4);
            dst[128 * h + l] = d * (float)sc[8 * h + is + 0] * (float)(q1 - 32);
            dst[128 * h + l + 32] = d * (float)sc[8 * h + is + 2] * (float)(q2 - 32);
            dst[128 * h + l + 64] = d * (float)sc[8 * h + is + 4] * (float)(q3 - 32);
            dst[128 * h + l + 96] = d * (float)sc[8 * h + is + 6] * (float)(q4 - 32);
        }
    }
}

/* Loading/GgmlQuant.cs:164-172 (PackScalesMins). */
static void pack_scales_mins(const uint8_t *sc, const uint8_t *m, uint8_t *p) {
    for (int j = 0; j < 4; j++) {
        p[j] = (uint8_t)((sc[j] & 0x3F) | ((sc[j + 4] >> 4) << 6));
        p[j + 4] = (uint8_t)((m[j] & 0x3F) | ((m[j + 4] >> 4) << 6));
        p[j + 8] = (uint8_t)((sc[j + 4] & 0x0F) | ((m[j + 4] & 0x0F) << 4));
    }
}

/* Loading/GgmlQuant.cs:31-135 (EncodeQ4_KBlock): plain per-32 min/max,
 * 6-bit scales/mins under fp16 d/dmin; nibbles re-quantized with the fp32
 * d/dmin (before fp16 storage). */
void orc_encode_q4k_block(const float *src, uint8_t *blk) {
    float subScale[8], subMin[8];
    for (int j = 0; j < 8; j++) {
        float lo = INFINITY, hi = -INFINITY;
        for (int e = 0; e < 32; e++) {
            float v = src[j * 32 + e];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (lo > 0.0f) lo = 0.0f;
        subScale[j] = (hi - lo) / 15.0f;
        subMin[j] = -lo;
    }
    float maxScale = 0.0f, maxMin = 0.0f;
    for (int j = 0; j < 8; j++) {
        if (subScale[j] > maxScale) maxScale = subScale[j];
        if (subMin[j] > maxMin) maxMin = subMin[j];
    }
    float invScale = maxScale > 0.0f ? 63.0f / maxScale : 0.0f;
    float invMin = maxMin > 0.0f ? 63.0f / maxMin : 0.0f;
    uint8_t sc[8], m[8];
    for (int j = 0; j < 8; j++) {
        int a = (int)rintf(invScale * subScale[j]);
        int b = (int)rintf(invMin * subMin[j]);
        sc[j] = (uint8_t)(a < 63 ? a : 63);
        m[j] = (uint8_t)(b < 63 ? b : 63);
    }
    float d = maxScale / 63.0f, dmin = maxMin / 63.0f;
    f2h(d, blk);
    f2h(dmin, blk + 2);
    pack_scales_mins(sc, m, blk + 4);
    uint8_t q[256];
    for (int j = 0; j < 8; j++) {
        float es = d * (float)sc[j];
        float em = dmin * (float)m[j];
        for (int e = 0; e < 32; e++) {
            int i = j * 32 + e;
            int l = es > 0.0f ? (int)rintf((src[i] + em) / es) : 0;
            q[i] = (uint8_t)(l < 0 ? 0 : (l > 15 ? 15 : l));
        }
    }
    uint8_t *qs = blk + 16;
    for (int p = 0; p < 4; p++)
        for (int e = 0; e < 32; e++)
            qs[32 * p + e] = (uint8_t)(q[64 * p + e] | (q[64 * p + 32 + e] << 4));
}

/* Loading/GgmlQuant.cs:141-161 (QuantizeQ4_K): output-major rows. */
void orc_quantize_q4k(const float *w, int64_t rows, int64_t k, uint8_t *out) {
    int64_t spr = k / ORC_QK_K;
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < rows; o++)
        for (int64_t sb = 0; sb < spr; sb++)
            orc_encode_q4k_block(w + o * k + sb * ORC_QK_K, out + (o * spr + sb) * ORC_Q4K_BYTES);
}

/* Q6_K encoder.  The reference has none (it only decodes Q6_K,
 * GgmlDequant.cs:159-209); this symmetric absmax scheme writes exactly the
 * layout that decoder reads: 16 signed int8 sub-scales under one fp16 d,
 * 6-bit quants biased by 32.  Same convention as the Q4_K encoder: the
 * quants are computed with the fp32 d before its fp16 storage. */
void orc_encode_q6k_block(const float *src, uint8_t *blk) {
    float sf[16];
    float maxsf = 0.0f;
    for (int s = 0; s < 16; s++) {
        float amax = 0.0f;
        for (int e = 0; e < 16; e++) {
            float a = fabsf(src[s * 16 + e]);
            if (a > amax) amax = a;
        }
        sf[s] = amax / 31.0f;
        if (sf[s] > maxsf) maxsf = sf[s];
    }
    float d = maxsf / 127.0f;
    float inv = maxsf > 0.0f ? 127.0f / maxsf : 0.0f;
    int8_t sc[16];
    for (int s = 0; s < 16; s++) {
        int a = (int)rintf(inv * sf[s]);
        sc[s] = (int8_t)(a > 127 ? 127 : a);
    }
    uint8_t u[256];
    for (int s = 0; s < 16; s++) {
        float es = d * (float)sc[s];
        for (int e = 0; e < 16; e++) {
            int i = s * 16 + e;
            int q = es > 0.0f ? (int)rintf(src[i] / es) : 0;
            q = q < -32 ? -32 : (q > 31 ? 31 : q);
            u[i] = (uint8_t)(q + 32);
        }
    }
    uint8_t *ql = blk, *qh = blk + 128;
    for (int h = 0; h < 2; h++) {
        for (int l = 0; l < 32; l++) {
            int u1 = u[128 * h + l], u2 = u[128 * h + l + 32];
            int u3 = u[128 * h + l + 64], u4 = u[128 * h + l + 96];
            ql[64 * h + l] = (uint8_t)((u1 & 15) | ((u3 & 15) << 4));
            ql[64 * h + l + 32] = (uint8_t)((u2 & 15) | ((u4 & 15) << 4));
            qh[32 * h + l] = (uint8_t)((u1 >> 4) | ((u2 >> 4) << 2) | ((u3 >> 4) << 4) | ((u4 >> 4) << 6));
        }
    }
    memcpy(blk + 192, sc, 16);
    f2h(d, blk + 208);
}

void orc_quantize_q6k(const float *w, int64_t rows, int64_t k, uint8_t *out) {
    int64_t spr = k / ORC_QK_K;
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < rows; o++)
        for (int64_t sb = 0; sb < spr; sb++)
            orc_encode_q6k_block(w + o * k + sb * ORC_QK_K, out + (o * spr + sb) * ORC_Q6K_BYTES);
}

/* Q8_0 GGUF encoder (fp16 scale + 32 int8).  The reference reads Q8_0 only
 * (GgufReader.cs:198-266); the quants follow its own Q8_0 scheme
 * (Runtime/Q8DotKernel.cs:42-91: scale = absmax/127, q = round(x * 1/scale)),
 * with the scale then stored as fp16. */
void orc_quantize_q8_0_gguf(const float *w, int64_t n, uint8_t *out) {
    int64_t nb = n / 32;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; b++) {
        const float *x = w + b * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(x[i]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float id = d > 0.0f ? 1.0f / d : 0.0f;
        uint8_t *o = out + b * ORC_Q8_0_BYTES;
        f2h(d, o);
        for (int i = 0; i < 32; i++) {
            float r = rintf(x[i] * id);
            r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
            o[2 + i] = (uint8_t)(int8_t)r;
        }
    }
}

/* Loading/GgufReader.cs:198-266 (LoadTensorQ8_0Raw): fp16 scale widened to
 * fp32, quants copied — the de-interleaved Q8Weight form. */
void orc_q8_0_deinterleave(const uint8_t *g, int64_t n, int8_t *quants, float *scales) {
    int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; b++) {
        scales[b] = h2f(g + b * ORC_Q8_0_BYTES);
        memcpy(quants + b * 32, g + b * ORC_Q8_0_BYTES + 2, 32);
    }
}

/* Row decode: Runtime/Q4KWeight.cs:122-140 (DecodeRow), the Q6_K analogue,
 * Q8_0 de-interleaved rows (scale * q, Runtime/Q8Weight.cs:90-105) and F32. */
void orc_dequant_rows(int type, const void *data, const float *q8s,
                      int64_t row0, int64_t nrows, int64_t k, float *dst) {
    for (int64_t r = 0; r < nrows; r++) {
        int64_t row = row0 + r;
        float *o = dst + r * k;
        if (type == ORC_Q4_K) {
            int64_t spr = k / ORC_QK_K;
            const uint8_t *b = (const uint8_t *)data + row * spr * ORC_Q4K_BYTES;
            for (int64_t sb = 0; sb < spr; sb++) orc_decode_q4k_block(b + sb * ORC_Q4K_BYTES, o + sb * ORC_QK_K);
        } else if (type == ORC_Q6_K) {
            int64_t spr = k / ORC_QK_K;
            const uint8_t *b = (const uint8_t *)data + row * spr * ORC_Q6K_BYTES;
            for (int64_t sb = 0; sb < spr; sb++) orc_decode_q6k_block(b + sb * ORC_Q6K_BYTES, o + sb * ORC_QK_K);
        } else if (type == ORC_Q8_0) {
            const int8_t *q = (const int8_t *)data + row * k;
            const float *s = q8s + row * (k / 32);
            for (int64_t i = 0; i < k; i++) o[i] = s[i / 32] * (float)q[i];
        } else {
            memcpy(o, (const float *)data + row * k, (size_t)k * sizeof(float));
        }
    }
}

/* Loading/GgufLlamaLoader.cs:977-995 + :1298-1336 (LoadOutputHeads ->
 * SplitOutput -> Q8Weight.QuantizeRows, Runtime/Q8Weight.cs:115-158): a
 * non-Q8_0 attn_output is decoded to fp32 and re-quantized to Q8_0 with fp32
 * scales.  Head slices of a row are whole 32-blocks, so quantizing each full
 * row in 32-blocks gives the same bytes as the per-head gather. */
void orc_quantize_q8_0(const float *x, int64_t k, int8_t *q, float *scales);
void orc_requant_q8_0(int type, const void *data, int64_t rows, int64_t k, int8_t *q, float *scales) {
#pragma omp parallel
    {
        float *row = (float *)malloc((size_t)k * sizeof(float));
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            orc_dequant_rows(type, data, NULL, r, 1, k, row);
            orc_quantize_q8_0(row, k, q + r * k, scales + r * (k / 32));
        }
        free(row);
    }
}

/* ------------------------------------------------------------------ */
/* Activation quantizers                                               */
/* ------------------------------------------------------------------ */

/* Runtime/Q4KDotKernel.cs:71-136 (QuantizeActivationQ8K; the AVX2 variant
 * :148-209 is stated bit-identical). */
void orc_quantize_q8k(const float *x, int64_t k, int8_t *q, float *scales, int16_t *bsums) {
    int64_t blocks = k / ORC_QK_K;
    for (int64_t b = 0; b < blocks; b++) {
        const float *blk = x + b * ORC_QK_K;
        float absMax = 0.0f;
        for (int i = 0; i < ORC_QK_K; i++) {
            float a = fabsf(blk[i]);
            if (a > absMax) absMax = a;
        }
        float scale = absMax / 127.0f;
        scales[b] = scale;
        float inverse = scale > 0.0f ? 1.0f / scale : 0.0f;
        for (int g = 0; g < 16; g++) {
            int sum = 0;
            for (int kk = 0; kk < 16; kk++) {
                int idx = g * 16 + kk;
                float r = rintf(blk[idx] * inverse);
                r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
                int qi = (int)r;
                q[b * ORC_QK_K + idx] = (int8_t)qi;
                sum += qi;
            }
            bsums[b * 16 + g] = (int16_t)sum;
        }
    }
}

/* Runtime/Q8DotKernel.cs:42-91 (Quantize): per-32 fp32 scale absmax/127. */
void orc_quantize_q8_0(const float *x, int64_t k, int8_t *q, float *scales) {
    int64_t blocks = k / 32;
    for (int64_t b = 0; b < blocks; b++) {
        const float *blk = x + b * 32;
        float absMax = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(blk[i]);
            if (a > absMax) absMax = a;
        }
        float scale = absMax / 127.0f;
        scales[b] = scale;
        float inverse = scale > 0.0f ? 1.0f / scale : 0.0f;
        for (int i = 0; i < 32; i++) {
            float r = rintf(blk[i] * inverse);
            r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
            q[b * 32 + i] = (int8_t)(int)r;
        }
    }
}

/* ------------------------------------------------------------------ */
/* Dots                                                                */
/* ------------------------------------------------------------------ */

/* Runtime/Q4KDotKernel.cs:216-256 (Dot) with MainDotScalar :364-383:
 * q8d * (d * mainAcc - dmin * minAcc); integer parts exact. */
float orc_q4k_dot(const uint8_t *blk, const int8_t *q8, float q8scale, const int16_t *bsums) {
    float d = h2f(blk), dmin = h2f(blk + 2);
    uint8_t sc[8], m[8];
    orc_unpack_q4k_scales_mins(blk + 4, sc, m);
    const uint8_t *qs = blk + 16;
    int32_t mainAcc = 0;
    for (int s = 0; s < 8; s++) {
        int qsBase = 32 * (s >> 1);
        int high = s & 1;
        int32_t dot = 0;
        for (int e = 0; e < 32; e++) {
            int packed = qs[qsBase + e];
            int nib = high ? (packed >> 4) : (packed & 0x0F);
            dot += nib * q8[32 * s + e];
        }
        mainAcc += (int32_t)sc[s] * dot;
    }
    int32_t minAcc = 0;
    for (int s = 0; s < 8; s++) minAcc += (int32_t)m[s] * ((int32_t)bsums[2 * s] + (int32_t)bsums[2 * s + 1]);
    return q8scale * (d * (float)mainAcc - dmin * (float)minAcc);
}

/* Runtime/Q6KDotKernel.cs:77-121 (Dot) with the scalar unsigned dot
 * :186-215: d * q8d * (Σ sc·Σ q6u·q8 − 32·Σ sc·bsum). */
float orc_q6k_dot(const uint8_t *blk, const int8_t *q8, float q8scale, const int16_t *bsums) {
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    float d = h2f(blk + 208);
    int32_t sum = 0;
    for (int h = 0; h < 2; h++) {
        for (int l = 0; l < 32; l++) {
            int qhb = qh[32 * h + l];
            int so = l >> 4;
            int q1 = (ql[64 * h + l] & 0x0F) | (((qhb >> 0) & 3) << 4);
            int q2 = (ql[64 * h + l + 32] & 0x0F) | (((qhb >> 2) & 3) << 4);
            int q3 = (ql[64 * h + l] >> 4) | (((qhb >> 4) & 3) << 4);
            int q4 = (ql[64 * h + l + 32] >> 4) | (((qhb >> 6) & 3) << 4);
            int s1 = sc[8 * h + so], s2 = sc[8 * h + so + 2], s3 = sc[8 * h + so + 4], s4 = sc[8 * h + so + 6];
            sum += s1 * q1 * q8[128 * h + l] + s2 * q2 * q8[128 * h + l + 32] +
                   s3 * q3 * q8[128 * h + l + 64] + s4 * q4 * q8[128 * h + l + 96];
        }
    }
    int32_t bsumTerm = 0;
    for (int s = 0; s < 16; s++) bsumTerm += (int32_t)sc[s] * (int32_t)bsums[s];
    int32_t mainAcc = sum - 32 * bsumTerm;
    return d * q8scale * (float)mainAcc;
}

/* Runtime/Q8DotKernel.cs:99-140 (Dot): Σ_blk (wScale·xScale)·int8dot,
 * sequential fp32 over blocks; the weight is the left operand. */
float orc_q8_0_dot(const int8_t *wq, const float *ws, const int8_t *xq, const float *xs, int64_t len) {
    float result = 0.0f;
    for (int64_t b = 0; b < len / 32; b++) {
        int32_t dot = 0;
        for (int i = 0; i < 32; i++) dot += (int32_t)wq[b * 32 + i] * (int32_t)xq[b * 32 + i];
        result += ws[b] * xs[b] * (float)dot;
    }
    return result;
}

/* ------------------------------------------------------------------ */
/* Projections                                                         */
/* ------------------------------------------------------------------ */

/* Runtime/Q4KDotKernel.cs:445-476 (ProjectPreQuantized) / :528-552
 * (ProjectChunk), and the Q6_K twins Runtime/Q6KDotKernel.cs:274-400:
 * y[o] = bias[o] + Σ_sb Dot(...) with the sum sequential over super-blocks. */
void orc_kq_project_prequantized(int type, const uint8_t *w, int64_t n, int64_t k,
                                 const float *bias, float *y,
                                 const int8_t *q, const float *s, const int16_t *bsums) {
    int64_t spr = k / ORC_QK_K;
    int64_t bb = type == ORC_Q6_K ? ORC_Q6K_BYTES : ORC_Q4K_BYTES;
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < n; o++) {
        const uint8_t *row = w + o * spr * bb;
        float sum = 0.0f;
        for (int64_t sb = 0; sb < spr; sb++) {
            float dv = type == ORC_Q6_K
                           ? orc_q6k_dot(row + sb * bb, q + sb * ORC_QK_K, s[sb], bsums + sb * 16)
                           : orc_q4k_dot(row + sb * bb, q + sb * ORC_QK_K, s[sb], bsums + sb * 16);
            sum += dv;
        }
        y[o] = bias ? bias[o] + sum : sum;
    }
}

/* Runtime/Q4KDotKernel.cs:485-523 (ProjectParallel): quantize once, then
 * the pre-quantized projection. */
void orc_kq_project(int type, const float *x, const uint8_t *w, int64_t n, int64_t k,
                    const float *bias, float *y, int8_t *q, float *s, int16_t *bsums) {
    orc_quantize_q8k(x, k, q, s, bsums);
    orc_kq_project_prequantized(type, w, n, k, bias, y, q, s, bsums);
}

/* Runtime/Q4KDotKernel.cs:663-758 (ProjectBatched) and :819-955
 * (ProjectBatchedWeightStationary), both bit-identical to per-row Project:
 * each row is quantized on its own and contracted exactly like decode.  The
 * batched kernels write biasO + sum with biasO = 0 when there is no bias. */
void orc_kq_project_batched(int type, const float *x, int64_t rows, const uint8_t *w,
                            int64_t n, int64_t k, const float *bias, float *y) {
    int64_t spr = k / ORC_QK_K;
    int64_t bb = type == ORC_Q6_K ? ORC_Q6K_BYTES : ORC_Q4K_BYTES;
    int8_t *q = (int8_t *)malloc((size_t)(rows * k));
    float *s = (float *)malloc((size_t)(rows * spr) * sizeof(float));
    int16_t *bs = (int16_t *)malloc((size_t)(rows * spr * 16) * sizeof(int16_t));
    for (int64_t r = 0; r < rows; r++) orc_quantize_q8k(x + r * k, k, q + r * k, s + r * spr, bs + r * spr * 16);
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < n; o++) {
        const uint8_t *row = w + o * spr * bb;
        float biasO = bias ? bias[o] : 0.0f;
        for (int64_t r = 0; r < rows; r++) {
            float sum = 0.0f;
            for (int64_t sb = 0; sb < spr; sb++) {
                const int8_t *qq = q + r * k + sb * ORC_QK_K;
                float sc = s[r * spr + sb];
                const int16_t *bsum = bs + (r * spr + sb) * 16;
                sum += type == ORC_Q6_K ? orc_q6k_dot(row + sb * bb, qq, sc, bsum)
                                        : orc_q4k_dot(row + sb * bb, qq, sc, bsum);
            }
            y[r * n + o] = biasO + sum;
        }
    }
    free(q);
    free(s);
    free(bs);
}

/* Runtime/Q8DotKernel.cs:252-328 (ProjectParallel / ProjectChunk). */
void orc_q8_0_project(const float *x, const int8_t *wq, const float *ws, int64_t n, int64_t k,
                      const float *bias, float *y, int8_t *xq, float *xs) {
    orc_quantize_q8_0(x, k, xq, xs);
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < n; o++) {
        float dot = orc_q8_0_dot(wq + o * k, ws + o * (k / 32), xq, xs, k);
        y[o] = bias ? bias[o] + dot : dot;
    }
}

/* Runtime/Q8DotKernel.cs:352-445 (ProjectBatched). */
void orc_q8_0_project_batched(const float *x, int64_t rows, const int8_t *wq, const float *ws,
                              int64_t n, int64_t k, const float *bias, float *y) {
    int8_t *xq = (int8_t *)malloc((size_t)(rows * k));
    float *xs = (float *)malloc((size_t)(rows * (k / 32)) * sizeof(float));
    for (int64_t r = 0; r < rows; r++) orc_quantize_q8_0(x + r * k, k, xq + r * k, xs + r * (k / 32));
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < n; o++) {
        float biasO = bias ? bias[o] : 0.0f;
        for (int64_t r = 0; r < rows; r++)
            y[r * n + o] = biasO + orc_q8_0_dot(wq + o * k, ws + o * (k / 32), xq + r * k, xs + r * (k / 32), k);
    }
    free(xq);
    free(xs);
}

/* F32 input-major projection used by the MoE router
 * (Runtime/SingleTokenProjectionKernel.cs:44-160): y[e] = Σ_i x[i]·W[i,e],
 * sequential over i. */
void orc_f32_project_input_major(const float *x, const float *w, int64_t k, int64_t n, float *y) {
    for (int64_t e = 0; e < n; e++) y[e] = 0.0f;
    for (int64_t i = 0; i < k; i++) {
        if (x[i] == 0.0f) continue; /* ProjectChunk skips zero inputs (:255-260) */
        for (int64_t e = 0; e < n; e++) y[e] = y[e] + x[i] * w[i * n + e];
    }
}

/* ------------------------------------------------------------------ */
/* Small ops                                                           */
/* ------------------------------------------------------------------ */

/* Runtime/CachedTransformerBlock.cs:525-552 (RmsNormalize) and the final
 * norm Runtime/CachedGptStack.cs:255-285: sequential fp32 Σx²;
 * s = 1/sqrt(Σx²/D + eps); y = (x·s)·γ. */
void orc_rmsnorm(const float *x, const float *gamma, float *y, int64_t d, float eps) {
    float sumSq = 0.0f;
    for (int64_t i = 0; i < d; i++) sumSq += x[i] * x[i];
    float scale = 1.0f / sqrtf(sumSq / (float)d + eps);
    for (int64_t i = 0; i < d; i++) y[i] = gamma ? x[i] * scale * gamma[i] : x[i] * scale;
}

/* Rope/RopeTable.cs:109-133 (Precompute): freq_i = 1/θ^(2i/hd) (MathF.Pow),
 * angle = pos·freq, tables [pos][hd/2]. */
void orc_rope_table(int max_seq, int hd, float theta, float *cos_t, float *sin_t) {
    int half = hd / 2;
    for (int i = 0; i < half; i++) {
        float freq = 1.0f / powf(theta, 2.0f * (float)i / (float)hd);
        for (int pos = 0; pos < max_seq; pos++) {
            float angle = (float)pos * freq;
            cos_t[(int64_t)pos * half + i] = cosf(angle);
            sin_t[(int64_t)pos * half + i] = sinf(angle);
        }
    }
}

/* Rope/RopeKernel.cs:46-93 (Apply): adjacent pairs (2i,2i+1) for
 * llama/mistral, split-half (i, i+hd/2) for qwen2. */
void orc_rope_apply(float *v, int hd, const float *c, const float *s, int split_half) {
    int half = hd / 2;
    if (split_half) {
        for (int i = 0; i < half; i++) {
            float x0 = v[i], x1 = v[i + half];
            v[i] = x0 * c[i] - x1 * s[i];
            v[i + half] = x0 * s[i] + x1 * c[i];
        }
    } else {
        for (int p = 0; p < half; p++) {
            float x0 = v[2 * p], x1 = v[2 * p + 1];
            v[2 * p] = x0 * c[p] - x1 * s[p];
            v[2 * p + 1] = x0 * s[p] + x1 * c[p];
        }
    }
}

/* e^x as the reference computes it: MathF.Exp, i.e. the host C library's
 * expf (glibc's ARM optimized-routines expf on Linux). */
static float orc_expf(float x) { return expf(x); }

/* MathF.Exp over an array (test helper for the device exp). */
void orc_expf_array(const float *x, float *y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = expf(x[i]);
}

/* Runtime/CachedAttentionKernel.cs:342-390 (Dot, AVX2 branch): two 8-lane
 * accumulators over 16-wide steps, then Vector256.Sum(acc0 + acc1).  The lane
 * fold order of Vector256.Sum is the .NET runtime's; it is restated as
 * ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)) — ULP-level parity unpinned. */
static float attn_dot(const float *l, const float *r, int n) {
    if (n >= 8) {
        float a0[8] = {0}, a1[8] = {0};
        int i = 0;
        for (; i + 16 <= n; i += 16)
            for (int j = 0; j < 8; j++) {
                a0[j] = a0[j] + l[i + j] * r[i + j];
                a1[j] = a1[j] + l[i + 8 + j] * r[i + 8 + j];
            }
        for (; i + 8 <= n; i += 8)
            for (int j = 0; j < 8; j++) a0[j] = a0[j] + l[i + j] * r[i + j];
        float v[8];
        for (int j = 0; j < 8; j++) v[j] = a0[j] + a1[j];
        float sum = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
        for (; i < n; i++) sum += l[i] * r[i];
        return sum;
    }
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += l[i] * r[i];
    return s;
}

/* Runtime/CachedAttentionKernel.cs:36-128 (ComputeSingleHead): scores ·scale,
 * max-subtracted exp, invSum, out += p_t·v_t over ascending t; an empty or
 * non-finite sum yields zeros. */
void orc_attention_single_head(const float *q, const float *keys, const float *values,
                               float *out, float *scratch, int seq_len, int hd, float scale) {
    if (seq_len == 0) {
        for (int d = 0; d < hd; d++) out[d] = 0.0f;
        return;
    }
    float maxScore = -INFINITY;
    for (int t = 0; t < seq_len; t++) {
        float sc = attn_dot(q, keys + (int64_t)t * hd, hd) * scale;
        scratch[t] = sc;
        if (sc > maxScore) maxScore = sc;
    }
    float sumExp = 0.0f;
    for (int t = 0; t < seq_len; t++) {
        float e = orc_expf(scratch[t] - maxScore);
        scratch[t] = e;
        sumExp += e;
    }
    for (int d = 0; d < hd; d++) out[d] = 0.0f;
    if (sumExp <= 0.0f || isnan(sumExp) || isinf(sumExp)) return;
    float invSum = 1.0f / sumExp;
    for (int t = 0; t < seq_len; t++) {
        float p = scratch[t] * invSum;
        const float *v = values + (int64_t)t * hd;
        for (int d = 0; d < hd; d++) out[d] = out[d] + p * v[d];
    }
}

/* Runtime/Q8KvQuant.cs:25-77 (Quantize): one K or V vector -> int8 + scale,
 * scale = maxAbs/127, values round-half-even(x * (127/maxAbs)) clamped to
 * +-127; a zero vector gives scale 0 and zero bytes. */
float orc_q8kv_quantize(const float *src, int n, int8_t *dst) {
    float maxAbs = 0.0f;
    for (int i = 0; i < n; i++) {
        float a = fabsf(src[i]);
        if (a > maxAbs) maxAbs = a;
    }
    if (!(maxAbs > 0.0f)) {
        for (int i = 0; i < n; i++) dst[i] = 0;
        return 0.0f;
    }
    float scale = maxAbs / 127.0f;
    float inv = 127.0f / maxAbs;
    for (int d = 0; d < n; d++) {
        float q = nearbyintf(src[d] * inv);
        if (q > 127.0f) q = 127.0f;
        else if (q < -127.0f) q = -127.0f;
        dst[d] = (int8_t)q;
    }
    return scale;
}

/* Runtime/CachedAttentionKernel.cs:200-235 (DotF32I8): the two-accumulator
 * dot of attn_dot with the int8 key widened to float. */
static float attn_dot_i8(const float *l, const int8_t *r, int n) {
    if (n >= 8) {
        float a0[8] = {0}, a1[8] = {0};
        int i = 0;
        for (; i + 16 <= n; i += 16)
            for (int j = 0; j < 8; j++) {
                a0[j] = a0[j] + l[i + j] * (float)r[i + j];
                a1[j] = a1[j] + l[i + 8 + j] * (float)r[i + 8 + j];
            }
        for (; i + 8 <= n; i += 8)
            for (int j = 0; j < 8; j++) a0[j] = a0[j] + l[i + j] * (float)r[i + j];
        float v[8];
        for (int j = 0; j < 8; j++) v[j] = a0[j] + a1[j];
        float sum = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
        for (; i < n; i++) sum += l[i] * (float)r[i];
        return sum;
    }
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += l[i] * (float)r[i];
    return s;
}

/* Runtime/CachedAttentionKernel.cs:139-200 (ComputeSingleHeadQ8): score =
 * DotF32I8(q, kQ[t]) * keyScale[t] * scale; max-subtracted exp; sumExp in
 * order; out[d] += (p_t * invSum * valueScale[t]) * vQ[t][d] in order. */
void orc_attention_single_head_q8(const float *q, const int8_t *kq, const float *ks, const int8_t *vq,
                                  const float *vs, float *out, float *scratch, int seq_len, int hd, float scale) {
    for (int d = 0; d < hd; d++) out[d] = 0.0f;
    if (seq_len == 0) return;
    float maxScore = -INFINITY;
    for (int t = 0; t < seq_len; t++) {
        float sc = attn_dot_i8(q, kq + (int64_t)t * hd, hd) * ks[t] * scale;
        scratch[t] = sc;
        if (sc > maxScore) maxScore = sc;
    }
    float sumExp = 0.0f;
    for (int t = 0; t < seq_len; t++) {
        float e = orc_expf(scratch[t] - maxScore);
        scratch[t] = e;
        sumExp += e;
    }
    if (sumExp <= 0.0f || isnan(sumExp) || isinf(sumExp)) return;
    float invSum = 1.0f / sumExp;
    for (int t = 0; t < seq_len; t++) {
        float coef = scratch[t] * invSum * vs[t];
        const int8_t *v = vq + (int64_t)t * hd;
        for (int d = 0; d < hd; d++) out[d] = out[d] + coef * (float)v[d];
    }
}

/* Runtime/CachedFeedForwardBlock.cs:464-472 (ApplySiLU): sigmoid then
 * multiply; TensorPrimitives.Sigmoid is 1/(1+e^-x) to a few ULP. */
void orc_silu_inplace(float *v, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        float sg = 1.0f / (1.0f + orc_expf(-v[i]));
        v[i] = v[i] * sg;
    }
}

/* Runtime/MoeRouter.cs:40-128 (SelectTopK): insertion into a descending
 * list (ties keep the lower index), then softmax over the k selected
 * (normalize) or full-softmax probabilities of the selected. */
int orc_moe_select_topk(const float *logits, int n, int top_k, int *idx, float *w, int normalize) {
    int k = top_k < n ? top_k : n;
    for (int i = 0; i < k; i++) {
        idx[i] = -1;
        w[i] = -INFINITY;
    }
    int filled = 0;
    for (int e = 0; e < n; e++) {
        float l = logits[e];
        if (filled == k && l <= w[k - 1]) continue;
        int pos = filled < k ? filled : k - 1;
        while (pos > 0 && w[pos - 1] < l) {
            w[pos] = w[pos - 1];
            idx[pos] = idx[pos - 1];
            pos--;
        }
        w[pos] = l;
        idx[pos] = e;
        if (filled < k) filled++;
    }
    float mx = w[0];
    if (normalize) {
        float sum = 0.0f;
        for (int i = 0; i < k; i++) {
            float x = expf(w[i] - mx);
            w[i] = x;
            sum += x;
        }
        float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        for (int i = 0; i < k; i++) w[i] *= inv;
    } else {
        float total = 0.0f;
        for (int e = 0; e < n; e++) total += expf(logits[e] - mx);
        float inv = total > 0.0f ? 1.0f / total : 0.0f;
        for (int i = 0; i < k; i++) w[i] = expf(w[i] - mx) * inv;
    }
    return k;
}

/* Maths/MathUtils.cs:25-28 / Runtime/TokenSampler.cs:170-181 (greedy):
 * first index of the maximum. */
int orc_argmax(const float *v, int64_t n) {
    int best = 0;
    for (int64_t i = 1; i < n; i++)
        if (v[i] > v[best]) best = (int)i;
    return best;
}

/* ------------------------------------------------------------------ */
/* Deterministic synthetic data                                        */
/* ------------------------------------------------------------------ */
static inline uint64_t splitmix64(uint64_t *x) {
    uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
void orc_fill_normal(float *dst, int64_t n, uint64_t seed, float mean, float stddev) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (n + 1) / 2; i++) {
        uint64_t st = seed * 0x100000001B3ull + (uint64_t)i * 2654435761ull;
        uint64_t a = splitmix64(&st), b = splitmix64(&st);
        double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740993.0);
        double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        dst[2 * i] = (float)(mean + stddev * r * cos(6.283185307179586 * u2));
        if (2 * i + 1 < n) dst[2 * i + 1] = (float)(mean + stddev * r * sin(6.283185307179586 * u2));
    }
}

/* ------------------------------------------------------------------ */
/* Whole-model decode (Runtime/CachedLlamaSession.cs:773-868,          */
/* Runtime/CachedGptStack.cs:175-285,492-536,                          */
/* Runtime/CachedTransformerBlock.cs:160-299,                          */
/* Runtime/CachedMultiHeadAttention.cs:166-298,876-908,                */
/* Runtime/CachedSingleHeadAttention.cs:247-337,394-568,               */
/* Runtime/CachedFeedForwardBlock.cs:261-386,                          */
/* Runtime/MoeFeedForwardBlock.cs:79-138)                              */
/* ------------------------------------------------------------------ */
struct orc_session {
    const orc_model *m;
    int max_ctx, pos;
    int kv_fp16;                  /* test switch: round cached K/V to fp16 like the GPU cache */
    float *kcache, *vcache;       /* F32 [layer][kvh][max_ctx][hd] (KeyValueCache.cs:593-602) */
    int kv_q8;                    /* KvCacheDType.Q8: int8 vectors + one scale each */
    int8_t *kq8, *vq8;            /* [layer][kvh][max_ctx][hd] */
    float *ks8, *vs8;             /* [layer][kvh][max_ctx] */
    float *rope_cos, *rope_sin;   /* [max_ctx][hd/2] */
    float *hidden, *after, *ln, *attn_out, *ffo, *fin;
    float *head_out;              /* [n_heads][d_model] per-head Wo outputs */
    float *gate, *up, *eo, *moe_acc;
    int8_t *q8;                   /* Q8_K / Q8_0 quants scratch (max dim) */
    float *q8s;
    int16_t *q8b;
};

static int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

orc_session *orc_session_create(const orc_model *m, int max_ctx) {
    orc_session *s = (orc_session *)calloc(1, sizeof(orc_session));
    s->m = m;
    s->max_ctx = max_ctx;
    int64_t kv = (int64_t)m->n_layers * m->n_kv_heads * max_ctx * m->head_dim;
    s->kcache = (float *)calloc((size_t)kv, sizeof(float));
    s->vcache = (float *)calloc((size_t)kv, sizeof(float));
    s->rope_cos = (float *)malloc((size_t)max_ctx * (m->head_dim / 2) * sizeof(float));
    s->rope_sin = (float *)malloc((size_t)max_ctx * (m->head_dim / 2) * sizeof(float));
    orc_rope_table(max_ctx, m->head_dim, m->theta, s->rope_cos, s->rope_sin);
    int64_t D = m->d_model;
    int64_t big = max64(max64(D, m->d_ff), (int64_t)m->n_heads * m->head_dim);
    s->hidden = (float *)malloc(D * sizeof(float));
    s->after = (float *)malloc(D * sizeof(float));
    s->ln = (float *)malloc(D * sizeof(float));
    s->attn_out = (float *)malloc(D * sizeof(float));
    s->ffo = (float *)malloc(D * sizeof(float));
    s->fin = (float *)malloc(D * sizeof(float));
    s->head_out = (float *)malloc((size_t)m->n_heads * D * sizeof(float));
    s->gate = (float *)malloc(big * sizeof(float));
    s->up = (float *)malloc(big * sizeof(float));
    s->eo = (float *)malloc(D * sizeof(float));
    s->moe_acc = (float *)malloc(D * sizeof(float));
    s->q8 = (int8_t *)malloc(big);
    s->q8s = (float *)malloc(big / 32 * sizeof(float) + 64);
    s->q8b = (int16_t *)malloc(big / 16 * sizeof(int16_t) + 64);
    return s;
}

void orc_session_destroy(orc_session *s) {
    if (!s) return;
    free(s->kcache); free(s->vcache); free(s->rope_cos); free(s->rope_sin);
    free(s->kq8); free(s->vq8); free(s->ks8); free(s->vs8);
    free(s->hidden); free(s->after); free(s->ln); free(s->attn_out); free(s->ffo); free(s->fin);
    free(s->head_out); free(s->gate); free(s->up); free(s->eo); free(s->moe_acc);
    free(s->q8); free(s->q8s); free(s->q8b);
    free(s);
}
void orc_session_reset(orc_session *s) { s->pos = 0; }

/* Timing support (not part of the reference): positions [0, n) of every
 * layer's F32 cache filled with N(0, 0.5) rows (seeded) and the position set
 * to n, so a decode step can be timed at a long context without running the
 * prompt through the model first. */
int orc_session_fill_context(orc_session *s, int n, uint64_t seed) {
    const orc_model *m = s->m;
    if (n < 0 || n >= s->max_ctx || s->kv_q8) return -1;
    const int hd = m->head_dim;
    for (int l = 0; l < m->n_layers; l++)
        for (int g = 0; g < m->n_kv_heads; g++) {
            const int64_t base = (((int64_t)l * m->n_kv_heads + g) * s->max_ctx) * hd;
            orc_fill_normal(s->kcache + base, (int64_t)n * hd, seed + 2 * ((uint64_t)l * m->n_kv_heads + g), 0.0, 0.5);
            orc_fill_normal(s->vcache + base, (int64_t)n * hd, seed + 2 * ((uint64_t)l * m->n_kv_heads + g) + 1, 0.0, 0.5);
        }
    s->pos = n;
    return 0;
}
void orc_session_set_kv_fp16(orc_session *s, int on) { s->kv_fp16 = on; }
/* CreateSession(kvCacheDType: Q8) (CachedLlamaInferenceEngine.cs:360): set
 * before the first token. */
void orc_session_set_kv_q8(orc_session *s, int on) {
    s->kv_q8 = on;
    if (on && !s->kq8) {
        const orc_model *m = s->m;
        int64_t vec = (int64_t)m->n_layers * m->n_kv_heads * s->max_ctx;
        s->kq8 = (int8_t *)calloc((size_t)(vec * m->head_dim), 1);
        s->vq8 = (int8_t *)calloc((size_t)(vec * m->head_dim), 1);
        s->ks8 = (float *)calloc((size_t)vec, sizeof(float));
        s->vs8 = (float *)calloc((size_t)vec, sizeof(float));
    }
}
int orc_session_position(const orc_session *s) { return s->pos; }

static int is_kq(int t) { return t == ORC_Q4_K || t == ORC_Q6_K; }

/* Projection of rows [r0, r0+nr) of w, dispatched on residency
 * (CachedSingleHeadAttention.ProjectHiddenDispatched :394-440 and
 * CachedFeedForwardBlock.ProjectParallelDispatched :355-386).  For K-quants a
 * valid shared Q8_K form of x is used when given; Q8_0 always quantizes its
 * own input.  Row slices are bit-identical to the reference's per-head
 * weight views because every row is an independent dot. */
static void project_rows(const orc_weight *w, int64_t r0, int64_t nr, const float *x,
                         const float *bias, float *y, const int8_t *sq, const float *ss,
                         const int16_t *sb, int8_t *q, float *qs, int16_t *qb) {
    int64_t k = w->cols;
    if (is_kq(w->type)) {
        int64_t bb = w->type == ORC_Q6_K ? ORC_Q6K_BYTES : ORC_Q4K_BYTES;
        const uint8_t *base = (const uint8_t *)w->data + r0 * (k / ORC_QK_K) * bb;
        if (!sq) {
            orc_quantize_q8k(x, k, q, qs, qb);
            sq = q; ss = qs; sb = qb;
        }
        orc_kq_project_prequantized(w->type, base, nr, k, bias, y, sq, ss, sb);
    } else if (w->type == ORC_Q8_0) {
        orc_q8_0_project(x, (const int8_t *)w->data + r0 * k, w->scales + r0 * (k / 32), nr, k, bias, y, q, qs);
    } else {
        /* F32 output-major rows (test models only) */
        const float *wf = (const float *)w->data + r0 * k;
        for (int64_t o = 0; o < nr; o++) {
            float acc = 0.0f;
            for (int64_t i = 0; i < k; i++) acc += wf[o * k + i] * x[i];
            y[o] = bias ? bias[o] + acc : acc;
        }
    }
}

static void swiglu(orc_session *s, const orc_weight *wg, const orc_weight *wu, const orc_weight *wd,
                   const float *x, float *out) {
    int64_t dff = wg->rows;
    if (wg->type == ORC_Q4_K && wu->type == ORC_Q4_K) {
        /* ProjectGateUpParallel (Q4KDotKernel.cs:563-645): one Q8_K quantize. */
        orc_quantize_q8k(x, wg->cols, s->q8, s->q8s, s->q8b);
        orc_kq_project_prequantized(ORC_Q4_K, (const uint8_t *)wg->data, dff, wg->cols, NULL, s->gate, s->q8, s->q8s, s->q8b);
        orc_kq_project_prequantized(ORC_Q4_K, (const uint8_t *)wu->data, dff, wu->cols, NULL, s->up, s->q8, s->q8s, s->q8b);
    } else {
        project_rows(wg, 0, dff, x, NULL, s->gate, NULL, NULL, NULL, s->q8, s->q8s, s->q8b);
        project_rows(wu, 0, dff, x, NULL, s->up, NULL, NULL, NULL, s->q8, s->q8s, s->q8b);
    }
    orc_silu_inplace(s->gate, dff);
    for (int64_t i = 0; i < dff; i++) s->up[i] = s->gate[i] * s->up[i];
    project_rows(wd, 0, wd->rows, s->up, NULL, out, NULL, NULL, NULL, s->q8, s->q8s, s->q8b);
}

static void attention_block(orc_session *s, const orc_layer *L, int layer, int pos, const float *hidden,
                            float *out) {
    const orc_model *m = s->m;
    int D = m->d_model, H = m->n_heads, KVH = m->n_kv_heads, hd = m->head_dim;
    int group = H / KVH;
    int half = hd / 2;
    const float *cp = s->rope_cos + (int64_t)pos * half, *sp = s->rope_sin + (int64_t)pos * half;
    float scale = 1.0f / sqrtf((float)hd);
    for (int i = 0; i < D; i++) out[i] = L->bo ? L->bo[i] : 0.0f;

    int shared = is_kq(L->wq.type);
    int8_t *hq = NULL; float *hs = NULL; int16_t *hb = NULL;
    int8_t *sq = (int8_t *)malloc((size_t)D);
    float *ss = (float *)malloc((size_t)(D / 32 + 8) * sizeof(float));
    int16_t *sb = (int16_t *)malloc((size_t)(D / 16 + 8) * sizeof(int16_t));
    if (shared) {
        orc_quantize_q8k(hidden, D, sq, ss, sb);
        hq = sq; hs = ss; hb = sb;
    }
    /* K/V once per KV group (CachedSingleHeadAttention.ProjectKvDispatched :247-282). */
    float *kb = (float *)malloc((size_t)hd * sizeof(float));
    float *vb = (float *)malloc((size_t)hd * sizeof(float));
    for (int g = 0; g < KVH; g++) {
        int tk = is_kq(L->wk.type);
        int tv = is_kq(L->wv.type);
        project_rows(&L->wk, (int64_t)g * hd, hd, hidden, L->bk ? L->bk + g * hd : NULL, kb,
                     tk ? hq : NULL, hs, hb, s->q8, s->q8s, s->q8b);
        project_rows(&L->wv, (int64_t)g * hd, hd, hidden, L->bv ? L->bv + g * hd : NULL, vb,
                     tv ? hq : NULL, hs, hb, s->q8, s->q8s, s->q8b);
        orc_rope_apply(kb, hd, cp, sp, m->rope_split_half);
        int64_t off = (((int64_t)layer * KVH + g) * s->max_ctx + pos) * hd;
        if (s->kv_fp16)
            for (int i = 0; i < hd; i++) {
                kb[i] = (float)(_Float16)kb[i];
                vb[i] = (float)(_Float16)vb[i];
            }
        if (s->kv_q8) {
            int64_t vi = ((int64_t)layer * KVH + g) * s->max_ctx + pos;
            s->ks8[vi] = orc_q8kv_quantize(kb, hd, s->kq8 + off);
            s->vs8[vi] = orc_q8kv_quantize(vb, hd, s->vq8 + off);
        } else {
            memcpy(s->kcache + off, kb, (size_t)hd * sizeof(float));
            memcpy(s->vcache + off, vb, (size_t)hd * sizeof(float));
        }
    }
    free(kb);
    free(vb);
    /* Per Q head: Q projection, RoPE, attend, per-head Wo (DecodeHeadQao
     * CachedMultiHeadAttention.cs:876-908), heads in parallel; each head
     * owns its scratch and its band of head_out. */
    int seq = pos + 1;
#pragma omp parallel
    {
        float *qv = (float *)malloc((size_t)hd * sizeof(float));
        float *att = (float *)malloc((size_t)hd * sizeof(float));
        float *scr = (float *)malloc((size_t)seq * sizeof(float));
        int8_t *lq = (int8_t *)malloc((size_t)(D > hd ? D : hd));
        float *ls = (float *)malloc((size_t)(D / 32 + 8) * sizeof(float));
        int16_t *lb = (int16_t *)malloc((size_t)(D / 16 + 8) * sizeof(int16_t));
#pragma omp for schedule(static)
        for (int h = 0; h < H; h++) {
            int g = h / group;
            project_rows(&L->wq, (int64_t)h * hd, hd, hidden, L->bq ? L->bq + h * hd : NULL, qv,
                         shared ? hq : NULL, hs, hb, lq, ls, lb);
            orc_rope_apply(qv, hd, cp, sp, m->rope_split_half);
            int64_t base = (((int64_t)layer * KVH + g) * s->max_ctx) * hd;
            if (s->kv_q8) {
                int64_t vb0 = ((int64_t)layer * KVH + g) * s->max_ctx;
                orc_attention_single_head_q8(qv, s->kq8 + base, s->ks8 + vb0, s->vq8 + base, s->vs8 + vb0, att, scr,
                                             seq, hd, scale);
            } else {
                orc_attention_single_head(qv, s->kcache + base, s->vcache + base, att, scr, seq, hd, scale);
            }
            /* Wo_h: Q8_0 per head [D x hd] (GgufLlamaLoader.cs:977-995,1298-1336):
             * quantize att to Q8_0 and contract row o's slice for head h. */
            float *ho = s->head_out + (int64_t)h * D;
            int64_t K = L->wo.cols;
            orc_quantize_q8_0(att, hd, lq, ls);
            for (int o = 0; o < D; o++)
                ho[o] = orc_q8_0_dot((const int8_t *)L->wo.data + (int64_t)o * K + (int64_t)h * hd,
                                     L->wo.scales + (int64_t)o * (K / 32) + (int64_t)h * (hd / 32), lq, ls, hd);
        }
        free(qv); free(att); free(scr); free(lq); free(ls); free(lb);
    }
    /* Head-ordered reduction (CachedMultiHeadAttention.cs:294-297). */
    for (int h = 0; h < H; h++)
        for (int i = 0; i < D; i++) out[i] += s->head_out[(int64_t)h * D + i];
    free(sq);
    free(ss);
    free(sb);
}

static void run_layer(orc_session *s, int layer, int pos) {
    const orc_model *m = s->m;
    const orc_layer *L = &m->layers[layer];
    int D = m->d_model;
    orc_rmsnorm(s->hidden, L->attn_norm, s->ln, D, m->eps);
    attention_block(s, L, layer, pos, s->ln, s->attn_out);
    for (int i = 0; i < D; i++) s->after[i] = s->hidden[i] + s->attn_out[i];
    orc_rmsnorm(s->after, L->ffn_norm, s->ln, D, m->eps);
    if (m->n_experts > 0 && L->router) {
        float logits[256];
        int idx[64];
        float wts[64];
        orc_f32_project_input_major(s->ln, L->router, D, m->n_experts, logits);
        int k = orc_moe_select_topk(logits, m->n_experts, m->n_experts_used, idx, wts, m->normalize_experts);
        for (int i = 0; i < D; i++) s->ffo[i] = 0.0f;
        for (int i = 0; i < k; i++) {
            int e = idx[i];
            swiglu(s, &L->e_gate[e], &L->e_up[e], &L->e_down[e], s->ln, s->eo);
            for (int d = 0; d < D; d++) s->ffo[d] += wts[i] * s->eo[d];
        }
    } else {
        swiglu(s, &L->w_gate, &L->w_up, &L->w_down, s->ln, s->ffo);
    }
    for (int i = 0; i < D; i++) s->hidden[i] = s->after[i] + s->ffo[i];
}

int orc_session_decode_layers(orc_session *s, int token, int n_run, int with_logits, float *logits) {
    const orc_model *m = s->m;
    if (s->pos >= s->max_ctx || token < 0 || token >= m->vocab) return -1;
    int pos = s->pos++;
    orc_dequant_rows(m->embed.type, m->embed.data, m->embed.scales, token, 1, m->d_model, s->hidden);
    if (n_run > m->n_layers) n_run = m->n_layers;
    for (int l = 0; l < n_run; l++) run_layer(s, l, pos);
    if (with_logits && logits) {
        orc_rmsnorm(s->hidden, m->final_norm, s->fin, m->d_model, m->eps);
        project_rows(&m->lm_head, 0, m->vocab, s->fin, NULL, logits, NULL, NULL, NULL, s->q8, s->q8s, s->q8b);
    }
    return 0;
}

int orc_session_decode(orc_session *s, int token, float *logits) {
    return orc_session_decode_layers(s, token, s->m->n_layers, logits != NULL, logits);
}
