/*
 * Quantized block formats: f16 conversion, own K-quant encoders, bit-exact
 * dequantizers and reference GEMMs.  TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Compile with -ffp-contract=off: the reference's Julia dequantizers do not
 * fuse multiply-add (src/Dequant.jl has no @fastmath/@muladd), so the
 * dequantized values are reproduced bit for bit only without contraction.
 */
#include "oracle.h"
#include <math.h>
#include <string.h>
#include <stdlib.h>

#define QK_K 256

float or_f16_to_f32(uint16_t h) {
    /* exact widening; same result as Float32(reinterpret(Float16, h)) in
       src/Dequant.jl and fp16_to_fp32 in src/kernels/quant_kernels.c:66-86 */
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, f;
    if (e == 0) {
        if (m == 0) f = sign;
        else {
            int sh = 0;
            while (!(m & 0x400)) { m <<= 1; sh++; }
            m &= 0x3ff;
            f = sign | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 0x1f) {
        f = sign | 0x7f800000u | (m << 13);
    } else {
        f = sign | ((e + 127 - 15) << 23) | (m << 13);
    }
    float r; memcpy(&r, &f, 4); return r;
}

uint16_t or_f32_to_f16(float x) {
    uint32_t f; memcpy(&f, &x, 4);
    uint32_t sign = (f >> 16) & 0x8000;
    uint32_t ax = f & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00 | (ax > 0x7f800000u ? 0x200 : 0));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00);          /* overflow -> inf */
    if (ax < 0x38800000u) {                                            /* subnormal half */
        if (ax < 0x33000000u) return (uint16_t)sign;                   /* < 2^-25 -> 0 */
        /* value = m * 2^(e-150); half subnormal unit = 2^-24 -> q = m * 2^(e-126) */
        uint32_t e = ax >> 23, m = (ax & 0x7fffff) | 0x800000;
        int shift = 126 - (int)e;
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = ((ax >> 23) - 127 + 15), m = ax & 0x7fffff;
    uint32_t q = (e << 10) | (m >> 13), rem = m & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

int64_t or_row_bytes(int type, int64_t cols) {
    switch (type) {
    case OR_F32: return cols * 4;
    case OR_F16: return cols * 2;
    case OR_Q8_0: return (cols % 32) ? 0 : cols / 32 * 34;
    case OR_Q4_K: return (cols % QK_K) ? 0 : cols / QK_K * 144;
    case OR_Q5_K: return (cols % QK_K) ? 0 : cols / QK_K * 176;
    case OR_Q6_K: return (cols % QK_K) ? 0 : cols / QK_K * 210;
    }
    return 0;
}

static inline void put16(uint8_t *p, uint16_t v) { p[0] = v & 0xff; p[1] = v >> 8; }
static inline uint16_t get16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline int iclamp(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

/* ------------------------------------------------------------------ */
/* Encoders (own design: per-sub-block min/max affine fit, no search) */
/* ------------------------------------------------------------------ */

/* 6-bit scale/min packing, inverse of src/Dequant.jl:345-362 */
static void pack_scales_k(uint8_t s[12], const int sc[8], const int mn[8]) {
    memset(s, 0, 12);
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)(sc[j] & 63);
        s[j + 4] = (uint8_t)(mn[j] & 63);
    }
    for (int j = 4; j < 8; j++) {
        s[j + 4] = (uint8_t)((sc[j] & 15) | ((mn[j] & 15) << 4));
        s[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
        s[j] |= (uint8_t)((mn[j] >> 4) << 6);
    }
}

static void enc_qk_affine(const float *x, int nlev, uint8_t *hdr /*d,dmin,scales*/, int q[QK_K]) {
    float scale[8], mnv[8];
    float maxs = 0.f, maxm = 0.f;
    for (int j = 0; j < 8; j++) {
        float lo = 0.f, hi = -INFINITY;
        for (int i = 0; i < 32; i++) {
            float v = x[32 * j + i];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (hi < lo) hi = lo;
        scale[j] = (hi - lo) / (float)nlev;
        mnv[j] = -lo;
        if (scale[j] > maxs) maxs = scale[j];
        if (mnv[j] > maxm) maxm = mnv[j];
    }
    uint16_t dh = or_f32_to_f16(maxs / 63.f), mh = or_f32_to_f16(maxm / 63.f);
    float d = or_f16_to_f32(dh), dmin = or_f16_to_f32(mh);
    int sc[8], mn[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = d > 0 ? iclamp((int)lrintf(scale[j] / d), 0, 63) : 0;
        mn[j] = dmin > 0 ? iclamp((int)lrintf(mnv[j] / dmin), 0, 63) : 0;
        float ds = d * (float)sc[j], dm = dmin * (float)mn[j];
        for (int i = 0; i < 32; i++) {
            int v = ds > 0 ? (int)lrintf((x[32 * j + i] + dm) / ds) : 0;
            q[32 * j + i] = iclamp(v, 0, nlev);
        }
    }
    put16(hdr, dh);
    put16(hdr + 2, mh);
    pack_scales_k(hdr + 4, sc, mn);
}

static void enc_q4_k(const float *x, uint8_t *b) {
    int q[QK_K];
    enc_qk_affine(x, 15, b, q);
    uint8_t *qs = b + 16;
    for (int j = 0; j < 4; j++)
        for (int l = 0; l < 32; l++)
            qs[32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
}

static void enc_q5_k(const float *x, uint8_t *b) {
    int q[QK_K];
    enc_qk_affine(x, 31, b, q);
    uint8_t *qh = b + 16, *qs = b + 48;
    memset(qh, 0, 32);
    for (int j = 0; j < 4; j++)
        for (int l = 0; l < 32; l++) {
            int a = q[64 * j + l], c = q[64 * j + 32 + l];
            qs[32 * j + l] = (uint8_t)((a & 15) | ((c & 15) << 4));
            qh[l] |= (uint8_t)(((a >> 4) << (2 * j)) | ((c >> 4) << (2 * j + 1)));
        }
}

static void enc_q6_k(const float *x, uint8_t *b) {
    float gs[16], maxs = 0.f;
    for (int g = 0; g < 16; g++) {
        float amax = 0.f, sv = 0.f;
        for (int i = 0; i < 16; i++) {
            float v = x[16 * g + i];
            if (fabsf(v) > amax) { amax = fabsf(v); sv = v; }
        }
        gs[g] = -sv / 32.f;          /* signed so the extreme maps to -32 */
        if (fabsf(gs[g]) > maxs) maxs = fabsf(gs[g]);
    }
    uint16_t dh = or_f32_to_f16(maxs / 127.f);
    float d = or_f16_to_f32(dh);
    int8_t sc[16];
    int q[QK_K];
    for (int g = 0; g < 16; g++) {
        sc[g] = (int8_t)(d > 0 ? iclamp((int)lrintf(gs[g] / d), -128, 127) : 0);
        float ds = d * (float)sc[g];
        for (int i = 0; i < 16; i++) {
            int v = ds != 0 ? (int)lrintf(x[16 * g + i] / ds) : 0;
            q[16 * g + i] = iclamp(v, -32, 31) + 32;
        }
    }
    uint8_t *ql = b, *qh = b + 128;
    memset(qh, 0, 64);
    for (int n = 0; n < 2; n++)
        for (int l = 0; l < 32; l++) {
            int q1 = q[128 * n + l], q2 = q[128 * n + 32 + l];
            int q3 = q[128 * n + 64 + l], q4 = q[128 * n + 96 + l];
            ql[64 * n + l] = (uint8_t)((q1 & 15) | ((q3 & 15) << 4));
            ql[64 * n + 32 + l] = (uint8_t)((q2 & 15) | ((q4 & 15) << 4));
            qh[32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    memcpy(b + 192, sc, 16);
    put16(b + 208, dh);
}

static void enc_q8_0(const float *x, uint8_t *b) {
    float amax = 0.f;
    for (int i = 0; i < 32; i++) if (fabsf(x[i]) > amax) amax = fabsf(x[i]);
    uint16_t dh = or_f32_to_f16(amax / 127.f);
    float d = or_f16_to_f32(dh);
    put16(b, dh);
    for (int i = 0; i < 32; i++)
        b[2 + i] = (uint8_t)(int8_t)(d > 0 ? iclamp((int)lrintf(x[i] / d), -127, 127) : 0);
}

int or_quantize(int type, const float *x, int64_t rows, int64_t cols, uint8_t *out) {
    int64_t rb = or_row_bytes(type, cols);
    if (rb == 0 || type == OR_F32 || type == OR_F16) return -1;
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * cols;
        uint8_t *o = out + r * rb;
        if (type == OR_Q8_0) {
            for (int64_t b = 0; b < cols / 32; b++) enc_q8_0(xr + 32 * b, o + 34 * b);
        } else {
            for (int64_t b = 0; b < cols / QK_K; b++) {
                if (type == OR_Q4_K) enc_q4_k(xr + QK_K * b, o + 144 * b);
                else if (type == OR_Q5_K) enc_q5_k(xr + QK_K * b, o + 176 * b);
                else enc_q6_k(xr + QK_K * b, o + 210 * b);
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Dequantizers, bit-exact restatements of src/Dequant.jl             */
/* ------------------------------------------------------------------ */

/* src/Dequant.jl:345-362: 6-bit (scale, min) of sub-block j */
static inline void get_scale_min_k(int j, const uint8_t *s, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* src/Dequant.jl:325-375 */
static void deq_q4_k(const uint8_t *b, float *y) {
    float d = or_f16_to_f32(get16(b)), dmin = or_f16_to_f32(get16(b + 2));
    const uint8_t *s = b + 4, *qs = b + 16;
    for (int j = 0; j < 4; j++) {
        uint8_t sc1, m1, sc2, m2;
        get_scale_min_k(2 * j, s, &sc1, &m1);
        get_scale_min_k(2 * j + 1, s, &sc2, &m2);
        float d1 = d * (float)sc1, min1 = dmin * (float)m1;
        float d2 = d * (float)sc2, min2 = dmin * (float)m2;
        for (int l = 0; l < 32; l++) {
            uint8_t v = qs[32 * j + l];
            y[64 * j + l] = d1 * (float)(v & 0x0f) - min1;
            y[64 * j + 32 + l] = d2 * (float)(v >> 4) - min2;
        }
    }
}

/* src/Dequant.jl:379-441 */
static void deq_q5_k(const uint8_t *b, float *y) {
    float d = or_f16_to_f32(get16(b)), dmin = or_f16_to_f32(get16(b + 2));
    const uint8_t *s = b + 4, *qh = b + 16, *qs = b + 48;
    for (int j = 0; j < 4; j++) {
        uint8_t sc1, m1, sc2, m2;
        get_scale_min_k(2 * j, s, &sc1, &m1);
        get_scale_min_k(2 * j + 1, s, &sc2, &m2);
        float d1 = d * (float)sc1, min1 = dmin * (float)m1;
        float d2 = d * (float)sc2, min2 = dmin * (float)m2;
        uint8_t u1 = (uint8_t)(1u << (2 * j)), u2 = (uint8_t)(1u << (2 * j + 1));
        for (int l = 0; l < 32; l++) {
            uint8_t v = qs[32 * j + l], h = qh[l];
            y[64 * j + l] = d1 * (float)((v & 0x0f) + ((h & u1) ? 16 : 0)) - min1;
            y[64 * j + 32 + l] = d2 * (float)((v >> 4) + ((h & u2) ? 16 : 0)) - min2;
        }
    }
}

/* src/Dequant.jl:558-601 (NOT src/QuantsCPU.jl:674, whose scale index is wrong) */
static void deq_q6_k(const uint8_t *b, float *y) {
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    float d = or_f16_to_f32(get16(b + 208));
    for (int n = 0; n < 2; n++) {
        const uint8_t *qls = ql + 64 * n, *qhs = qh + 32 * n;
        const int8_t *scs = sc + 8 * n;
        for (int l = 0; l < 32; l++) {
            int is = l / 16;
            uint8_t h = qhs[l];
            int q1 = (int)(int8_t)((qls[l] & 0x0f) | ((h & 0x03) << 4)) - 32;
            int q2 = (int)(int8_t)((qls[l + 32] & 0x0f) | (((h >> 2) & 0x03) << 4)) - 32;
            int q3 = (int)(int8_t)((qls[l] >> 4) | (((h >> 4) & 0x03) << 4)) - 32;
            int q4 = (int)(int8_t)((qls[l + 32] >> 4) | (((h >> 6) & 0x03) << 4)) - 32;
            y[128 * n + l] = d * (float)scs[is] * (float)q1;
            y[128 * n + l + 32] = d * (float)scs[is + 2] * (float)q2;
            y[128 * n + l + 64] = d * (float)scs[is + 4] * (float)q3;
            y[128 * n + l + 96] = d * (float)scs[is + 6] * (float)q4;
        }
    }
}

/* src/Dequant.jl:304-321 */
static void deq_q8_0(const uint8_t *b, float *y) {
    float d = or_f16_to_f32(get16(b));
    for (int j = 0; j < 32; j++) y[j] = d * (float)(int8_t)b[2 + j];
}

int or_dequantize(int type, const uint8_t *blk, int64_t n, float *out) {
    if (type == OR_F32) { memcpy(out, blk, (size_t)n * 4); return 0; }
    if (type == OR_F16) {
        for (int64_t i = 0; i < n; i++) out[i] = or_f16_to_f32(get16(blk + 2 * i));
        return 0;
    }
    if (type == OR_Q8_0) {
        if (n % 32) return -1;
        for (int64_t b = 0; b < n / 32; b++) deq_q8_0(blk + 34 * b, out + 32 * b);
        return 0;
    }
    if (n % QK_K) return -1;
    for (int64_t b = 0; b < n / QK_K; b++) {
        if (type == OR_Q4_K) deq_q4_k(blk + 144 * b, out + QK_K * b);
        else if (type == OR_Q5_K) deq_q5_k(blk + 176 * b, out + QK_K * b);
        else if (type == OR_Q6_K) deq_q6_k(blk + 210 * b, out + QK_K * b);
        else return -1;
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Reference GEMMs over dequantized rows                               */
/* ------------------------------------------------------------------ */

int or_gemm_f64(int type, const uint8_t *W, int64_t rows, int64_t cols,
                const float *X, int ncols, double *Y) {
    int64_t rb = or_row_bytes(type, cols);
    if (rb == 0) return -1;
    float *w = (float *)malloc((size_t)cols * sizeof(float));
    if (!w) return -2;
    for (int64_t r = 0; r < rows; r++) {
        if (or_dequantize(type, W + r * rb, cols, w)) { free(w); return -1; }
        for (int n = 0; n < ncols; n++) {
            const float *x = X + (int64_t)n * cols;
            double acc = 0.0;
            for (int64_t k = 0; k < cols; k++) acc += (double)w[k] * (double)x[k];
            Y[(int64_t)n * rows + r] = acc;
        }
    }
    free(w);
    return 0;
}

/* quantize_row_q8_K (src/kernels/quant_kernels.c:166-194): per block of 256,
 * d = amax / 127, q = roundf(x * (1/d)) (0 when amax is 0), f32 throughout */
void or_quantize_q8k(const float *x, int64_t k, float *d, int8_t *q) {
    for (int64_t b = 0; b < k / QK_K; b++) {
        const float *s = x + QK_K * b;
        float amax = 0.f;
        for (int j = 0; j < QK_K; j++) {
            const float a = fabsf(s[j]);
            if (a > amax) amax = a;
        }
        const float dd = amax / 127.0f;
        const float id = dd != 0.f ? 1.0f / dd : 0.f;
        d[b] = dd;
        for (int j = 0; j < QK_K; j++) q[QK_K * b + j] = (int8_t)roundf(s[j] * id);
    }
}

/* The reference's quantized matvec (q4_k_gemv .. q6_k_gemv, quant_kernels.c:602-650):
 * activations quantized to Q8_K, then sum_b d8_b * sum_{k in b} w[k] q8[k], here in
 * double over the dequantized weights ("truth" for the quantized activations). */
int or_gemm_q8k(int type, const uint8_t *W, int64_t rows, int64_t cols,
                const float *X, int ncols, double *Y) {
    int64_t rb = or_row_bytes(type, cols);
    if (rb == 0 || cols % QK_K || type == OR_Q8_0) return -1;
    const int64_t nb = cols / QK_K;
    float *w = (float *)malloc((size_t)cols * sizeof(float));
    float *d8 = (float *)malloc((size_t)nb * ncols * sizeof(float));
    int8_t *q8 = (int8_t *)malloc((size_t)cols * ncols);
    if (!w || !d8 || !q8) { free(w); free(d8); free(q8); return -2; }
    for (int n = 0; n < ncols; n++) or_quantize_q8k(X + (int64_t)n * cols, cols, d8 + nb * n, q8 + cols * n);
    for (int64_t r = 0; r < rows; r++) {
        if (or_dequantize(type, W + r * rb, cols, w)) { free(w); free(d8); free(q8); return -1; }
        for (int n = 0; n < ncols; n++) {
            const int8_t *q = q8 + cols * n;
            double acc = 0.0;
            for (int64_t b = 0; b < nb; b++) {
                double s = 0.0;
                for (int j = 0; j < QK_K; j++) s += (double)w[QK_K * b + j] * (double)q[QK_K * b + j];
                acc += (double)d8[nb * n + b] * s;
            }
            Y[(int64_t)n * rows + r] = acc;
        }
    }
    free(w); free(d8); free(q8);
    return 0;
}

int or_gemm_f32(int type, const uint8_t *W, int64_t rows, int64_t cols,
                const float *X, int ncols, float *Y) {
    int64_t rb = or_row_bytes(type, cols);
    if (rb == 0) return -1;
    float *w = (float *)malloc((size_t)cols * sizeof(float));
    if (!w) return -2;
    for (int64_t r = 0; r < rows; r++) {
        if (or_dequantize(type, W + r * rb, cols, w)) { free(w); return -1; }
        for (int n = 0; n < ncols; n++) {
            const float *x = X + (int64_t)n * cols;
            float acc = 0.f;
            for (int64_t k = 0; k < cols; k++) acc += w[k] * x[k];
            Y[(int64_t)n * rows + r] = acc;
        }
    }
    free(w);
    return 0;
}
