// Device layouts, re-layout (repack) of GGUF blocks, and the bit-exact
// dequantization kernels.
//
// Dequantized values follow the reference's src/Dequant.jl exactly: f32
// products rounded separately (no fused multiply-add, which Julia does not
// form there), hence the explicit __fmul_rn/__fsub_rn.
#include "common.cuh"

namespace ifr {

int64_t raw_row_bytes(int type, int64_t cols) {
    switch (type) {
    case 8: return (cols % 32) ? 0 : cols / 32 * 34;
    case 12: return (cols % 256) ? 0 : cols / 256 * 144;
    case 13: return (cols % 256) ? 0 : cols / 256 * 176;
    case 14: return (cols % 256) ? 0 : cols / 256 * 210;
    }
    return 0;
}

int64_t device_bytes(int type, int64_t rows, int64_t cols) {
    int64_t rb = raw_row_bytes(type, cols);
    if (rb == 0) return 0;
    int64_t b = rb * rows;
    // planes are 16-byte aligned; leave room for the alignment of the d plane
    return (b + 255) / 256 * 256 + 256;
}

// ---------------------------------------------------------------- repack ----

// Q6_K: one thread per 16-byte destination piece of ql'/qh'
__global__ void repack_q6k_kernel(const uint8_t *__restrict__ raw, uint8_t *__restrict__ ql,
                                  uint8_t *__restrict__ qh, uint8_t *__restrict__ sc,
                                  uint16_t *__restrict__ d, int64_t nblk) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= nblk) return;
    const uint8_t *b = raw + i * 210;
    uint8_t *qlo = ql + i * 128, *qho = qh + i * 64, *sco = sc + i * 16;
    for (int t = 0; t < 4; t++)
        for (int k = 0; k < 8; k++)
            for (int j = 0; j < 4; j++) qlo[32 * t + 4 * k + j] = b[16 * k + 4 * t + j];
    for (int t = 0; t < 4; t++)
        for (int k = 0; k < 4; k++)
            for (int j = 0; j < 4; j++) qho[16 * t + 4 * k + j] = b[128 + 16 * k + 4 * t + j];
    for (int j = 0; j < 16; j++) sco[j] = b[192 + j];
    d[i] = (uint16_t)(b[208] | (b[209] << 8));
}

__global__ void repack_q80_kernel(const uint8_t *__restrict__ raw, uint8_t *__restrict__ qs,
                                  uint16_t *__restrict__ d, int64_t nblk) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= nblk) return;
    const uint8_t *b = raw + i * 34;
    d[i] = (uint16_t)(b[0] | (b[1] << 8));
    uint8_t *o = qs + i * 32;
    for (int j = 0; j < 32; j++) o[j] = b[2 + j];
}

cudaError_t repack(const QTensor &t, const uint8_t *raw, cudaStream_t s) {
    int64_t nblk = t.rows * t.nb;
    if (nblk == 0) return cudaSuccess;
    int threads = 256;
    unsigned grid = (unsigned)((nblk + threads - 1) / threads);
    if (t.type == 14) {
        repack_q6k_kernel<<<grid, threads, 0, s>>>(raw, t.data + t.off_ql, t.data + t.off_qh,
                                                   t.data + t.off_sc,
                                                   (uint16_t *)(t.data + t.off_d), nblk);
    } else if (t.type == 8) {
        repack_q80_kernel<<<grid, threads, 0, s>>>(raw, t.data + t.off_ql,
                                                   (uint16_t *)(t.data + t.off_d), nblk);
    } else {
        return cudaMemcpyAsync(t.data, raw, raw_row_bytes(t.type, t.cols) * t.rows,
                               cudaMemcpyDeviceToDevice, s);
    }
    return cudaGetLastError();
}

// --------------------------------------------------------------- dequant ----

// src/Dequant.jl:345-362
IFR_DEV void scale_min_k(int j, const uint8_t *s, uint32_t &sc, uint32_t &m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// one thread per 32 elements; Q4_K (src/Dequant.jl:325-375), Q5_K (:379-441)
template <bool Q5>
__global__ void dequant_qk_kernel(const uint8_t *__restrict__ w, float *__restrict__ out,
                                  int64_t nsub) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= nsub) return;
    int64_t blk = i >> 3;
    int sub = (int)(i & 7);  // sub-block of 32: group j = sub/2, high nibbles if odd
    const uint8_t *b = w + blk * (Q5 ? 176 : 144);
    float d = h2f((uint16_t)(b[0] | (b[1] << 8)));
    float dmin = h2f((uint16_t)(b[2] | (b[3] << 8)));
    uint32_t sc, m;
    scale_min_k(sub, b + 4, sc, m);
    float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
    int j = sub >> 1, hi = sub & 1;
    const uint8_t *qs = b + (Q5 ? 48 : 16) + 32 * j;
    const uint8_t *qh = b + 16;
    float *o = out + i * 32;
    for (int l = 0; l < 32; l++) {
        uint32_t q = hi ? (qs[l] >> 4) : (qs[l] & 0x0f);
        if (Q5 && ((qh[l] >> (2 * j + hi)) & 1)) q += 16;
        o[l] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
}

// Q6_K from the planar layout, one thread per 16-element group
// (src/Dequant.jl:558-601: d * sc * q evaluated left to right)
__global__ void dequant_q6k_kernel(const uint8_t *__restrict__ ql, const uint8_t *__restrict__ qh,
                                   const int8_t *__restrict__ sc, const uint16_t *__restrict__ dd,
                                   float *__restrict__ out, int64_t ngrp) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= ngrp) return;
    int64_t blk = i >> 4;
    int g = (int)(i & 15);
    int n = g >> 3, qq = (g >> 1) & 3, bsel = g & 1;
    float d = h2f(dd[blk]);
    float ds = __fmul_rn(d, (float)sc[blk * 16 + g]);
    const uint8_t *qlb = ql + blk * 128, *qhb = qh + blk * 64;
    float *o = out + blk * 256 + 128 * n + 32 * qq + 16 * bsel;
    for (int e = 0; e < 16; e++) {
        int l = 16 * bsel + e;            // position inside the 32-run
        int t = (l >> 2) & 3, j = l & 3;  // lane-permuted layout, see QTensor
        int a = qq & 1;
        int k = 4 * n + 2 * a + bsel;     // original ql offset 64n+32a+16b+4t+j = 16k+4t+j
        uint8_t lb = qlb[32 * t + 4 * k + j];
        uint32_t lo = (qq < 2) ? (lb & 0x0f) : (lb >> 4);
        int kh = 2 * n + bsel;            // original qh offset 32n+16b+4t+j = 16kh+4t+j
        uint8_t hb = qhb[16 * t + 4 * kh + j];
        uint32_t h = (hb >> (2 * qq)) & 3;
        int q = (int)(lo | (h << 4)) - 32;
        o[e] = __fmul_rn(ds, (float)q);
    }
}

// Q8_0 (src/Dequant.jl:304-321), one thread per block
__global__ void dequant_q80_kernel(const int8_t *__restrict__ qs, const uint16_t *__restrict__ dd,
                                   float *__restrict__ out, int64_t nblk) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= nblk) return;
    float d = h2f(dd[i]);
    for (int j = 0; j < 32; j++) out[i * 32 + j] = __fmul_rn(d, (float)qs[i * 32 + j]);
}

cudaError_t dequant(const QTensor &t, float *out, cudaStream_t s) {
    int threads = 256;
    int64_t nblk = t.rows * t.nb;
    if (nblk == 0) return cudaSuccess;
    if (t.type == 12 || t.type == 13) {
        int64_t n = nblk * 8;
        unsigned grid = (unsigned)((n + threads - 1) / threads);
        if (t.type == 12) dequant_qk_kernel<false><<<grid, threads, 0, s>>>(t.data, out, n);
        else dequant_qk_kernel<true><<<grid, threads, 0, s>>>(t.data, out, n);
    } else if (t.type == 14) {
        int64_t n = nblk * 16;
        unsigned grid = (unsigned)((n + threads - 1) / threads);
        dequant_q6k_kernel<<<grid, threads, 0, s>>>(t.data + t.off_ql, t.data + t.off_qh,
                                                    (const int8_t *)(t.data + t.off_sc),
                                                    (const uint16_t *)(t.data + t.off_d), out, n);
    } else if (t.type == 8) {
        unsigned grid = (unsigned)((nblk + threads - 1) / threads);
        dequant_q80_kernel<<<grid, threads, 0, s>>>((const int8_t *)(t.data + t.off_ql),
                                                    (const uint16_t *)(t.data + t.off_d), out,
                                                    nblk);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace ifr
