// Bit-exact dequantization of one 32-element group of an M-tile tensor (the
// values of the reference's src/Dequant.jl), shared by the dequant kernel and
// the engine's embedding gathers.  Products are rounded separately (no fused
// multiply-add, which Julia does not form there), hence __fmul_rn/__fsub_rn.
#pragma once
#include "common.cuh"
#include "tiles.cuh"

namespace ifr {

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

IFR_DEV float h2f_bytes(const uint8_t *p) { return h2f((uint16_t)(p[0] | (p[1] << 8))); }

// elements 32 sub .. 32 sub + 31 of unit u of `row` into o[0..32)
// (Q8_0: nothing for blocks beyond the tensor's nb_raw blocks per row)
template <int T>
IFR_DEV void dequant_group(const uint8_t *__restrict__ w, int64_t nu, int64_t nb_raw, int64_t row, int64_t u,
                           int sub, float *o) {
    const int r = (int)(row & 15);
    const uint8_t *tile = w + ((row >> 4) * nu + u) * mtile_bytes(T);
    if (T == 12 || T == 13) {
        // src/Dequant.jl:325-375 (Q4_K), :379-441 (Q5_K): element e = 32 sub + l is
        // nibble (e % 64 >= 32) of raw qs byte 32 (e / 64) + e % 32, Q5_K bit sub of qh byte l
        constexpr bool q5 = T == 13;
        const uint8_t *hdr = tile + qk_hdr(r);
        const float d = h2f_bytes(hdr), dmin = h2f_bytes(hdr + 2);
        uint32_t sc, m;
        scale_min_k(sub, hdr + 4, sc, m);
        const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
        const int hi = sub & 1;
        for (int l = 0; l < 32; l++) {
            const int e = 32 * sub + l;
            const uint8_t v = tile[qk_qs_byte(q5, r, 32 * (e >> 6) + (e & 31))];
            uint32_t q = hi ? (v >> 4) : (v & 0x0f);
            if (q5 && ((tile[q5_qh_byte(r, l)] >> sub) & 1)) q += 16;
            o[l] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
        }
    } else if (T == 14) {
        // src/Dequant.jl:558-601: (d * sc[e / 16]) * (q - 32)
        const float d = h2f_bytes(tile + q6_d(r));
        for (int l = 0; l < 32; l++) {
            const int e = 32 * sub + l;
            const float ds = __fmul_rn(d, (float)(int8_t)tile[q6_sc(r) + (e >> 4)]);
            const int l4 = (tile[q6_ql_byte(r, q6_raw_lo_byte(e))] >> q6_raw_lo_shift(e)) & 15;
            const int h2 = (tile[q6_qh_byte(r, q6_raw_hi_byte(e) - 128)] >> q6_raw_hi_shift(e)) & 3;
            o[l] = __fmul_rn(ds, (float)((l4 | (h2 << 4)) - 32));
        }
    } else {
        // Q8_0, src/Dequant.jl:304-321; block `sub` of the unit
        const int64_t blk = 8 * u + sub;
        if (blk >= nb_raw) return;
        const float d = h2f_bytes(tile + q8_d(r) + 2 * sub);
        for (int l = 0; l < 32; l++) o[l] = __fmul_rn(d, (float)(int8_t)tile[q8_qs_byte(r, 32 * sub + l)]);
    }
}

}  // namespace ifr
