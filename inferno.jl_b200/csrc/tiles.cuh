// Device layout of quantized weights ("M-tiles") and the index maps shared by
// the repack, dequant and GEMV kernels.  Plain integer arithmetic, usable from
// host code (the CPU tests compile this header with g++ to check the maps).
//
// A matrix of M rows x K columns is stored as [row block of 16][unit][M-tile]
// where a unit is 256 consecutive columns (one K-quant super-block per row,
// or eight Q8_0 blocks) and an M-tile holds the 16 rows' data of one unit.
// The M-tile has exactly the bits of the 16 GGUF blocks it came from (no
// padding, nothing added), so traffic equals the algorithmic bytes; rows
// beyond M (to a multiple of 16) and Q8_0 blocks beyond K are zero-filled.
//
// Tensor-core mapping.  In 16-element step s of a unit (s = 2c + h: half h of
// 32-element chunk c), MMA lane quad t (t = lane % 4) holds the elements
// 16 s + 4t + {0..3}, the 4 bytes of one 4-byte word of its stream:
//   * exact f32 activations (fp16 hi + lo on mma.m16n8k16.f16): bytes (0, 2)
//     are k-slots (2t, 2t+1) and bytes (1, 3) are k-slots (2t+8, 2t+9), which
//     is what the fp16 magic-number unpack (w & 0x000F000F) | 0x64006400 and
//     the same on (w >> 8) produce;
//   * Q8_K activations (mma.m16n8k32.s8, K-quants): chunk c is one k32 step,
//     its two words are k-slots 4t..4t+3 and 16+4t..16+4t+3 (Q6_K: two k16
//     steps, one per 16-element scale group).
// A K-quant sub-block (32 elements) is one chunk, so one scale per step.  The
// weight bytes a lane needs are stored as a contiguous "stream" in 16-byte
// pieces placed so that a warp reads them with conflict-free 16-byte
// shared-memory loads; bytes keep their raw order inside each word.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define IFR_HD __host__ __device__ __forceinline__ constexpr
#else
#define IFR_HD static inline constexpr
#endif

namespace ifr {

constexpr int kUnitElems = 256;

IFR_HD int mtile_bytes(int type) {
    return type == 12 ? 2304 : type == 13 ? 2816 : type == 14 ? 3360 : type == 8 ? 4352 : 0;
}
IFR_HD int raw_block_elems(int type) { return type == 8 ? 32 : 256; }
IFR_HD int raw_block_bytes(int type) {
    return type == 12 ? 144 : type == 13 ? 176 : type == 14 ? 210 : type == 8 ? 34 : 0;
}

// K-quants: element of chunk c, lane quad t, slot j (0..7; j >= 4 is the +16 half)
IFR_HD int elem_k(int c, int t, int j) { return 32 * c + 4 * t + (j & 3) + ((j & 4) ? 16 : 0); }
// element of step s, lane quad t, byte j of its word (all formats)
IFR_HD int elem_s(int s, int t, int j) { return 16 * s + 4 * t + j; }
// the lane word (0..1) and byte of element e within its 32-element chunk:
// word h = (e % 32) / 16, byte (e % 4); lane t = (e % 16) / 4
IFR_HD int k_lane(int e) { return (e >> 2) & 3; }
IFR_HD int k_half(int e) { return (e >> 4) & 1; }

// ---- Q4_K / Q5_K --------------------------------------------------------------
//   header of row r (raw bytes 0..15: d, dmin, 12 scale bytes)       16 r
//   Q5_K qh words of rows g and g+8 for lane quad t                 256 + (4g+t)*16
//        row g: raw qh bytes 4t..4t+3, 16+4t..16+4t+3; then row g+8 (bit c = chunk c)
//   qs piece (q, r, t): raw qs bytes 32p + 4t.., 32p + 16 + 4t.. for p = 2q, 2q+1
//                                                                   QS0 + ((16q+r)*4+t)*16
// Raw qs byte 32p + l holds element 64p + l (low nibble, chunk 2p) and
// 64p + 32 + l (high nibble, chunk 2p+1).
IFR_HD int qk_hdr(int r) { return 16 * r; }
IFR_HD int q5_qh(int g, int t) { return 256 + (4 * g + t) * 16; }
IFR_HD int qk_qs(bool q5, int q, int r, int t) { return (q5 ? 768 : 256) + ((16 * q + r) * 4 + t) * 16; }
IFR_HD int qk_qs_byte(bool q5, int r, int qb) {  // raw qs byte qb (0..127) of row r
    const int p = qb >> 5, l = qb & 31;
    return qk_qs(q5, p >> 1, r, k_lane(l)) + 8 * (p & 1) + 4 * k_half(l) + (l & 3);
}
IFR_HD int q5_qh_byte(int r, int l) {  // raw qh byte l (0..31) of row r
    return q5_qh(r & 7, k_lane(l)) + 8 * (r >> 3) + 4 * k_half(l) + (l & 3);
}

// ---- Q6_K -----------------------------------------------------------------------
//   d of row r                                   2 r
//   16 int8 group scales of row r (raw order)     32 + 16 r
//   ql piece (n, r, t)                            288 + ((16n+r)*4+t)*16
//        words: raw ql bytes 64n + 32h1 + 16h + 4t .. +4 for (h1, h) = (0,0), (0,1), (1,0), (1,1)
//   qh piece (r, t)                               2336 + (4r+t)*16
//        words: raw qh bytes 32n + 16h + 4t .. +4 for (n, h) = (0,0), (0,1), (1,0), (1,1)
// Element e = 128n + 32qq + l of the raw block: 6-bit q = (ql[64n + 32(qq%2) + l]
// >> 4(qq/2)) & 15 | ((qh[32n + l] >> 2qq) & 3) << 4, value d * sc[e/16] * (q - 32)
// (src/Dequant.jl:558-601).  Chunk c = 4n + qq.
IFR_HD int q6_d(int r) { return 2 * r; }
IFR_HD int q6_sc(int r) { return 32 + 16 * r; }
IFR_HD int q6_ql(int n, int r, int t) { return 288 + ((16 * n + r) * 4 + t) * 16; }
IFR_HD int q6_qh(int r, int t) { return 2336 + (4 * r + t) * 16; }
IFR_HD int q6_ql_byte(int r, int qb) {  // raw ql byte qb (0..127)
    const int n = qb >> 6, h1 = (qb >> 5) & 1, l = qb & 31;
    return q6_ql(n, r, k_lane(l)) + 8 * h1 + 4 * k_half(l) + (l & 3);
}
IFR_HD int q6_qh_byte(int r, int hb) {  // raw qh byte hb (0..63)
    const int n = hb >> 5, l = hb & 31;
    return q6_qh(r, k_lane(l)) + 8 * n + 4 * k_half(l) + (l & 3);
}
// raw Q6_K block: the two parts of element e (ql at 0, qh at 128, sc at 192, d at 208)
IFR_HD int q6_raw_lo_byte(int e) { return 64 * (e >> 7) + 32 * ((e >> 5) & 1) + (e & 31); }
IFR_HD int q6_raw_lo_shift(int e) { return ((e >> 6) & 1) ? 4 : 0; }
IFR_HD int q6_raw_hi_byte(int e) { return 128 + 32 * (e >> 7) + (e & 31); }
IFR_HD int q6_raw_hi_shift(int e) { return 2 * ((e >> 5) & 3); }

// ---- Q8_0 (unit = 8 blocks) --------------------------------------------------------
//   d of the 8 blocks of row r (raw order)         16 r
//   qs piece (q, r, t): lane stream words 4q .. 4q+3, word s = block s/2 bytes
//        16 (s%2) + 4t .. +4 (elements 16 s + 4t + {0..3})
IFR_HD int q8_d(int r) { return 16 * r; }
IFR_HD int q8_qs(int q, int r, int t) { return 256 + ((16 * q + r) * 4 + t) * 16; }
IFR_HD int q8_qs_byte(int r, int e) {
    const int s = e >> 4, t = (e >> 2) & 3;
    return q8_qs(s >> 2, r, t) + 4 * (s & 3) + (e & 3);
}

}  // namespace ifr
