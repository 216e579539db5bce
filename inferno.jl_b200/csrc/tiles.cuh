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
// Tensor-core mapping.  The GEMV multiplies one M-tile by the activations with
// 16 steps of mma.m16n8k16.  In step s, MMA lane quad t (t = lane % 4) holds
// the k-slots {2t, 2t+1, 2t+8, 2t+9} ("slots" 0..3); slot `slot` of step s is
// unit element elem(type, s, t, slot):
//   Q4_K / Q5_K   64 t + 4 s + slot   lane quad t owns the contiguous elements
//                                     64t .. 64t+63 = sub-blocks 2t (steps 0-7)
//                                     and 2t+1 (steps 8-15); their 6-bit scales
//                                     are folded into the fp16 weights, so a
//                                     step may mix sub-blocks
//   Q6_K / Q8_0   16 s + 4 t + slot   step s is one Q6_K scale group of 16 (and
//                                     steps 2b, 2b+1 one Q8_0 block): their
//                                     scales multiply the f32 MMA results
// Each lane's weight bits are stored as a contiguous "stream" in 16-byte
// pieces placed so that a warp reads them with conflict-free 16-byte
// shared-memory loads, and inside every 4-byte word the bytes are ordered
// (b0, b2, b1, b3): the fp16 magic-number unpack (w & 0x000F000F) | 0x64006400
// then yields slots (0, 1) from the bytes at positions 0 and 2, and the same
// on (w >> 8) yields slots (2, 3).
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

IFR_HD int elem(int type, int s, int t, int slot) {
    return (type == 12 || type == 13) ? 64 * t + 4 * s + slot : 16 * s + 4 * t + slot;
}
// byte order inside a stored 4-byte word (self-inverse): raw i <-> position wperm(i)
IFR_HD int wperm(int i) { return i == 1 ? 2 : (i == 2 ? 1 : i); }
// position of byte i (0..15) of a lane stream inside its 16-byte piece
IFR_HD int piece_byte(int i) { return (i & 12) + wperm(i & 3); }

// ---- Q4_K / Q5_K --------------------------------------------------------------
//   header of row r (raw bytes 0..15: d, dmin, 12 scale bytes)       16 r
//   Q5_K qh bit-words of rows g and g+8 for lane quad t              256 + (4g+t)*16
//        (8 bytes per row: word 0 = slots 0 | 1 << 16, word 1 = slots 2 | 3 << 16,
//         bit s of each half = step s)
//   qs piece (p, r, t): raw qs bytes 32t + 16p .. +16, word-permuted   QS0 + ((16p+r)*4+t)*16
// Raw qs byte 32t + w holds element 64t + w (low nibble, step w/4) and
// 64t + 32 + w (high nibble, step 8 + w/4).
IFR_HD int qk_hdr(int r) { return 16 * r; }
IFR_HD int q5_qh(int g, int t) { return 256 + (4 * g + t) * 16; }
IFR_HD int qk_qs(bool q5, int p, int r, int t) { return (q5 ? 768 : 256) + ((16 * p + r) * 4 + t) * 16; }
IFR_HD int qk_qs_byte(bool q5, int r, int q) {  // raw qs byte q (0..127) of row r
    return qk_qs(q5, (q & 31) >> 4, r, q >> 5) + piece_byte(q & 15);
}
// Q5_K high bit of element e of row r: tile byte, and the bit inside it
IFR_HD int q5_bit_byte(int r, int e) {
    const int t = e >> 6, j = e & 63, s = j >> 2, slot = j & 3;
    const int b = ((slot & 1) ? 16 : 0) + s;
    return q5_qh(r & 7, t) + 8 * (r >> 3) + 4 * (slot >> 1) + (b >> 3);
}
IFR_HD int q5_bit_shift(int e) {
    const int j = e & 63, s = j >> 2, slot = j & 3;
    return (((slot & 1) ? 16 : 0) + s) & 7;
}

// ---- Q6_K -----------------------------------------------------------------------
//   d of row r                                   2 r
//   16 int8 group scales of row r (raw order)     32 + 16 r   (step s uses scale s)
//   ql piece (p, r, t)                            288 + ((16p+r)*4+t)*16
//        lane stream word w (0..7) = raw ql bytes of elements 16 s + 4t + {0..3}
//        for s = (w & 3) + 8 (w >> 2): low nibbles = step s, high nibbles = step s + 4
//   qh piece (r, t)                               2336 + (4r+t)*16
//        word j (0..3) = raw qh bytes 32 (j/2) + 16 (j%2) + 4t + {0..3}: bits 2qq of
//        step 8 (j/2) + 2 qq + j%2
// Element e of the raw block: 6-bit q = ql nibble | qh 2 bits << 4, value
// d * sc[e/16] * (q - 32) (src/Dequant.jl:558-601).
IFR_HD int q6_d(int r) { return 2 * r; }
IFR_HD int q6_sc(int r) { return 32 + 16 * r; }
IFR_HD int q6_ql(int p, int r, int t) { return 288 + ((16 * p + r) * 4 + t) * 16; }
IFR_HD int q6_qh(int r, int t) { return 2336 + (4 * r + t) * 16; }
// ql word of step s and its nibble; qh word of step s and its bit pair
IFR_HD int q6_lo_word(int s) { return (s & 3) + 4 * (s >> 3); }
IFR_HD int q6_lo_shift(int e) { return ((e >> 6) & 1) ? 4 : 0; }
IFR_HD int q6_hi_word(int s) { return 2 * (s >> 3) + (s & 1); }
IFR_HD int q6_hi_shift(int e) { return 2 * ((e >> 5) & 3); }
IFR_HD int q6_lo_byte(int r, int e) {
    const int s = e >> 4, t = (e >> 2) & 3, slot = e & 3;
    const int i = 4 * q6_lo_word(s) + wperm(slot);
    return q6_ql(i >> 4, r, t) + (i & 15);
}
IFR_HD int q6_hi_byte(int r, int e) {
    const int s = e >> 4, t = (e >> 2) & 3, slot = e & 3;
    return q6_qh(r, t) + 4 * q6_hi_word(s) + wperm(slot);
}
// raw Q6_K block: the two parts of element e (ql at 0, qh at 128, sc at 192, d at 208)
IFR_HD int q6_raw_lo_byte(int e) { return 64 * (e >> 7) + 32 * ((e >> 5) & 1) + (e & 31); }
IFR_HD int q6_raw_lo_shift(int e) { return ((e >> 6) & 1) ? 4 : 0; }
IFR_HD int q6_raw_hi_byte(int e) { return 128 + 32 * (e >> 7) + (e & 31); }
IFR_HD int q6_raw_hi_shift(int e) { return 2 * ((e >> 5) & 3); }

// ---- Q8_0 (unit = 8 blocks) --------------------------------------------------------
//   d of the 8 blocks of row r (raw order)         16 r
//   qs piece (q, r, t): lane stream words 4q .. 4q+3, word s = block s/2 bytes
//        16 (s%2) + 4t .. +4 (elements 16 s + 4t + {0..3}), word-permuted
IFR_HD int q8_d(int r) { return 16 * r; }
IFR_HD int q8_qs(int q, int r, int t) { return 256 + ((16 * q + r) * 4 + t) * 16; }
IFR_HD int q8_qs_byte(int r, int e) {
    const int s = e >> 4, t = (e >> 2) & 3, slot = e & 3;
    return q8_qs(s >> 2, r, t) + 4 * (s & 3) + wperm(slot);
}

}  // namespace ifr
