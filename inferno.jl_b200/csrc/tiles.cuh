// Device layout of quantized weights ("M-tiles") and the index maps shared by
// the repack, dequant and GEMV kernels.  Plain integer arithmetic, usable from
// host code (the CPU tests compile this header with g++ to check the maps).
//
// A matrix of M rows x K columns is stored as [row block of 16][unit][M-tile]
// where a unit is 256 consecutive columns (one K-quant super-block per row,
// or eight Q8_0 blocks) and an M-tile holds the 16 rows' bytes of one unit,
// re-arranged so that lane (g = lane/4, t = lane%4) of a warp reads its bytes
// with bank-conflict-free 16-byte shared-memory loads.  The M-tile has exactly
// the bytes of the 16 GGUF blocks it came from (no padding), so traffic equals
// the algorithmic bytes; rows beyond M (to a multiple of 16) and Q8_0 blocks
// beyond K (to a multiple of 256) are zero-filled.
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

// ---- byte offsets inside an M-tile ----------------------------------------
// Q4_K / Q5_K
//   header of row r (raw bytes 0..15: d, dmin, 12 scale bytes)  16*r
//   Q5_K qh half h of row r (raw bytes 16+16h .. +16)           256 + (2r+h)*16
//   qs piece (c, r, t) (raw qs bytes 64c+16t .. +16)            QS0 + ((16c+r)*4+t)*16
IFR_HD int qk_hdr(int r) { return 16 * r; }
IFR_HD int q5_qh(int r, int h) { return 256 + (2 * r + h) * 16; }
IFR_HD int qk_qs(bool q5, int c, int r, int t) { return (q5 ? 768 : 256) + ((16 * c + r) * 4 + t) * 16; }
// Q6_K
//   d of row r                                   2*r
//   16 int8 group scales of row r                32 + 16*r
//   ql half h of lane quad t, row r              288 + ((16h+r)*4+t)*16
//        holding raw ql bytes 16k+4t+j for k = 4h..4h+3, j = 0..3
//   qh of lane quad t, row r                     2336 + (4r+t)*16
//        holding raw qh bytes 16k+4t+j for k = 0..3, j = 0..3
IFR_HD int q6_d(int r) { return 2 * r; }
IFR_HD int q6_sc(int r) { return 32 + 16 * r; }
IFR_HD int q6_ql(int h, int r, int t) { return 288 + ((16 * h + r) * 4 + t) * 16; }
IFR_HD int q6_qh(int r, int t) { return 2336 + (4 * r + t) * 16; }
// Q8_0 (unit = 8 blocks)
//   d of the 8 blocks of row r                   16*r
//   qs piece (q, r, t): block 2q bytes 8t..8t+7, then block 2q+1 bytes 8t..8t+7
IFR_HD int q8_d(int r) { return 16 * r; }
IFR_HD int q8_qs(int q, int r, int t) { return 256 + ((16 * q + r) * 4 + t) * 16; }

// ---- MMA k-slot -> element of the unit ------------------------------------
// slot 0..3 = k columns 2t, 2t+1, 2t+8, 2t+9 of step s (16 steps per unit)
IFR_HD int jmap(int slot) { return slot == 0 ? 0 : slot == 1 ? 2 : slot == 2 ? 1 : 3; }
IFR_HD int elem_qk(int s, int t, int slot) {
    int c = s >> 3, w = (s >> 1) & 3, h = s & 1, p = t >> 1;
    int j4 = 2 * c + p;
    int l = 16 * (t & 1) + 4 * w + h + ((slot & 1) ? 2 : 0);
    return 64 * j4 + ((slot & 2) ? 32 : 0) + l;
}
IFR_HD int elem_q6k(int s, int t, int slot) {
    int n = s >> 3, qq = (s >> 1) & 3, b = s & 1;
    return 128 * n + 32 * qq + 16 * b + 4 * t + jmap(slot);
}
IFR_HD int elem_q80(int s, int t, int slot) { return 32 * (s >> 1) + 8 * t + 4 * (s & 1) + jmap(slot); }
IFR_HD int elem_of(int type, int s, int t, int slot) {
    return type == 14 ? elem_q6k(s, t, slot) : type == 8 ? elem_q80(s, t, slot) : elem_qk(s, t, slot);
}
// sub-block feeding k-row 2t+kr of the Q4_K/Q5_K min MMA (m16n8k8)
IFR_HD int minsub_qk(int t, int kr) { return (t & 1) ? (4 + 2 * (t >> 1) + kr) : (2 * (t >> 1) + kr); }

// ---- holders: which lane of an 8-lane column group keeps element e ---------
// (holder j, register r) <-> e is a bijection of 0..255 onto 8 x 32 with r
// independent of t for every (s, slot), so one warp shuffle per k-slot moves
// activations from holders to fragments.
IFR_HD int holder_of(int type, int e) {
    if (type == 12 || type == 13) return (e >> 4) & 7;
    if (type == 14) return ((e >> 2) & 3) + 4 * ((e >> 4) & 1);
    return ((e >> 3) & 3) + 4 * ((e >> 2) & 1);  // Q8_0
}
IFR_HD int hreg_of(int type, int e) {
    if (type == 12 || type == 13) return (e & 15) + 16 * (e >> 7);
    return (e & 3) + 4 * (e >> 5);
}
IFR_HD int elem_of_holder(int type, int j, int r) {
    if (type == 12 || type == 13) return 128 * (r >> 4) + 16 * j + (r & 15);
    if (type == 14) return 32 * (r >> 2) + 16 * (j >> 2) + 4 * (j & 3) + (r & 3);
    return 32 * (r >> 2) + 8 * (j & 3) + 4 * (j >> 2) + (r & 3);
}
// the holder register of slot `slot` in step s (t-free form of hreg_of(elem_of))
IFR_HD int slot_reg(int type, int s, int slot) {
    if (type == 12 || type == 13)
        return 4 * ((s >> 1) & 3) + (s & 1) + 2 * (slot & 1) + 16 * (s >> 3);
    return jmap(slot) + 4 * (s >> 1);
}

}  // namespace ifr
