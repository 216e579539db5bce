"""CPU check of the device-layout index maps in csrc/tiles.cuh: compiled with
g++ as host code and run (no GPU).  These maps decide which activation meets
which weight on the tensor cores, so they are checked exhaustively."""
import os
import subprocess
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "inferno.jl_b200", "csrc")

CHECKER = r"""
#include "tiles.cuh"
#include <cstdio>
#include <cstring>
#include <initializer_list>
using namespace ifr;
static int fails = 0;
#define CHECK(c) do { if (!(c)) { std::printf("FAIL %s line %d\n", #c, __LINE__); fails++; } } while (0)

// bit coverage of one M-tile
static int cov[4352 * 8];
static void mark_bits(int byte, int bit0, int nbits) { for (int i = 0; i < nbits; i++) cov[byte * 8 + bit0 + i]++; }
static void mark_bytes(int byte, int n) { for (int i = 0; i < n; i++) mark_bits(byte + i, 0, 8); }
static int pos_of_slot(int slot) { return wperm(slot); }  // stored position the GEMV unpack reads

int main() {
    // the MMA element map covers the unit once
    int seen[256]; std::memset(seen, 0, sizeof seen);
    for (int T : {12, 14}) {
        std::memset(seen, 0, sizeof seen);
        for (int s = 0; s < 16; s++) for (int t = 0; t < 4; t++) for (int sl = 0; sl < 4; sl++) seen[elem(T, s, t, sl)]++;
        for (int e = 0; e < 256; e++) CHECK(seen[e] == 1);
    }
    for (int i = 0; i < 4; i++) CHECK(wperm(wperm(i)) == i);

    const int types[4] = {12, 13, 14, 8};
    for (int ti = 0; ti < 4; ti++) {
        const int T = types[ti], nb = mtile_bytes(T);
        CHECK(nb == 16 * (T == 8 ? 8 * 34 : raw_block_bytes(T)));
        std::memset(cov, 0, sizeof cov);
        for (int r = 0; r < 16; r++) {
            if (T == 12 || T == 13) {
                const bool q5 = T == 13;
                mark_bytes(qk_hdr(r), 16);
                for (int q = 0; q < 128; q++) mark_bytes(qk_qs_byte(q5, r, q), 1);
                if (q5) for (int e = 0; e < 256; e++) mark_bits(q5_bit_byte(r, e), q5_bit_shift(e), 1);
            } else if (T == 14) {
                mark_bytes(q6_d(r), 2);
                mark_bytes(q6_sc(r), 16);
                for (int e = 0; e < 256; e++) {
                    mark_bits(q6_lo_byte(r, e), q6_lo_shift(e), 4);
                    mark_bits(q6_hi_byte(r, e), q6_hi_shift(e), 2);
                }
            } else {
                mark_bytes(q8_d(r), 16);
                for (int e = 0; e < 256; e++) mark_bytes(q8_qs_byte(r, e), 1);
            }
        }
        for (int i = 0; i < nb * 8; i++) CHECK(cov[i] == 1);
    }

    // what the GEMV reads for (step s, lane quad t, slot) of row r is element elem(type, s, t, slot)
    for (int r = 0; r < 16; r++) for (int s = 0; s < 16; s++) for (int t = 0; t < 4; t++) for (int sl = 0; sl < 4; sl++) {
        // Q4_K / Q5_K: word s % 8 of lane t's qs stream, nibble s >= 8, stored position of the slot
        const int e = elem(12, s, t, sl), w = s & 7;
        for (int q5 = 0; q5 < 2; q5++) {
            const int rawq = 32 * (e >> 6) + (e & 31);
            CHECK(qk_qs_byte(q5, r, rawq) == qk_qs(q5, w >> 2, r, t) + 4 * (w & 3) + pos_of_slot(sl));
            CHECK(((e & 63) >= 32) == (s >= 8));
            CHECK((e >> 5) == 2 * t + (s >= 8));  // sub-block of the lane's scale
        }
        // Q5_K bit: word (slot >> 1), bit s (+16 for odd slots), rows g / g+8 in bytes 0-7 / 8-15
        CHECK(q5_bit_byte(r, e) * 8 + q5_bit_shift(e) ==
              (q5_qh(r & 7, t) + 8 * (r >> 3) + 4 * (sl >> 1)) * 8 + ((sl & 1) ? 16 : 0) + s);
        // Q6_K: ql word q6_lo_word(s) (high nibble for steps with bit 2 set), qh word
        // q6_hi_word(s) at bits 2 ((s >> 1) & 3) of the slot's byte; scale = step
        const int e6 = elem(14, s, t, sl);
        const int lw = q6_lo_word(s);
        CHECK(q6_lo_byte(r, e6) == q6_ql(lw >> 2, r, t) + 4 * (lw & 3) + pos_of_slot(sl));
        CHECK(q6_lo_shift(e6) == (((s >> 2) & 1) ? 4 : 0));
        CHECK(q6_hi_byte(r, e6) == q6_qh(r, t) + 4 * q6_hi_word(s) + pos_of_slot(sl));
        CHECK(q6_hi_shift(e6) == 2 * ((s >> 1) & 3));
        CHECK((e6 >> 4) == s);
        // Q8_0: word s of the 64-byte stream, block s / 2
        const int e8 = elem(8, s, t, sl);
        CHECK(q8_qs_byte(r, e8) == q8_qs(s >> 2, r, t) + 4 * (s & 3) + pos_of_slot(sl));
        CHECK((e8 >> 5) == (s >> 1));
    }
    // raw Q6_K parts: every (byte, bits) of ql / qh used once over the block
    std::memset(cov, 0, sizeof cov);
    for (int e = 0; e < 256; e++) {
        mark_bits(q6_raw_lo_byte(e), q6_raw_lo_shift(e), 4);
        mark_bits(q6_raw_hi_byte(e), q6_raw_hi_shift(e), 2);
    }
    for (int i = 0; i < 192 * 8; i++) CHECK(cov[i] == 1);
    // 16-byte pieces of one (p, row) across the 32 lanes of a warp are consecutive
    for (int g = 0; g < 8; g++) for (int t = 0; t < 4; t++) {
        CHECK(qk_qs(false, 1, g, t) == qk_qs(false, 1, 0, 0) + 16 * (4 * g + t));
        CHECK(q6_ql(0, g, t) == q6_ql(0, 0, 0) + 16 * (4 * g + t));
        CHECK(q6_qh(g, t) == q6_qh(0, 0) + 16 * (4 * g + t));
        CHECK(q8_qs(2, g, t) == q8_qs(2, 0, 0) + 16 * (4 * g + t));
        CHECK(q5_qh(g, t) == q5_qh(0, 0) + 16 * (4 * g + t));
    }
    std::printf(fails ? "FAILED %d\n" : "OK\n", fails);
    return fails != 0;
}
"""


def test_tile_maps_exhaustive():
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "chk.cpp")
        exe = os.path.join(d, "chk")
        open(src, "w").write(CHECKER)
        r = subprocess.run(["g++", "-std=c++17", "-O1", "-I", CSRC, src, "-o", exe],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        r = subprocess.run([exe], capture_output=True, text=True)
        assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout
