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
using namespace ifr;
static int fails = 0;
#define CHECK(c) do { if (!(c)) { std::printf("FAIL %s line %d\n", #c, __LINE__); fails++; } } while (0)

static int cov[4352];
static void mark(int byte, int n) { for (int i = 0; i < n; i++) cov[byte + i]++; }

int main() {
    // element maps cover a unit once
    int seen[256];
    std::memset(seen, 0, sizeof seen);
    for (int c = 0; c < 8; c++) for (int t = 0; t < 4; t++) for (int j = 0; j < 8; j++) seen[elem_k(c, t, j)]++;
    for (int e = 0; e < 256; e++) CHECK(seen[e] == 1);
    std::memset(seen, 0, sizeof seen);
    for (int s = 0; s < 16; s++) for (int t = 0; t < 4; t++) for (int j = 0; j < 4; j++) seen[elem_s(s, t, j)]++;
    for (int e = 0; e < 256; e++) CHECK(seen[e] == 1);
    // a step is half a chunk: the fp16 step s = 2c + h covers the k32 chunk c's word h
    for (int c = 0; c < 8; c++) for (int t = 0; t < 4; t++) for (int j = 0; j < 8; j++)
        CHECK(elem_k(c, t, j) == elem_s(2 * c + (j >> 2), t, j & 3));

    // every byte of each M-tile written once by the repack maps
    const int types[4] = {12, 13, 14, 8};
    for (int ti = 0; ti < 4; ti++) {
        const int T = types[ti], nb = mtile_bytes(T);
        CHECK(nb == 16 * (T == 8 ? 8 * 34 : raw_block_bytes(T)));
        std::memset(cov, 0, sizeof cov);
        for (int r = 0; r < 16; r++) {
            if (T == 12 || T == 13) {
                mark(qk_hdr(r), 16);
                for (int q = 0; q < 128; q++) mark(qk_qs_byte(T == 13, r, q), 1);
                if (T == 13) for (int l = 0; l < 32; l++) mark(q5_qh_byte(r, l), 1);
            } else if (T == 14) {
                mark(q6_d(r), 2);
                mark(q6_sc(r), 16);
                for (int q = 0; q < 128; q++) mark(q6_ql_byte(r, q), 1);
                for (int h = 0; h < 64; h++) mark(q6_qh_byte(r, h), 1);
            } else {
                mark(q8_d(r), 16);
                for (int e = 0; e < 256; e++) mark(q8_qs_byte(r, e), 1);
            }
        }
        for (int i = 0; i < nb; i++) CHECK(cov[i] == 1);
    }

    // what the integer GEMV reads for chunk c, lane quad t, slot j of row r is element elem_k(c, t, j)
    for (int r = 0; r < 16; r++) for (int c = 0; c < 8; c++) for (int t = 0; t < 4; t++) for (int j = 0; j < 8; j++) {
        const int e = elem_k(c, t, j), h = j >> 2, i = j & 3;
        // Q4_K / Q5_K: piece c/4, word 2 ((c/2) % 2) + h, byte i; nibble c % 2
        const int p = c >> 1;
        for (int q5 = 0; q5 < 2; q5++)
            CHECK(qk_qs_byte(q5, r, 32 * (e >> 6) + (e & 31)) == qk_qs(q5, p >> 1, r, t) + 4 * (2 * (p & 1) + h) + i);
        CHECK(((e >> 5) & 1) == (c & 1));  // high nibble for odd chunks
        CHECK((e >> 5) == c);              // sub-block = chunk
        // Q5_K bit c of qh byte e % 32: row word h (rows g, g+8 in bytes 0-7, 8-15)
        CHECK(q5_qh_byte(r, e & 31) == q5_qh(r & 7, t) + 8 * (r >> 3) + 4 * h + i);
        // Q6_K: chunk c = 4n + qq; ql word (qq % 2, h) of piece n, nibble qq / 2; qh word (n, h), bits 2qq
        const int n = c >> 2, qq = c & 3;
        CHECK(q6_ql_byte(r, q6_raw_lo_byte(e)) == q6_ql(n, r, t) + 4 * (2 * (qq & 1) + h) + i);
        CHECK(q6_raw_lo_shift(e) == 4 * (qq >> 1));
        CHECK(q6_qh_byte(r, q6_raw_hi_byte(e) - 128) == q6_qh(r, t) + 4 * (2 * n + h) + i);
        CHECK(q6_raw_hi_shift(e) == 2 * qq);
        CHECK((e >> 4) == 2 * c + h);  // scale group = k16 step
    }
    // Q8_0 (fp16 path): word s of the lane stream, byte j
    for (int r = 0; r < 16; r++) for (int s = 0; s < 16; s++) for (int t = 0; t < 4; t++) for (int j = 0; j < 4; j++) {
        const int e = elem_s(s, t, j);
        CHECK(q8_qs_byte(r, e) == q8_qs(s >> 2, r, t) + 4 * (s & 3) + j);
        CHECK((e >> 5) == (s >> 1));
    }
    // raw Q6_K parts: every (byte, bits) of ql / qh used once over the block
    static int bits[192 * 8];
    std::memset(bits, 0, sizeof bits);
    for (int e = 0; e < 256; e++) {
        for (int i = 0; i < 4; i++) bits[q6_raw_lo_byte(e) * 8 + q6_raw_lo_shift(e) + i]++;
        for (int i = 0; i < 2; i++) bits[q6_raw_hi_byte(e) * 8 + q6_raw_hi_shift(e) + i]++;
    }
    for (int i = 0; i < 192 * 8; i++) CHECK(bits[i] == 1);
    // 16-byte pieces of one (piece, row) across the 32 lanes of a warp are consecutive
    for (int g = 0; g < 8; g++) for (int t = 0; t < 4; t++) {
        CHECK(qk_qs(false, 1, g, t) == qk_qs(false, 1, 0, 0) + 16 * (4 * g + t));
        CHECK(q6_ql(1, g, t) == q6_ql(1, 0, 0) + 16 * (4 * g + t));
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
