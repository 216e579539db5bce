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

int main() {
    const int types[4] = {12, 13, 14, 8};
    for (int ti = 0; ti < 4; ti++) {
        int T = types[ti];
        // element map: every (s, t, slot) hits each element of the unit once
        int seen[256]; std::memset(seen, 0, sizeof seen);
        for (int s = 0; s < 16; s++) for (int t = 0; t < 4; t++) for (int sl = 0; sl < 4; sl++) {
            int e = elem_of(T, s, t, sl);
            CHECK(e >= 0 && e < 256);
            seen[e]++;
            // holder register is independent of t and given by slot_reg
            CHECK(hreg_of(T, e) == slot_reg(T, s, sl));
            // four t's of one (s, slot) live in distinct holders
            for (int t2 = 0; t2 < t; t2++) CHECK(holder_of(T, elem_of(T, s, t2, sl)) != holder_of(T, e));
        }
        for (int e = 0; e < 256; e++) CHECK(seen[e] == 1);
        // holder bijection
        for (int j = 0; j < 8; j++) for (int r = 0; r < 32; r++) {
            int e = elem_of_holder(T, j, r);
            CHECK(e >= 0 && e < 256 && holder_of(T, e) == j && hreg_of(T, e) == r);
        }
        // holders load runs of 4 (or 16) consecutive elements, 16-byte aligned
        for (int j = 0; j < 8; j++) for (int r = 0; r < 32; r += 4) {
            int e = elem_of_holder(T, j, r);
            CHECK(e % 4 == 0);
            for (int i = 1; i < 4; i++) CHECK(elem_of_holder(T, j, r + i) == e + i);
        }
    }
    // Q4_K / Q5_K: lane quad t reads sub-blocks 2p,2p+1 (c=0) and 4+2p,5+2p (c=1)
    for (int s = 0; s < 16; s++) for (int t = 0; t < 4; t++) for (int sl = 0; sl < 4; sl++) {
        int e = elem_qk(s, t, sl), c = s >> 3, p = t >> 1;
        int sub = e >> 5;
        CHECK(sub == 2 * (2 * c + p) + ((sl & 2) ? 1 : 0));
        // the byte holding e in the raw block sits in lane t's qs piece of chunk c
        int lq = e & 31, j4 = e >> 6;  // raw qs byte = 32*j4 + l
        int byte = 32 * j4 + lq;
        CHECK(byte >= 64 * c + 16 * t && byte < 64 * c + 16 * t + 16);
    }
    // min-MMA sub-blocks: the 4 lane quads x 2 k-rows cover sub-blocks 0..7 once
    int ms[8] = {0};
    for (int t = 0; t < 4; t++) for (int kr = 0; kr < 2; kr++) ms[minsub_qk(t, kr)]++;
    for (int i = 0; i < 8; i++) CHECK(ms[i] == 1);
    // M-tile byte maps: pieces cover the tile exactly once
    const int T2[4] = {12, 13, 14, 8};
    for (int ti = 0; ti < 4; ti++) {
        int T = T2[ti], nb = mtile_bytes(T);
        static int cov[8192]; std::memset(cov, 0, sizeof cov);
        auto mark = [&](int off, int n) { for (int i = 0; i < n; i++) cov[off + i]++; };
        for (int r = 0; r < 16; r++) {
            if (T == 12 || T == 13) {
                mark(qk_hdr(r), 16);
                if (T == 13) for (int h = 0; h < 2; h++) mark(q5_qh(r, h), 16);
                for (int c = 0; c < 2; c++) for (int t = 0; t < 4; t++) mark(qk_qs(T == 13, c, r, t), 16);
            } else if (T == 14) {
                mark(q6_d(r), 2); mark(q6_sc(r), 16);
                for (int h = 0; h < 2; h++) for (int t = 0; t < 4; t++) mark(q6_ql(h, r, t), 16);
                for (int t = 0; t < 4; t++) mark(q6_qh(r, t), 16);
            } else {
                mark(q8_d(r), 16);
                for (int q = 0; q < 4; q++) for (int t = 0; t < 4; t++) mark(q8_qs(q, r, t), 16);
            }
        }
        for (int i = 0; i < nb; i++) CHECK(cov[i] == 1);
        CHECK(nb == 16 * (T == 8 ? 8 * 34 : raw_block_bytes(T)));
        CHECK(nb % 16 == 0);
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
