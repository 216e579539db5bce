// Host-side quantizer: f32 rows -> GGUF Q4_K / Q5_K / Q6_K / Q8_0 blocks.
//
// The reference ships no K-quant encoder (it only reads GGUF files); this
// one produces the seeded synthetic models and lets a caller quantize f32
// weights at load time.  Scheme (per 256-element super-block):
//   Q4_K/Q5_K: each 32-element sub-block is fitted as scale*q - min with
//     min = -min(0, x) and scale = (max - min_x)/levels; the 8 scales and 8
//     mins are quantized to 6 bits against f16 super-scales d = max/63,
//     dmin = max/63, then q = round((x + dmin*m)/(d*sc)).
//   Q6_K: 16 groups of 16, signed scale so the extreme maps to -32, int8
//     group scales against d = max|scale|/127.
//   Q8_0: d = max|x|/127 per 32, q = round(x/d).
// Block byte layouts are GGML's (src/kernels/quant_kernels.c:25-62 of the
// reference).  Rows are split over hardware threads.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

uint16_t f32_to_f16(float x) {
    uint32_t f;
    std::memcpy(&f, &x, 4);
    const uint32_t sign = (f >> 16) & 0x8000u, ax = f & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return (uint16_t)sign;
        const uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u;
        const int shift = 126 - (int)e;
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = (((ax >> 23) - 112) << 10) | ((ax & 0x7fffffu) >> 13);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, f;
    if (e == 0) {
        if (m == 0) {
            f = sign;
        } else {
            int sh = 0;
            while (!(m & 0x400)) { m <<= 1; sh++; }
            f = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 0x1f) {
        f = sign | 0x7f800000u | (m << 13);
    } else {
        f = sign | ((e + 112) << 23) | (m << 13);
    }
    float r;
    std::memcpy(&r, &f, 4);
    return r;
}

inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
inline void put16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)(v & 0xff); p[1] = (uint8_t)(v >> 8); }

void affine_superblock(const float *x, int levels, uint8_t *hdr, int *q) {
    float scale[8], mn[8], maxs = 0.f, maxm = 0.f;
    for (int j = 0; j < 8; j++) {
        float lo = 0.f, hi = -INFINITY;
        for (int i = 0; i < 32; i++) {
            lo = std::fmin(lo, x[32 * j + i]);
            hi = std::fmax(hi, x[32 * j + i]);
        }
        if (hi < lo) hi = lo;
        scale[j] = (hi - lo) / (float)levels;
        mn[j] = -lo;
        maxs = std::fmax(maxs, scale[j]);
        maxm = std::fmax(maxm, mn[j]);
    }
    const uint16_t dh = f32_to_f16(maxs / 63.f), mh = f32_to_f16(maxm / 63.f);
    const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = d > 0 ? clampi((int)std::lrint(scale[j] / d), 0, 63) : 0;
        m[j] = dmin > 0 ? clampi((int)std::lrint(mn[j] / dmin), 0, 63) : 0;
        const float ds = d * (float)sc[j], dm = dmin * (float)m[j];
        for (int i = 0; i < 32; i++)
            q[32 * j + i] = ds > 0 ? clampi((int)std::lrint((x[32 * j + i] + dm) / ds), 0, levels) : 0;
    }
    put16(hdr, dh);
    put16(hdr + 2, mh);
    uint8_t *s = hdr + 4;
    std::memset(s, 0, 12);
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)(sc[j] & 63);
        s[j + 4] = (uint8_t)(m[j] & 63);
    }
    for (int j = 4; j < 8; j++) {
        s[j + 4] = (uint8_t)((sc[j] & 15) | ((m[j] & 15) << 4));
        s[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
        s[j] |= (uint8_t)((m[j] >> 4) << 6);
    }
}

void enc_q4k(const float *x, uint8_t *b) {
    int q[256];
    affine_superblock(x, 15, b, q);
    for (int j = 0; j < 4; j++)
        for (int l = 0; l < 32; l++) b[16 + 32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
}

void enc_q5k(const float *x, uint8_t *b) {
    int q[256];
    affine_superblock(x, 31, b, q);
    uint8_t *qh = b + 16, *qs = b + 48;
    std::memset(qh, 0, 32);
    for (int j = 0; j < 4; j++)
        for (int l = 0; l < 32; l++) {
            const int a = q[64 * j + l], c = q[64 * j + 32 + l];
            qs[32 * j + l] = (uint8_t)((a & 15) | ((c & 15) << 4));
            qh[l] |= (uint8_t)(((a >> 4) << (2 * j)) | ((c >> 4) << (2 * j + 1)));
        }
}

void enc_q6k(const float *x, uint8_t *b) {
    float gs[16], maxs = 0.f;
    for (int g = 0; g < 16; g++) {
        float amax = 0.f, sv = 0.f;
        for (int i = 0; i < 16; i++)
            if (std::fabs(x[16 * g + i]) > amax) { amax = std::fabs(x[16 * g + i]); sv = x[16 * g + i]; }
        gs[g] = -sv / 32.f;
        maxs = std::fmax(maxs, std::fabs(gs[g]));
    }
    const uint16_t dh = f32_to_f16(maxs / 127.f);
    const float d = f16_to_f32(dh);
    int8_t sc[16];
    int q[256];
    for (int g = 0; g < 16; g++) {
        sc[g] = (int8_t)(d > 0 ? clampi((int)std::lrint(gs[g] / d), -128, 127) : 0);
        const float ds = d * (float)sc[g];
        for (int i = 0; i < 16; i++)
            q[16 * g + i] = clampi(ds != 0 ? (int)std::lrint(x[16 * g + i] / ds) : 0, -32, 31) + 32;
    }
    uint8_t *ql = b, *qh = b + 128;
    std::memset(qh, 0, 64);
    for (int n = 0; n < 2; n++)
        for (int l = 0; l < 32; l++) {
            const int q1 = q[128 * n + l], q2 = q[128 * n + 32 + l], q3 = q[128 * n + 64 + l], q4 = q[128 * n + 96 + l];
            ql[64 * n + l] = (uint8_t)((q1 & 15) | ((q3 & 15) << 4));
            ql[64 * n + 32 + l] = (uint8_t)((q2 & 15) | ((q4 & 15) << 4));
            qh[32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    std::memcpy(b + 192, sc, 16);
    put16(b + 208, dh);
}

void enc_q80(const float *x, uint8_t *b) {
    float amax = 0.f;
    for (int i = 0; i < 32; i++) amax = std::fmax(amax, std::fabs(x[i]));
    const uint16_t dh = f32_to_f16(amax / 127.f);
    const float d = f16_to_f32(dh);
    put16(b, dh);
    for (int i = 0; i < 32; i++) b[2 + i] = (uint8_t)(int8_t)(d > 0 ? clampi((int)std::lrint(x[i] / d), -127, 127) : 0);
}

}  // namespace

namespace ifr {

// returns 0 on success, -1 for an unsupported type or cols
int quantize_host(int type, const float *x, int64_t rows, int64_t cols, uint8_t *out) {
    const int be = type == 8 ? 32 : 256;
    const int bb = type == 12 ? 144 : type == 13 ? 176 : type == 14 ? 210 : type == 8 ? 34 : 0;
    if (bb == 0 || cols % be || rows < 0) return -1;
    const int64_t nb = cols / be, rb = nb * bb;
    auto work = [&](int64_t r0, int64_t r1) {
        for (int64_t r = r0; r < r1; r++)
            for (int64_t b = 0; b < nb; b++) {
                const float *xs = x + r * cols + b * be;
                uint8_t *o = out + r * rb + b * bb;
                if (type == 12) enc_q4k(xs, o);
                else if (type == 13) enc_q5k(xs, o);
                else if (type == 14) enc_q6k(xs, o);
                else enc_q80(xs, o);
            }
    };
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 1;
    if (nt > 32) nt = 32;
    if (rows * cols < (1 << 16)) nt = 1;
    std::vector<std::thread> th;
    for (unsigned i = 0; i < nt; i++) {
        const int64_t r0 = rows * i / nt, r1 = rows * (i + 1) / nt;
        if (r1 > r0) th.emplace_back(work, r0, r1);
    }
    for (auto &t : th) t.join();
    return 0;
}

}  // namespace ifr
