// Verify-step engine: GGUF model loading, generation state and the
// speculative-decoding step (MTP draft -> K+1-column verify -> greedy accept
// -> commit), all enqueued on the context's stream.
//
// Reference: Inferno.jl src/GGUF.jl:119-165 (file format), src/LoaderCPU.jl
// (tensor names :471-694, config keys :439-469), src/ModelCPU.jl:976-1020
// (forward), :2099-2115 (greedy verify), src/SpeculativeDecoding.jl (loop).
#include "../../include/inferno_b200.h"
#include "comm.h"
#include "common.cuh"
#include "model.cuh"
#include "fused.cuh"
#include "dequant.cuh"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <string>
#include <vector>

// error reporting shared with api.cu
int ifr_fail(int code, const char *fmt, ...);
int ifr_cuda_fail(cudaError_t e, const char *what);
int ifr_ctx_device(const ifr_ctx *c);
int ifr_ctx_activation(const ifr_ctx *c);
int ifr_ctx_dense_min(const ifr_ctx *c);
int ifr_ctx_prefill_dense(const ifr_ctx *c);
int ifr_ctx_fused_layers(const ifr_ctx *c);
int ifr_ctx_dense_f16(const ifr_ctx *c);
int ifr_ctx_kv_bf16(const ifr_ctx *c);
void ifr_ctx_retain(ifr_ctx *c);
void ifr_ctx_release(ifr_ctx *c);
cudaStream_t ifr_ctx_stream_of(const ifr_ctx *c);
int ifr_upload_raw(ifr_ctx *c, int type, const void *host, int64_t rows, int64_t cols, ifr::QTensor *out);

#define ECHECK(expr, what)                                  \
    do {                                                    \
        cudaError_t _e = (expr);                            \
        if (_e != cudaSuccess) return ifr_cuda_fail(_e, what); \
    } while (0)

namespace {

// ------------------------------------------------------------------ GGUF ----
struct GTensor {
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
    int64_t nel() const {
        int64_t n = 1;
        for (auto d : dims) n *= (int64_t)d;
        return n;
    }
};

struct Gguf {
    int fd = -1;
    uint8_t *map = nullptr;
    size_t size = 0;
    uint64_t data_off = 0;
    std::map<std::string, double> num;
    std::map<std::string, std::string> str;
    std::map<std::string, GTensor> t;

    ~Gguf() {
        if (map) munmap(map, size);
        if (fd >= 0) close(fd);
    }

    bool open_file(const char *path, std::string &err) {
        fd = ::open(path, O_RDONLY);
        if (fd < 0) { err = std::string("cannot open ") + path; return false; }
        struct stat st;
        if (fstat(fd, &st) != 0) { err = "fstat failed"; return false; }
        size = (size_t)st.st_size;
        map = (uint8_t *)mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (map == MAP_FAILED) { map = nullptr; err = "mmap failed"; return false; }
        size_t p = 0;
        auto need = [&](size_t n) { return p + n <= size; };
        auto rd = [&](void *dst, size_t n) -> bool {
            if (!need(n)) return false;
            memcpy(dst, map + p, n);
            p += n;
            return true;
        };
        auto rd_str = [&](std::string &s) -> bool {
            uint64_t n;
            if (!rd(&n, 8) || n > (1u << 20) || !need(n)) return false;  // GGUF.jl:96-99
            s.assign((const char *)map + p, n);
            p += n;
            return true;
        };
        const size_t scal[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        std::function<bool(uint32_t, const std::string &, bool)> rd_val;
        rd_val = [&](uint32_t ty, const std::string &key, bool keep) -> bool {
            if (ty == 8) {
                std::string s;
                if (!rd_str(s)) return false;
                if (keep) str[key] = s;
                return true;
            }
            if (ty == 9) {
                uint32_t at;
                uint64_t n;
                if (!rd(&at, 4) || !rd(&n, 8)) return false;
                for (uint64_t i = 0; i < n; i++)
                    if (!rd_val(at, key, false)) return false;
                return true;
            }
            if (ty > 12) return false;
            uint8_t b[8] = {0};
            if (!rd(b, scal[ty])) return false;
            double v = 0;
            switch (ty) {
            case 0: v = *(uint8_t *)b; break;
            case 1: v = *(int8_t *)b; break;
            case 2: v = *(uint16_t *)b; break;
            case 3: v = *(int16_t *)b; break;
            case 4: v = *(uint32_t *)b; break;
            case 5: v = *(int32_t *)b; break;
            case 6: v = *(float *)b; break;
            case 7: v = b[0] ? 1 : 0; break;
            case 10: v = (double)*(uint64_t *)b; break;
            case 11: v = (double)*(int64_t *)b; break;
            case 12: v = *(double *)b; break;
            }
            if (keep) num[key] = v;
            return true;
        };
        uint32_t magic, version;
        uint64_t nt, nkv;
        if (!rd(&magic, 4) || magic != 0x46554747u) { err = "Not a valid GGUF file"; return false; }
        if (!rd(&version, 4) || !rd(&nt, 8) || !rd(&nkv, 8)) { err = "truncated header"; return false; }
        for (uint64_t i = 0; i < nkv; i++) {
            std::string k;
            uint32_t ty;
            if (!rd_str(k) || !rd(&ty, 4) || !rd_val(ty, k, true)) { err = "bad metadata"; return false; }
        }
        for (uint64_t i = 0; i < nt; i++) {
            std::string name;
            GTensor g;
            uint32_t nd;
            if (!rd_str(name) || !rd(&nd, 4) || nd > 4) { err = "bad tensor info"; return false; }
            g.dims.resize(nd);
            for (uint32_t d = 0; d < nd; d++)
                if (!rd(&g.dims[d], 8)) { err = "bad tensor info"; return false; }
            if (!rd(&g.type, 4) || !rd(&g.offset, 8)) { err = "bad tensor info"; return false; }
            t[name] = g;
        }
        const uint64_t align = num.count("general.alignment") ? (uint64_t)num["general.alignment"] : 32;
        data_off = (p + align - 1) / align * align;  // GGUF.jl:152-156
        return true;
    }
    const uint8_t *data(const GTensor &g) const { return map + data_off + g.offset; }
    bool has(const std::string &n) const { return t.count(n) != 0; }
};

int64_t tensor_bytes(uint32_t type, int64_t nel) {
    switch (type) {
    case 0: return nel * 4;
    case 1: return nel * 2;
    case 8: return nel / 32 * 34;
    case 12: return nel / 256 * 144;
    case 13: return nel / 256 * 176;
    case 14: return nel / 256 * 210;
    }
    return -1;
}

float h2f_host(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, f;
    if (e == 0) {
        if (m == 0) f = sign;
        else {
            int sh = 0;
            while (!(m & 0x400)) { m <<= 1; sh++; }
            f = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 0x1f) f = sign | 0x7f800000u | (m << 13);
    else f = sign | ((e + 112) << 23) | (m << 13);
    float r;
    memcpy(&r, &f, 4);
    return r;
}

}  // namespace

// A projection: one quantized matrix, or same-K parts of different types whose
// outputs land in consecutive row ranges of one output vector.
struct Proj {
    std::vector<ifr::QTensor> parts;
    int64_t rows = 0, cols = 0;
    bool glu = false;  // gate/up 16-row blocks interleaved in one tensor (SwiGLU epilogue)
};

struct DevLayer {
    bool ssm = false;
    float *attn_norm = nullptr, *post_norm = nullptr;
    Proj proj, out, gate_up, down;
    float *conv_w = nullptr, *ab_w = nullptr, *ssm_a = nullptr, *dt_bias = nullptr, *ssm_norm = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
    // Gemma4 blocks: post_norm follows the attention output, ffn_norm precedes
    // the MLP and post_ffw_norm follows it; layer_scalar [1] scales the layer's
    // output; sliding layers attend within the window
    bool sliding = false;
    float *ffn_norm = nullptr, *post_ffw_norm = nullptr, *layer_scalar = nullptr;
    // Gemma4 per-layer input block: gate (pli x d), projection (d x pli), post norm
    Proj pli_gate, pli_proj;
    float *pli_post_norm = nullptr;
};

struct ifr_model {
    ifr_ctx *ctx = nullptr;
    int states = 0;          // live states built on this model
    bool closing = false;    // ifr_model_free called while states were alive
    ifr_model_info info{};
    int conv_channels = 0, inner = 0;
    std::vector<DevLayer> layers;
    DevLayer mtp_layer;
    bool has_mtp = false;
    Proj embed, lm_head;
    float *final_norm = nullptr, *mtp_norm_e = nullptr, *mtp_norm_h = nullptr, *mtp_norm = nullptr;
    Proj mtp_fc;
    // tensor parallelism: this rank's query / KV heads, FFN width and lm_head rows
    ifr_comm *comm = nullptr;
    int tp_rank = 0, tp_world = 1;
    int nh = 0, nkv = 0, ffn = 0, ffn_off = 0, vocab = 0, vocab_off = 0;
    // Gemma4 blocks (general.architecture "gemma4", src/Gemma4.jl): layer i is
    // full attention iff (i + 1) % sliding_pattern == 0, else sliding-window
    bool gemma = false;
    int window = 0, sliding_pattern = 0;
    float attn_softcap = 0.f, final_softcap = 0.f, embed_scale = 1.f;
    float rope_theta_swa = 10000.f, partial_rotary = 0.25f;
    // Gemma4 per-layer inputs (compute_per_layer_inputs!, Gemma4.jl:459-503):
    // pli values per layer (0: none), the token table (vocab x L pli), the model
    // projection (L pli x d, stored pre-scaled by d^-1/2) and its norm
    int pli = 0;
    Proj pli_token_embd, pli_model_proj;
    float *pli_proj_norm = nullptr;
    std::vector<void *> dev_allocs;
    ~ifr_model() {
        for (void *p : dev_allocs) cudaFree(p);
    }
};

namespace {

constexpr int kNMax = 8;
// one request: split-KV attention from this cache length on (shorter caches use the cluster kernel)
constexpr int kSplitMinCtx = 1024;

int upload_f32(ifr_model *m, const Gguf &g, const std::string &name, int64_t expect, float **out) {
    auto it = g.t.find(name);
    if (it == g.t.end()) return ifr_fail(IFR_ERR_ARG, "tensor %s missing", name.c_str());
    const GTensor &t = it->second;
    if (expect >= 0 && t.nel() != expect)
        return ifr_fail(IFR_ERR_ARG, "tensor %s has %lld elements, expected %lld", name.c_str(), (long long)t.nel(),
                        (long long)expect);
    std::vector<float> host((size_t)t.nel());
    if (t.type == 0) memcpy(host.data(), g.data(t), host.size() * 4);
    else if (t.type == 1) {
        const uint16_t *h = (const uint16_t *)g.data(t);
        for (size_t i = 0; i < host.size(); i++) host[i] = h2f_host(h[i]);
    } else return ifr_fail(IFR_ERR_UNSUPPORTED, "tensor %s: type %u where F32/F16 is expected", name.c_str(), t.type);
    void *d = nullptr;
    ECHECK(cudaMalloc(&d, host.size() * 4), "cudaMalloc(f32 tensor)");
    m->dev_allocs.push_back(d);
    ECHECK(cudaMemcpy(d, host.data(), host.size() * 4, cudaMemcpyHostToDevice), "H2D f32 tensor");
    *out = (float *)d;
    return IFR_OK;
}

// concatenated f32 rows of several [rows][cols] tensors
int upload_f32_cat(ifr_model *m, const Gguf &g, const std::vector<std::string> &names, float **out) {
    std::vector<float> host;
    for (auto &n : names) {
        auto it = g.t.find(n);
        if (it == g.t.end()) return ifr_fail(IFR_ERR_ARG, "tensor %s missing", n.c_str());
        const GTensor &t = it->second;
        const size_t off = host.size();
        host.resize(off + (size_t)t.nel());
        if (t.type == 0) memcpy(host.data() + off, g.data(t), (size_t)t.nel() * 4);
        else if (t.type == 1) {
            const uint16_t *h = (const uint16_t *)g.data(t);
            for (int64_t i = 0; i < t.nel(); i++) host[off + i] = h2f_host(h[i]);
        } else return ifr_fail(IFR_ERR_UNSUPPORTED, "tensor %s: type %u where F32/F16 is expected", n.c_str(), t.type);
    }
    void *d = nullptr;
    ECHECK(cudaMalloc(&d, host.size() * 4), "cudaMalloc(f32 tensor)");
    m->dev_allocs.push_back(d);
    ECHECK(cudaMemcpy(d, host.data(), host.size() * 4, cudaMemcpyHostToDevice), "H2D f32 tensor");
    *out = (float *)d;
    return IFR_OK;
}

// a row range and an inner-dimension range of a quantized matrix (whole by default)
struct Slice {
    int64_t r0 = 0, r1 = -1, k0 = 0, k1 = -1;
};

// raw GGUF bytes of rows [r0, r1) x columns [k0, k1) (k at block boundaries)
int slice_raw(const Gguf &g, const std::string &name, const GTensor &t, const Slice &sl, std::vector<uint8_t> &out,
              int64_t &rows, int64_t &cols) {
    const int64_t C = (int64_t)t.dims[0], R = (int64_t)t.dims[1];
    const int64_t r0 = sl.r0, r1 = sl.r1 < 0 ? R : sl.r1, k0 = sl.k0, k1 = sl.k1 < 0 ? C : sl.k1;
    const int64_t be = t.type == 8 ? 32 : 256, rb = tensor_bytes(t.type, C);
    if (rb <= 0) return ifr_fail(IFR_ERR_UNSUPPORTED, "tensor %s: unsupported type %u", name.c_str(), t.type);
    if (r0 < 0 || r1 > R || r0 >= r1 || k0 < 0 || k1 > C || k0 >= k1 || k0 % be || k1 % be)
        return ifr_fail(IFR_ERR_ARG, "tensor %s: slice rows %lld..%lld cols %lld..%lld does not fit %lldx%lld blocks of %lld",
                        name.c_str(), (long long)r0, (long long)r1, (long long)k0, (long long)k1, (long long)R,
                        (long long)C, (long long)be);
    const int64_t bb = rb / (C / be);  // bytes per block
    const int64_t off = k0 / be * bb, len = (k1 - k0) / be * bb;
    out.resize((size_t)((r1 - r0) * len));
    const uint8_t *src = g.data(t);
    for (int64_t r = r0; r < r1; r++) memcpy(out.data() + (r - r0) * len, src + r * rb + off, (size_t)len);
    rows = r1 - r0;
    cols = k1 - k0;
    return IFR_OK;
}

// quantized matrices with the same inner dim, stacked along rows; parts of the
// same type are merged into one device tensor (one GEMV launch); `slices`
// (optional, one per name) take a shard of each matrix
int upload_proj(ifr_model *m, const Gguf &g, const std::vector<std::string> &names, Proj *p,
                const std::vector<Slice> &slices = {}) {
    p->parts.clear();
    p->rows = 0;
    p->cols = -1;
    size_t i = 0;
    while (i < names.size()) {
        auto it = g.t.find(names[i]);
        if (it == g.t.end()) return ifr_fail(IFR_ERR_ARG, "tensor %s missing", names[i].c_str());
        const GTensor &t0 = it->second;
        if (t0.dims.size() != 2) return ifr_fail(IFR_ERR_ARG, "tensor %s is not a matrix", names[i].c_str());
        const Slice s0 = i < slices.size() ? slices[i] : Slice();
        const int64_t cols = (s0.k1 < 0 ? (int64_t)t0.dims[0] : s0.k1) - s0.k0;
        if (p->cols >= 0 && cols != p->cols) return ifr_fail(IFR_ERR_ARG, "tensor %s: inner dim mismatch", names[i].c_str());
        p->cols = cols;
        std::vector<uint8_t> raw;
        int64_t rows = 0;
        size_t j = i;
        for (; j < names.size(); j++) {
            auto jt = g.t.find(names[j]);
            if (jt == g.t.end()) return ifr_fail(IFR_ERR_ARG, "tensor %s missing", names[j].c_str());
            const GTensor &tj = jt->second;
            const Slice sj = j < slices.size() ? slices[j] : Slice();
            const int64_t cj = (sj.k1 < 0 ? (int64_t)tj.dims[0] : sj.k1) - sj.k0;
            if (tj.type != t0.type || tj.dims.size() != 2 || cj != cols) break;
            std::vector<uint8_t> part;
            int64_t pr = 0, pc = 0;
            int rc = slice_raw(g, names[j], tj, sj, part, pr, pc);
            if (rc) return rc;
            raw.insert(raw.end(), part.begin(), part.end());
            rows += pr;
        }
        ifr::QTensor q{};
        int rc = ifr_upload_raw(m->ctx, (int)t0.type, raw.data(), rows, cols, &q);
        if (rc) return rc;
        m->dev_allocs.push_back(q.data);
        p->parts.push_back(q);
        p->rows += rows;
        i = j;
    }
    return IFR_OK;
}

// ffn_gate and ffn_up as one tensor with their 16-row blocks interleaved, so
// that the GEMV can form silu(gate) * up in its epilogue; falls back to the
// plain stack when the two differ in type or shape
int upload_gate_up(ifr_model *m, const Gguf &g, const std::string &gate, const std::string &up, Proj *p,
                   const Slice &sl = Slice()) {
    auto gi = g.t.find(gate), ui = g.t.find(up);
    if (gi == g.t.end() || ui == g.t.end()) return upload_proj(m, g, {gate, up}, p, {sl, sl});
    const GTensor &tg = gi->second, &tu = ui->second;
    const int64_t r0 = sl.r0, r1 = sl.r1 < 0 ? (int64_t)tg.dims[1] : sl.r1;
    if (tg.type != tu.type || tg.dims.size() != 2 || tu.dims.size() != 2 || tg.dims[0] != tu.dims[0] ||
        tg.dims[1] != tu.dims[1] || (r1 - r0) % 16 || sl.k0 != 0 || sl.k1 >= 0)
        return upload_proj(m, g, {gate, up}, p, {sl, sl});
    std::vector<uint8_t> sg, su;
    int64_t rows = 0, cols = 0;
    int rc = slice_raw(g, gate, tg, sl, sg, rows, cols);
    if (!rc) rc = slice_raw(g, up, tu, sl, su, rows, cols);
    if (rc) return rc;
    const int64_t nb = (int64_t)sg.size();
    const int64_t rb = nb / rows;
    std::vector<uint8_t> raw((size_t)nb * 2);
    const uint8_t *pg = sg.data(), *pu = su.data();
    for (int64_t b = 0; b < rows / 16; b++) {
        memcpy(raw.data() + (2 * b) * 16 * rb, pg + b * 16 * rb, (size_t)(16 * rb));
        memcpy(raw.data() + (2 * b + 1) * 16 * rb, pu + b * 16 * rb, (size_t)(16 * rb));
    }
    ifr::QTensor q{};
    rc = ifr_upload_raw(m->ctx, (int)tg.type, raw.data(), 2 * rows, cols, &q);
    if (rc) return rc;
    m->dev_allocs.push_back(q.data);
    p->parts.assign(1, q);
    p->rows = 2 * rows;
    p->cols = cols;
    p->glu = true;
    return IFR_OK;
}

int load_layer(ifr_model *m, const Gguf &g, const std::string &pre, DevLayer &L, int li = -1) {
    const ifr_model_info &c = m->info;
    int rc;
    L.ssm = g.has(pre + "ssm_a");
    if (m->gemma) {
        // attention-only Gemma4 layer (Gemma4Loader.jl:180-260): q rows nh x hd
        // (no gate), four norms, the layer scalar
        if (L.ssm) return ifr_fail(IFR_ERR_UNSUPPORTED, "%s: gemma4 layers are attention layers", pre.c_str());
        L.sliding = m->sliding_pattern <= 0 || (li + 1) % m->sliding_pattern != 0;
        const int64_t hd = c.head_dim, h0 = (int64_t)m->tp_rank * m->nh, kv0 = (int64_t)m->tp_rank * m->nkv;
        Slice sq, sk, so;
        sq.r0 = h0 * hd;
        sq.r1 = (h0 + m->nh) * hd;
        sk.r0 = kv0 * hd;
        sk.r1 = (kv0 + m->nkv) * hd;
        so.k0 = h0 * hd;
        so.k1 = (h0 + m->nh) * hd;
        if ((rc = upload_f32(m, g, pre + "attn_norm.weight", c.hidden, &L.attn_norm))) return rc;
        if ((rc = upload_f32(m, g, pre + "post_attention_norm.weight", c.hidden, &L.post_norm))) return rc;
        if ((rc = upload_f32(m, g, pre + "ffn_norm.weight", c.hidden, &L.ffn_norm))) return rc;
        if ((rc = upload_f32(m, g, pre + "post_ffw_norm.weight", c.hidden, &L.post_ffw_norm))) return rc;
        if (g.has(pre + "layer_scalar") && (rc = upload_f32(m, g, pre + "layer_scalar", 1, &L.layer_scalar)))
            return rc;
        if ((rc = upload_proj(m, g, {pre + "attn_q.weight", pre + "attn_k.weight", pre + "attn_v.weight"}, &L.proj,
                              {sq, sk, sk})))
            return rc;
        if ((rc = upload_proj(m, g, {pre + "attn_output.weight"}, &L.out, {so}))) return rc;
        if ((rc = upload_f32(m, g, pre + "attn_q_norm.weight", c.head_dim, &L.q_norm))) return rc;
        if ((rc = upload_f32(m, g, pre + "attn_k_norm.weight", c.head_dim, &L.k_norm))) return rc;
        if (L.proj.rows != (int64_t)(m->nh + 2 * m->nkv) * c.head_dim)
            return ifr_fail(IFR_ERR_ARG, "%s: attention projection shapes do not match the config", pre.c_str());
        Slice sf, sd;
        sf.r0 = sd.k0 = m->ffn_off;
        sf.r1 = sd.k1 = m->ffn_off + m->ffn;
        if ((rc = upload_gate_up(m, g, pre + "ffn_gate.weight", pre + "ffn_up.weight", &L.gate_up, sf))) return rc;
        if (!L.gate_up.glu)
            return ifr_fail(IFR_ERR_UNSUPPORTED, "%s: gemma4 gate/up must share a type and 16-row blocks", pre.c_str());
        if ((rc = upload_proj(m, g, {pre + "ffn_down.weight"}, &L.down, {sd}))) return rc;
        if (m->pli) {
            // per-layer input block (Gemma4Loader.jl:230-239), whole on every rank
            if ((rc = upload_proj(m, g, {pre + "pli_gate.weight"}, &L.pli_gate))) return rc;
            if ((rc = upload_proj(m, g, {pre + "pli_proj.weight"}, &L.pli_proj))) return rc;
            if ((rc = upload_f32(m, g, pre + "pli_post_norm.weight", c.hidden, &L.pli_post_norm))) return rc;
            if (L.pli_gate.rows != m->pli || L.pli_gate.cols != c.hidden || L.pli_proj.rows != c.hidden ||
                L.pli_proj.cols != m->pli)
                return ifr_fail(IFR_ERR_ARG, "%s: per-layer input shapes do not match the config", pre.c_str());
        }
        return IFR_OK;
    }
    if ((rc = upload_f32(m, g, pre + "attn_norm.weight", c.hidden, &L.attn_norm))) return rc;
    if ((rc = upload_f32(m, g, pre + "post_attention_norm.weight", c.hidden, &L.post_norm))) return rc;
    if (L.ssm) {
        if ((rc = upload_proj(m, g, {pre + "attn_qkv.weight", pre + "attn_gate.weight"}, &L.proj))) return rc;
        if ((rc = upload_proj(m, g, {pre + "ssm_out.weight"}, &L.out))) return rc;
        if ((rc = upload_f32(m, g, pre + "ssm_conv1d.weight", (int64_t)m->conv_channels * c.conv_kernel, &L.conv_w))) return rc;
        if ((rc = upload_f32_cat(m, g, {pre + "ssm_alpha.weight", pre + "ssm_beta.weight"}, &L.ab_w))) return rc;
        if ((rc = upload_f32(m, g, pre + "ssm_a", c.ssm_heads, &L.ssm_a))) return rc;
        if ((rc = upload_f32(m, g, pre + "ssm_dt.bias", c.ssm_heads, &L.dt_bias))) return rc;
        if ((rc = upload_f32(m, g, pre + "ssm_norm.weight", c.ssm_head_dim, &L.ssm_norm))) return rc;
        if (L.proj.rows != m->conv_channels + m->inner || L.out.cols != m->inner)
            return ifr_fail(IFR_ERR_ARG, "%s: SSM projection shapes do not match the config", pre.c_str());
    } else {
        // this rank's heads: q rows [q; gate] per head, k / v rows per KV head, the
        // output projection's inner range of those heads (the whole model for one rank)
        const int64_t hd = c.head_dim, h0 = (int64_t)m->tp_rank * m->nh, kv0 = (int64_t)m->tp_rank * m->nkv;
        Slice sq, sk, so;
        sq.r0 = h0 * 2 * hd;
        sq.r1 = (h0 + m->nh) * 2 * hd;
        sk.r0 = kv0 * hd;
        sk.r1 = (kv0 + m->nkv) * hd;
        so.k0 = h0 * hd;
        so.k1 = (h0 + m->nh) * hd;
        if ((rc = upload_proj(m, g, {pre + "attn_q.weight", pre + "attn_k.weight", pre + "attn_v.weight"}, &L.proj,
                              {sq, sk, sk})))
            return rc;
        if ((rc = upload_proj(m, g, {pre + "attn_output.weight"}, &L.out, {so}))) return rc;
        if ((rc = upload_f32(m, g, pre + "attn_q_norm.weight", c.head_dim, &L.q_norm))) return rc;
        if ((rc = upload_f32(m, g, pre + "attn_k_norm.weight", c.head_dim, &L.k_norm))) return rc;
        if (L.proj.rows != (int64_t)(2 * m->nh + 2 * m->nkv) * c.head_dim)
            return ifr_fail(IFR_ERR_ARG, "%s: attention projection shapes do not match the config", pre.c_str());
    }
    // this rank's FFN units: gate / up rows and the down projection's inner range
    Slice sf, sd;
    sf.r0 = sd.k0 = m->ffn_off;
    sf.r1 = sd.k1 = m->ffn_off + m->ffn;
    if ((rc = upload_gate_up(m, g, pre + "ffn_gate.weight", pre + "ffn_up.weight", &L.gate_up, sf))) return rc;
    if ((rc = upload_proj(m, g, {pre + "ffn_down.weight"}, &L.down, {sd}))) return rc;
    return IFR_OK;
}

}  // namespace
namespace {
int64_t proj_bytes(const Proj &p) {
    int64_t b = 0;
    for (auto &q : p.parts) b += ifr::raw_row_bytes(q.type, q.cols) * q.rows;
    return b;
}

}  // namespace

// ------------------------------------------------------------- state --------
// B requests share the model and advance together; request b's verify tokens
// are vtok[b * kNMax ..], its scalars sc[b], its caches offset by b per-request
// strides; a call with n tokens per request uses activation columns b * n + t.
struct ifr_state {
    ifr_model *m = nullptr;
    int B = 1;
    int max_ctx = 0, log_cap = 0;
    std::vector<void *> allocs;
    ifr::EngineScalars *sc = nullptr;   // device
    int32_t *vtok = nullptr, *acc = nullptr, *outtok = nullptr, *log = nullptr, *mtp_pos = nullptr;
    int32_t *h_tok = nullptr;           // pinned staging
    int32_t *chunk_pos = nullptr;       // prefill chunk: positions of its 8-token attention sub-calls
    int32_t *prompt = nullptr;          // device copy of the prompts being prefilled [B][max_ctx]
    float *x, *xn, *proj, *y, *gu, *hmid, *hid, *logits;
    float *mtp_h, *mtp_cat;
    float *cand = nullptr;              // tensor parallel: per-row (max, argmax) of every rank
    unsigned *gcount = nullptr;         // fused argmax/accept: per-launch completion counter (returns to 0)
    unsigned long long *am_cand = nullptr;  // lm_head GEMV epilogue argmax: per-CTA candidates [8][1024]
    unsigned *am_count = nullptr;       // its completion counter (returns to 0)
    float *rope_cos, *rope_sin;
    float *rope_cos_full = nullptr, *rope_sin_full = nullptr;  // Gemma4 full-attention layers
    float *pli_emb = nullptr, *pli_tmp = nullptr, *pli_in = nullptr, *pli_g = nullptr;  // Gemma4 per-layer inputs
    std::vector<float *> S, hist, rq, rkv;      // per layer (SSM) else null
    std::vector<float *> kc, vc;                // per layer (attention) else null
    float *mtp_kc = nullptr, *mtp_vc = nullptr;
    void *acc_scratch = nullptr;
    float *attn_part = nullptr;         // split-KV attention: partial softmax states (null: cluster kernel)
    bool kv16 = false;                  // kc / vc / mtp_kc / mtp_vc hold bf16 rows (ifr_ctx_set_kv_bf16)
    void *dense = nullptr;              // scratch of the dense tensor-core GEMMs
    int64_t dense_bytes = 0;
    int last_n = 0;
    int pending = -1;                   // gamma of a verify awaiting ifr_rollback, else -1
    bool prefill_chunk = false;         // a one-request prefill chunk is being enqueued
    // kernel launches enqueued (for the benchmark's launch count)
    int64_t launches = 0;
    // optional per-category CUDA-event timing of the launches
    bool prof = false;
    std::vector<cudaEvent_t> ev_pool;
    struct Rec { int ev0, cat; int64_t bytes; };
    std::vector<Rec> recs;
    int ev_next = 0;
    // fused layer stack (one request): device phase lists for n = 1..kNMax
    // columns (null: the model is not covered), its grid-barrier counter and
    // the split-KV partials of its attention phases
    ifr::FPhase *fused_ph[kNMax + 1] = {};
    int fused_np[kNMax + 1] = {};
    unsigned *fused_ctr = nullptr;
    float *fused_part = nullptr;
    float *fused_ssq = nullptr, *fused_stage = nullptr;  // split GatedDeltaNet step scratch
    // profiling: phase start times of the last fused launch, its phase kinds
    unsigned long long *fused_trace = nullptr;
    std::vector<int> fused_kinds[kNMax + 1];
    int fused_last = 0;
    // a captured CUDA graph of consecutive spec steps
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    ~ifr_state() {
        if (graph_exec) cudaGraphExecDestroy(graph_exec);
        if (graph) cudaGraphDestroy(graph);
        for (auto e : ev_pool) cudaEventDestroy(e);
        for (void *p : allocs) cudaFree(p);
        if (h_tok) cudaFreeHost(h_tok);
    }
};

namespace {

template <class T>
int dalloc(ifr_state *s, T **p, size_t n) {
    void *d = nullptr;
    ECHECK(cudaMalloc(&d, n * sizeof(T) + 16), "cudaMalloc(state)");
    ECHECK(cudaMemset(d, 0, n * sizeof(T) + 16), "cudaMemset(state)");
    s->allocs.push_back(d);
    *p = (T *)d;
    return IFR_OK;
}

// categories of timed launches (ifr_state_profile_read)
enum {
    CAT_LM_HEAD = 0, CAT_DRAFT_LM_HEAD, CAT_LAYER_GEMV, CAT_DRAFT_GEMV, CAT_SSM, CAT_ATTN, CAT_COMM, CAT_FUSED,
    CAT_NCAT = 8
};

struct ProfScope {
    ifr_state *s;
    cudaStream_t st;
    int ev0 = -1;
    ProfScope(ifr_state *s_, int cat, int64_t bytes, cudaStream_t st_) : s(s_), st(st_) {
        if (!s || !s->prof) return;
        while ((int)s->ev_pool.size() < s->ev_next + 2) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return;
            s->ev_pool.push_back(e);
        }
        ev0 = s->ev_next;
        s->ev_next += 2;
        cudaEventRecord(s->ev_pool[ev0], st);
        s->recs.push_back({ev0, cat, bytes});
    }
    ~ProfScope() {
        if (ev0 >= 0) cudaEventRecord(s->ev_pool[ev0 + 1], st);
    }
};

int64_t proj_bytes(const Proj &p);

// tensor parallelism: the sum all-reduce of n floats over the ranks (timed as
// CAT_COMM when profiling); no-op for one rank
int allreduce(ifr_state *s, float *x, size_t n, cudaStream_t st) {
    if (!s->m->comm) return IFR_OK;
    ProfScope ps(s, CAT_COMM, (int64_t)n * 4, st);
    return comm_allreduce_sum(s->m->comm, x, n, st);
}

// Y (+)= W X over n columns: the exact small-N kernel in passes of 8 columns,
// or the dense tensor-core kernel once n reaches the context's threshold
int gemv(ifr_state *s, int cat, const Proj &p, const float *X, int n, float *Y, bool accumulate, cudaStream_t st,
         const ifr::XForm &xf = ifr::XForm()) {
    ProfScope ps(s, cat, proj_bytes(p), st);
    int64_t r0 = 0;
    const int64_t ldy = xf.ep ? p.rows / 2 : p.rows;
    ifr::XForm f = xf;
    f.act = ifr_ctx_activation(s->m->ctx);
    // one request: dense only for the prefill chunks the context allows
    const bool dense = n >= ifr_ctx_dense_min(s->m->ctx) && s->dense &&
                       (s->B > 1 || (s->prefill_chunk && ifr_ctx_prefill_dense(s->m->ctx)));
    for (auto &q : p.parts) {
        if (dense) {
            ECHECK(ifr::qgemm_dense(q, X, n, Y + r0, accumulate, ldy, st, f, s->dense, s->dense_bytes), "qgemm_dense");
            s->launches += 2;
        } else {
            const int64_t ldx = f.ldx > 0 ? f.ldx : q.cols;
            for (int c0 = 0; c0 < n; c0 += kNMax) {
                const int k = std::min(kNMax, n - c0);
                ECHECK(ifr::qgemm_small(q, X + c0 * ldx, k, Y + r0 + c0 * ldy, accumulate, ldy, st, f), "qgemm");
                s->launches++;
            }
        }
        r0 += q.rows;
    }
    return IFR_OK;
}

// the attention of n tokens per request; a prefill chunk (n > kNMax, one
// request) runs as sub-calls of kNMax tokens in order, each at its own
// position (s->chunk_pos), so every sub-call finds the earlier ones' keys in
// the cache
int attn_call(ifr_state *s, ifr::AttnArgs a, int n, int B, cudaStream_t st) {
    if (n <= kNMax) {
        ECHECK(ifr::attn_step(a, B, st), "attn_step");
        return IFR_OK;
    }
    const float *qkv = a.qkv;
    float *out = a.out;
    for (int t0 = 0, i = 0; t0 < n; t0 += kNMax, i++) {
        a.N = std::min(kNMax, n - t0);
        a.qkv = qkv + (int64_t)t0 * a.ldq;
        a.out = out + (int64_t)t0 * a.ldo;
        a.pos = s->chunk_pos + i;
        if (s->attn_part) a.splits = ifr::attn_splits(a.nh, a.nkv, a.N, B, s->max_ctx);
        ECHECK(ifr::attn_step(a, B, st), "attn_step");
        s->launches += s->attn_part ? 2 : 1;
    }
    return IFR_OK;
}

// Gemma4 full-attention layers rotate Int(partial * hd / 2) pairs
// (precompute_rope, Gemma4.jl:214-228); the remaining pairs have cos 1, sin 0
int gemma_full_pairs(const ifr_model *m) {
    return (int)(m->partial_rotary * (float)m->info.head_dim) / 2;
}

// the GatedDeltaNet step of layer li over n columns per request (s->proj, s->x -> s->y)
ifr::SsmArgs ssm_args(ifr_state *s, const DevLayer &L, int li, int n) {
    const ifr_model *m = s->m;
    const ifr_model_info &c = m->info;
    ifr::SsmArgs a{};
    a.proj = s->proj;
    a.ldp = L.proj.rows;
    a.xn = s->x;
    a.in_norm = L.attn_norm;
    a.d = c.hidden;
    a.conv_w = L.conv_w;
    a.ab_w = L.ab_w;
    a.ssm_a = L.ssm_a;
    a.dt_bias = L.dt_bias;
    a.norm_w = L.ssm_norm;
    a.S = s->S[li];
    a.hist = s->hist[li];
    a.rq = s->rq[li];
    a.rkv = s->rkv[li];
    a.a_prev = &s->sc->a_prev;
    a.y = s->y;
    a.ldy = m->inner;
    a.N = n;
    a.H = c.ssm_heads;
    a.C = m->conv_channels;
    a.K = c.conv_kernel;
    a.eps = c.rms_eps;
    const int64_t hd = c.ssm_head_dim;
    a.b_S = (int64_t)c.ssm_heads * hd * hd;
    a.b_hist = (int64_t)(c.conv_kernel - 1) * m->conv_channels;
    a.b_rq = (int64_t)kNMax * m->conv_channels;
    a.b_rkv = (int64_t)c.ssm_heads * kNMax * (2 * hd + 2);
    a.b_prev = (int)(sizeof(ifr::EngineScalars) / sizeof(int32_t));
    return a;
}

// the gated attention step of a Qwen3.5 attention layer over n columns per
// request (s->proj -> s->y; keys and values of request b at kc / vc + b * kv_ld)
ifr::AttnArgs attn_args(ifr_state *s, const DevLayer &L, int n, float *kc, float *vc, const int32_t *pos,
                        int pos_ld, int64_t kv_ld) {
    const ifr_model *m = s->m;
    const ifr_model_info &c = m->info;
    ifr::AttnArgs a{};
    a.qkv = s->proj;
    a.ldq = L.proj.rows;
    a.q_norm = L.q_norm;
    a.k_norm = L.k_norm;
    a.kc = kc;
    a.vc = vc;
    a.pos = pos;
    a.rope_cos = s->rope_cos;
    a.rope_sin = s->rope_sin;
    a.out = s->y;
    a.ldo = (int64_t)m->nh * c.head_dim;
    a.N = n;
    a.nh = m->nh;
    a.nkv = m->nkv;
    a.hd = c.head_dim;
    a.rotary_dim = c.rotary_dim;
    a.eps = c.rms_eps;
    a.b_kv = kv_ld;
    a.b_pos = pos_ld;
    a.kv16 = s->kv16 ? 1 : 0;
    return a;
}

// one decoder layer (attention or SSM) on n columns of s->x
// n tokens per request, s->B requests (columns b * n + t); pos of request b at
// pos + b * pos_ld; kc / vc of request b at + b * kv_ld
int layer_forward(ifr_state *s, const DevLayer &L, int li, int n, float *kc, float *vc, const int32_t *pos,
                  int pos_ld, int64_t kv_ld, bool draft, cudaStream_t st) {
    ifr_model *m = s->m;
    const ifr_model_info &c = m->info;
    const int d = c.hidden;
    const int B = s->B, nc = B * n;
    const int gcat = draft ? CAT_DRAFT_GEMV : CAT_LAYER_GEMV;
    int rc;
    // the layer's two RMSNorms are applied inside their consumers: the input
    // GEMVs (folded into the epilogue on the small-N kernel, in the packing
    // kernel on the dense path) and the SSM's alpha / beta projections
    ifr::XForm in_norm;
    in_norm.kind = 1;
    in_norm.w = L.attn_norm;
    in_norm.eps = c.rms_eps;
    s->launches += (L.ssm || !s->attn_part) ? 1 : 2;  // the SSM / attention step (split-KV: two kernels)
    if ((rc = gemv(s, gcat, L.proj, s->x, nc, s->proj, false, st, in_norm))) return rc;
    if (m->gemma) {
        // Gemma4 layer (Gemma4.jl:622-650): x = x + RMSNorm(wo attn(norm_in(x)));
        // x = (x + RMSNorm(down(gelu_tanh(gate) up)(norm_ff(x)))) * layer_scalar
        ProfScope ps(s, CAT_ATTN, 0, st);
        ifr::AttnArgs a{};
        a.qkv = s->proj;
        a.ldq = L.proj.rows;
        a.q_norm = L.q_norm;
        a.k_norm = L.k_norm;
        a.kc = kc;
        a.vc = vc;
        a.pos = pos;
        a.out = s->y;
        a.ldo = (int64_t)m->nh * c.head_dim;
        a.N = n;
        a.nh = m->nh;
        a.nkv = m->nkv;
        a.hd = c.head_dim;
        a.rotary_dim = c.rotary_dim;
        a.eps = c.rms_eps;
        a.b_kv = kv_ld;
        a.b_pos = pos_ld;
        a.kv16 = s->kv16 ? 1 : 0;
        a.gated = 0;
        a.vnorm = 1;
        a.scale = 1.0f;
        a.softcap = m->attn_softcap;
        a.window = L.sliding ? m->window : 0;
        a.rope_off = a.rope_ld = c.head_dim / 2;
        a.rope_cos = L.sliding ? s->rope_cos : s->rope_cos_full;
        a.rope_sin = L.sliding ? s->rope_sin : s->rope_sin_full;
        a.rope_pairs = L.sliding ? c.head_dim / 2 : gemma_full_pairs(m);
        if (s->attn_part) {
            a.part = s->attn_part;
            a.splits = ifr::attn_splits(m->nh, m->nkv, n, B, s->max_ctx);
        }
        if ((rc = attn_call(s, a, n, B, st))) return rc;
        // row-parallel projections: every rank's partial, summed over the ranks
        if ((rc = gemv(s, gcat, L.out, s->y, nc, s->xn, false, st))) return rc;
        if ((rc = allreduce(s, s->xn, (size_t)nc * d, st))) return rc;
        ifr::norm_add(s->xn, L.post_norm, s->x, nc, d, c.rms_eps, nullptr, st);
        ifr::XForm glu = in_norm;
        glu.w = L.ffn_norm;
        glu.ep = 2;  // gelu_tanh(gate) * up
        if ((rc = gemv(s, gcat, L.gate_up, s->x, nc, s->hmid, false, st, glu))) return rc;
        if ((rc = gemv(s, gcat, L.down, s->hmid, nc, s->xn, false, st))) return rc;
        if ((rc = allreduce(s, s->xn, (size_t)nc * d, st))) return rc;
        const bool pli = m->pli && !draft && li >= 0;
        ifr::norm_add(s->xn, L.post_ffw_norm, s->x, nc, d, c.rms_eps, pli ? nullptr : L.layer_scalar, st);
        s->launches += 2;
        if (pli) {
            // per_layer_input_forward! (Gemma4.jl:505-533, :626-634):
            // x = (x + RMSNorm(proj(gelu_tanh(gate x) * pli_i))) * layer_scalar
            if ((rc = gemv(s, gcat, L.pli_gate, s->x, nc, s->pli_g, false, st))) return rc;
            ECHECK(ifr::pli_gate(s->pli_g, s->pli_in, m->pli, (int64_t)c.n_layers * m->pli, li, nc, st), "pli gate");
            if ((rc = gemv(s, gcat, L.pli_proj, s->pli_g, nc, s->xn, false, st))) return rc;
            ifr::norm_add(s->xn, L.pli_post_norm, s->x, nc, d, c.rms_eps, L.layer_scalar, st);
            s->launches += 2;
        }
        return IFR_OK;
    }
    if (L.ssm) {
        ProfScope ps(s, CAT_SSM, 0, st);
        const ifr::SsmArgs a = ssm_args(s, L, li, n);
        if (n > kNMax)  // a prefill chunk of one request: scanned and committed in one launch
            ECHECK(ifr::ssm_chunk(a, c.ssm_head_dim, st), "ssm_chunk");
        else
            ECHECK(ifr::ssm_step(a, c.ssm_head_dim, B, st), "ssm_step");
    } else {
        ProfScope ps(s, CAT_ATTN, 0, st);
        ifr::AttnArgs a = attn_args(s, L, n, kc, vc, pos, pos_ld, kv_ld);
        if (s->attn_part) {
            a.part = s->attn_part;
            a.splits = ifr::attn_splits(m->nh, m->nkv, n, B, s->max_ctx);
        }
        if ((rc = attn_call(s, a, n, B, st))) return rc;
    }
    // row-parallel projections: rank 0 adds its partial to the residual, the
    // others write theirs, and one sum all-reduce leaves x + sum on every rank
    if ((rc = gemv(s, gcat, L.out, s->y, nc, s->x, m->tp_rank == 0, st))) return rc;
    if ((rc = allreduce(s, s->x, (size_t)nc * d, st))) return rc;
    ifr::XForm post_norm = in_norm;
    post_norm.w = L.post_norm;
    if (L.gate_up.glu) {
        // silu(gate) * up formed in the gate/up GEMV's epilogue
        ifr::XForm glu = post_norm;
        glu.ep = 1;
        if ((rc = gemv(s, gcat, L.gate_up, s->x, nc, s->hmid, false, st, glu))) return rc;
        if ((rc = gemv(s, gcat, L.down, s->hmid, nc, s->x, m->tp_rank == 0, st))) return rc;
        return allreduce(s, s->x, (size_t)nc * d, st);
    }
    if ((rc = gemv(s, gcat, L.gate_up, s->x, nc, s->gu, false, st, post_norm))) return rc;
    // silu(gate) * up formed while the down GEMV reads [gate | up]
    ifr::XForm swiglu;
    swiglu.kind = 2;
    swiglu.ldx = 2 * (int64_t)m->ffn;
    if ((rc = gemv(s, gcat, L.down, s->gu, nc, s->x, m->tp_rank == 0, st, swiglu))) return rc;
    return allreduce(s, s->x, (size_t)nc * d, st);
}

// ---- the layer stack of a one-request verify as one launch (fused_step.cuh)

// the projection's GEMV phases over n columns, one per part (the parts write
// disjoint rows of Y from the same X: no barrier between them)
bool fused_proj(std::vector<ifr::FPhase> &v, const Proj &p, const float *X, int n, float *Y, bool acc,
                const float *xw, float eps, int ep) {
    if (p.parts.empty() || (ep && p.parts.size() != 1)) return false;
    int64_t r0 = 0;
    const int64_t ldy = ep ? p.rows / 2 : p.rows;
    for (size_t i = 0; i < p.parts.size(); i++) {
        const ifr::QTensor &q = p.parts[i];
        ifr::FGemv g{};
        g.W = q.data;
        g.M = q.rows;
        g.K = q.cols;
        g.nrb = (int)q.nrb;
        g.nu = (int)q.nu;
        g.fmt = q.type;
        g.nt = n <= 4 ? 1 : 2;
        g.xf = xw ? 3 : 0;
        g.ep = ep;
        g.accumulate = acc ? 1 : 0;
        g.gran = ep ? 2 : 1;
        g.X = X;
        g.ldx = q.cols;
        g.ncols = n;
        g.Y = Y + r0;
        g.ldy = ldy;
        g.xw = xw;
        g.eps = eps;
        ifr::FPhase ph;
        if (!ifr::fused_gemv_phase(g, ph)) return false;
        ph.nobar = i + 1 < p.parts.size() ? 1 : 0;
        v.push_back(ph);
        r0 += q.rows;
    }
    return true;
}

// the phases of the target's decoder layers over n columns (layer_forward's
// sequence for one request, one rank, SwiGLU MLPs); false when a layer is not
// covered
bool fused_plan(ifr_state *s, int n, std::vector<ifr::FPhase> &v) {
    ifr_model *m = s->m;
    const ifr_model_info &c = m->info;
    const int sc_ld = (int)(sizeof(ifr::EngineScalars) / sizeof(int32_t));
    const int64_t kv_ld = (int64_t)s->max_ctx * m->nkv * c.head_dim;
    v.clear();
    for (int li = 0; li < c.n_layers; li++) {
        const DevLayer &L = m->layers[li];
        if (!L.gate_up.glu) return false;
        if (!fused_proj(v, L.proj, s->x, n, s->proj, false, L.attn_norm, c.rms_eps, 0)) return false;
        if (L.ssm) {
            ifr::FPhase upd, fin;
            if (!ifr::fused_ssm_phases(ssm_args(s, L, li, n), c.ssm_head_dim, s->fused_ssq, s->fused_stage, upd, fin))
                return false;
            v.push_back(upd);
            v.push_back(fin);
        } else {
            ifr::AttnArgs a = attn_args(s, L, n, s->kc[li], s->vc[li], &s->sc->pos, sc_ld, kv_ld);
            a.part = s->fused_part;
            a.splits = ifr::attn_splits(m->nh, m->nkv, n, 1, s->max_ctx);
            ifr::FPhase part, comb;
            if (!ifr::fused_attn_phases(a, part, comb)) return false;
            v.push_back(part);
            v.push_back(comb);
        }
        if (!fused_proj(v, L.out, s->y, n, s->x, true, nullptr, 0.f, 0)) return false;
        if (!fused_proj(v, L.gate_up, s->x, n, s->hmid, false, L.post_norm, c.rms_eps, 1)) return false;
        if (!fused_proj(v, L.down, s->hmid, n, s->x, true, nullptr, 0.f, 0)) return false;
    }
    // L2 prefetch plan: the first phase sends the next two GEMV phases'
    // weights, every GEMV phase after it the one two GEMV phases ahead
    // (phase 0's own weights are sent at the kernel's start)
    std::vector<int> gi;
    for (int i = 0; i < (int)v.size(); i++)
        if (v[i].kind == ifr::FPhase::kGemv) gi.push_back(i);
    auto pf = [&](int k) {
        const ifr::FGemv &g = v[gi[k]].g;
        ifr::FPrefetch p;
        p.W = g.W;
        p.nrb = g.nrb;
        p.nu = g.nu;
        p.fmt = g.fmt;
        p.gran = g.gran;
        return p;
    };
    for (int k = 0; k < (int)gi.size(); k++) {
        if (k == 0) {
            if (gi.size() > 1) v[gi[0]].pf[0] = pf(1);
            if (gi.size() > 2) v[gi[0]].pf[1] = pf(2);
        } else if (k + 2 < (int)gi.size()) {
            v[gi[k]].pf[0] = pf(k + 2);
        }
    }
    // tile-buffer plan: a GEMV phase's tiles are copied as soon as the previous
    // GEMV phase has read its own (phase 0's at the kernel's start)
    for (int k = 1; k < (int)gi.size(); k++)
        if (v[gi[k]].tiles_smem) v[gi[k - 1]].tl = pf(k);
    if (!gi.empty() && gi[0] > 0 && v[gi[0]].tiles_smem) v[0].tl = pf(0);
    return true;
}

// builds the state's fused phase lists for n = 1..kNMax when the model is
// covered (one request, one rank, Qwen3.5 blocks); leaves them null otherwise
int fused_build(ifr_state *s) {
    ifr_model *m = s->m;
    const ifr_model_info &c = m->info;
    if (s->B != 1 || m->comm || m->gemma || s->kv16 || c.n_layers < 1) return IFR_OK;
    bool any_attn = false;
    for (auto &L : m->layers) any_attn |= !L.ssm;
    if (any_attn) {
        int rc = dalloc(s, &s->fused_part, (size_t)ifr::attn_part_floats(m->nh, m->nkv, c.head_dim, 1, s->max_ctx));
        if (rc) return rc;
    }
    if (c.ssm_heads > 0) {
        const size_t rec = (size_t)c.ssm_heads * kNMax * (2 * c.ssm_head_dim + 2);
        int rc = dalloc(s, &s->fused_ssq, (size_t)c.ssm_heads * ifr::kFusedSsmSplit * kNMax);
        if (!rc) rc = dalloc(s, &s->fused_stage, rec);
        if (rc) return rc;
    }
    std::vector<std::vector<ifr::FPhase>> plans(kNMax + 1);
    for (int n = 1; n <= kNMax; n++)
        if (!fused_plan(s, n, plans[n])) return IFR_OK;  // not covered: the separate launches
    int rc = dalloc(s, &s->fused_ctr, 4);
    size_t most = 0;
    for (int n = 1; n <= kNMax; n++) {
        most = std::max(most, plans[n].size());
        for (auto &ph : plans[n]) s->fused_kinds[n].push_back(ph.kind);
    }
    if (!rc) rc = dalloc(s, &s->fused_trace, 4 * most * (ifr::fused_ctas() + 1) + 1);
    for (int n = 1; !rc && n <= kNMax; n++) {
        rc = dalloc(s, &s->fused_ph[n], plans[n].size());
        if (!rc && cudaMemcpy(s->fused_ph[n], plans[n].data(), plans[n].size() * sizeof(ifr::FPhase),
                              cudaMemcpyHostToDevice) != cudaSuccess)
            rc = ifr_fail(IFR_ERR_CUDA, "H2D fused phases");
        s->fused_np[n] = (int)plans[n].size();
    }
    return rc;
}

// the fp16 operand stages of every projection of the model for the dense GEMM
// (ifr_ctx_set_dense_f16_weights); a part that cannot get its memory keeps
// the dequantizing path (same results)
int model_prepare_f16(ifr_model *m, cudaStream_t st) {
    auto prep = [&](Proj &p) {
        for (auto &q : p.parts) {
            if (q.f16) continue;
            void *d = nullptr;
            if (cudaMalloc(&d, ifr::qgemm_dense_f16_bytes(q)) != cudaSuccess) {
                cudaGetLastError();
                return IFR_OK;
            }
            m->dev_allocs.push_back(d);
            ECHECK(ifr::qgemm_dense_prepare_f16(q, static_cast<uint8_t *>(d), st), "fp16 stages");
        }
        return IFR_OK;
    };
    int rc = IFR_OK;
    for (auto &L : m->layers)
        for (Proj *p : {&L.proj, &L.out, &L.gate_up, &L.down})
            if (!rc) rc = prep(*p);
    if (!rc) rc = prep(m->lm_head);
    if (!rc && m->has_mtp) {
        for (Proj *p : {&m->mtp_fc, &m->mtp_layer.proj, &m->mtp_layer.out, &m->mtp_layer.gate_up, &m->mtp_layer.down})
            if (!rc) rc = prep(*p);
    }
    if (!rc) ECHECK(cudaStreamSynchronize(st), "fp16 stages sync");
    return rc;
}

// the verify of n columns runs as the fused launch
bool fused_on(const ifr_state *s, int n) {
    return n >= 1 && n <= kNMax && s->fused_ph[n] && !s->prefill_chunk && ifr_ctx_fused_layers(s->m->ctx) &&
           ifr_ctx_activation(s->m->ctx) == IFR_ACT_EXACT;
}

// embedding rows of the n verify tokens of each of B requests (row b * n + t):
// token 0 of request b from its last emitted token (first + b * first_ld) when
// `first` is set (and written to its vtok[0]), the others from vtok[b * kNMax + t];
// one thread per 32-element group (get_embedding, ModelCPU.jl:1005-1007)
template <int T>
__global__ void embed_kernel(const uint8_t *__restrict__ w, int64_t nu, int64_t nb_raw, int64_t rows, int64_t cols,
                             int32_t *vtok, const int32_t *first, int first_ld, int n, int B,
                             float *__restrict__ out, float scale) {
    ifr::pdl_trigger();
    ifr::pdl_wait();
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * n * nu * 8) return;
    const int sub = (int)(i & 7);
    const int64_t u = (i >> 3) % nu;
    const int tg = (int)((i >> 3) / nu), b = tg / n, t = tg % n;
    int32_t *vt = vtok + (int64_t)b * kNMax;
    int64_t tok = (t == 0 && first) ? first[(int64_t)b * first_ld] : vt[t];
    if (t == 0 && u == 0 && sub == 0 && first) vt[0] = (int32_t)tok;
    tok = tok < 0 ? 0 : (tok >= rows ? rows - 1 : tok);
    float *o = out + (int64_t)tg * cols + u * 256 + 32 * sub;
    ifr::dequant_group<T>(w, nu, nb_raw, tok, u, sub, o);
    if (scale != 1.0f)  // Gemma4: the embedding row times embed_scale (Gemma4.jl:612-615)
        for (int i = 0; i < 32; i++) o[i] = __fmul_rn(o[i], scale);
}

__device__ float block_sum_256(float v, float *red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.f;
    for (int w = 0; w < 8; w++) r += red[w];
    return r;
}

constexpr int kMtpPer = 24;  // mtp_prep_kernel: hidden sizes up to 256 x 24 = 6144

// MTP input of one draft (mtp_forward!, ModelCPU.jl:2031-2051), request
// b = blockIdx.x: cat = [RMSNorm(embed(tok), norm_e); RMSNorm(h, norm_h)], and
// the draft's position pos + add for the MTP attention layer
template <int T>
__global__ void __launch_bounds__(256) mtp_prep_kernel(const uint8_t *__restrict__ w, int64_t nu, int64_t nb_raw,
                                                       int64_t rows, const int32_t *tok, int tok_ld, const float *h,
                                                       const float *__restrict__ we, const float *__restrict__ wh,
                                                       float eps, int d, float *__restrict__ cat, int32_t *pos_out,
                                                       const ifr::EngineScalars *sc, int add) {
    extern __shared__ float e_s[];  // nu * 256 floats
    __shared__ float red[8];
    ifr::pdl_trigger();
    ifr::pdl_wait();
    const int b = blockIdx.x;
    tok += (int64_t)b * tok_ld;
    h += (int64_t)b * d;
    cat += (int64_t)b * 2 * d;
    pos_out += b;
    sc += b;
    int64_t t = *tok;
    t = t < 0 ? 0 : (t >= rows ? rows - 1 : t);
    for (int gi = threadIdx.x; gi < nu * 8; gi += 256) ifr::dequant_group<T>(w, nu, nb_raw, t, gi >> 3, gi & 7, e_s + 32 * gi);
    __syncthreads();
    // h and the two norm weights for this thread's elements, loaded once and
    // up front (each thread owns i = tid + 256 k; d <= 256 kMtpPer)
    float hv[kMtpPer], wev[kMtpPer], whv[kMtpPer];
#pragma unroll
    for (int k = 0; k < kMtpPer; k++) {
        const int i = threadIdx.x + 256 * k;
        hv[k] = i < d ? h[i] : 0.f;
        wev[k] = i < d ? we[i] : 0.f;
        whv[k] = i < d ? wh[i] : 0.f;
    }
    float se = 0.f, sh = 0.f;
#pragma unroll
    for (int k = 0; k < kMtpPer; k++) {
        const int i = threadIdx.x + 256 * k;
        if (i < d) {
            se += e_s[i] * e_s[i];
            sh += hv[k] * hv[k];
        }
    }
    se = block_sum_256(se, red);
    sh = block_sum_256(sh, red);
    const float ie = 1.0f / sqrtf(se / (float)d + eps), ih = 1.0f / sqrtf(sh / (float)d + eps);
#pragma unroll
    for (int k = 0; k < kMtpPer; k++) {
        const int i = threadIdx.x + 256 * k;
        if (i < d) {
            cat[i] = e_s[i] * ie * wev[k];
            cat[d + i] = hv[k] * ih * whv[k];
        }
    }
    if (threadIdx.x == 0) *pos_out = sc->pos + add;
}

template <int T>
cudaError_t launch_embed_t(const ifr::QTensor &e, int32_t *vtok, const int32_t *first, int first_ld, int n, int B,
                           float *out, float scale, cudaStream_t st) {
    const int64_t tot = (int64_t)B * n * e.nu * 8;
    return ifr::launch_k(embed_kernel<T>, dim3((unsigned)((tot + 127) / 128)), dim3(128), 0, st, (const uint8_t *)e.data,
                         (int64_t)e.nu, (int64_t)e.nb, (int64_t)e.rows, (int64_t)e.cols, vtok, first, first_ld, n, B,
                         out, scale);
}
cudaError_t launch_embed(const ifr::QTensor &e, int32_t *vtok, const int32_t *first, int first_ld, int n, int B,
                         float *out, float scale, cudaStream_t st) {
    switch (e.type) {
    case 12: return launch_embed_t<12>(e, vtok, first, first_ld, n, B, out, scale, st);
    case 13: return launch_embed_t<13>(e, vtok, first, first_ld, n, B, out, scale, st);
    case 14: return launch_embed_t<14>(e, vtok, first, first_ld, n, B, out, scale, st);
    case 8: return launch_embed_t<8>(e, vtok, first, first_ld, n, B, out, scale, st);
    }
    return cudaErrorInvalidValue;
}

template <int T>
cudaError_t launch_mtp_prep_t(const ifr::QTensor &e, const int32_t *tok, int tok_ld, const float *h, const float *we,
                              const float *wh, float eps, int d, float *cat, int32_t *pos_out,
                              const ifr::EngineScalars *sc, int add, int B, cudaStream_t st) {
    return ifr::launch_k(mtp_prep_kernel<T>, dim3(B), dim3(256), (size_t)e.nu * 256 * 4, st, (const uint8_t *)e.data,
                         (int64_t)e.nu, (int64_t)e.nb, (int64_t)e.rows, tok, tok_ld, h, we, wh, eps, d, cat, pos_out,
                         sc, add);
}
cudaError_t launch_mtp_prep(const ifr::QTensor &e, const int32_t *tok, int tok_ld, const float *h, const float *we,
                            const float *wh, float eps, int d, float *cat, int32_t *pos_out,
                            const ifr::EngineScalars *sc, int add, int B, cudaStream_t st) {
    if (d > 256 * kMtpPer) return cudaErrorInvalidValue;
    switch (e.type) {
    case 12: return launch_mtp_prep_t<12>(e, tok, tok_ld, h, we, wh, eps, d, cat, pos_out, sc, add, B, st);
    case 13: return launch_mtp_prep_t<13>(e, tok, tok_ld, h, we, wh, eps, d, cat, pos_out, sc, add, B, st);
    case 14: return launch_mtp_prep_t<14>(e, tok, tok_ld, h, we, wh, eps, d, cat, pos_out, sc, add, B, st);
    case 8: return launch_mtp_prep_t<8>(e, tok, tok_ld, h, we, wh, eps, d, cat, pos_out, sc, add, B, st);
    }
    return cudaErrorInvalidValue;
}

// greedy acceptance of G drafts per sequence over B x (G+1) logits rows (the
// argmax over all ranks' vocabulary shards under tensor parallelism)
int greedy_accept(ifr_state *s, const int32_t *drafts, int draft_ld, int B, int G, int32_t *out, int out_ld,
                  cudaStream_t st) {
    ifr_model *m = s->m;
    if (!m->comm) {
        ECHECK(ifr::accept_greedy_fused(s->logits, drafts, B, G, m->vocab, s->acc, out, s->acc_scratch, s->gcount, st,
                                        draft_ld, out_ld),
               "greedy accept");
        return IFR_OK;
    }
    const int rows = B * (G + 1), W = m->tp_world;
    float *mine = s->cand + (size_t)2 * rows * W;  // this rank's candidates, past the gathered block
    ECHECK(ifr::row_argmax(s->logits, rows, m->vocab, m->vocab_off, mine, st), "row argmax");
    int rc = comm_allgather_bytes(m->comm, mine, s->cand, (size_t)rows * 8, st);
    if (rc) return rc;
    ECHECK(ifr::tp_accept(s->cand, W, rows, drafts, draft_ld, B, G, s->acc, out, out_ld, st), "tp accept");
    s->launches += 2;
    return IFR_OK;
}

// target forward of the n tokens per request in vtok (request b: vtok[b *
// kNMax ..], positions sc[b].pos ..; device); final-normed hidden of every
// column in s->hid; logits of every column in s->logits when `logits` is set
int target_forward(ifr_state *s, int n, bool logits, bool first_from_state, cudaStream_t st,
                   const ifr::GemvArgmax *am = nullptr) {
    ifr_model *m = s->m;
    const ifr_model_info &c = m->info;
    const int B = s->B, nc = B * n;
    const int sc_ld = (int)(sizeof(ifr::EngineScalars) / sizeof(int32_t));
    ECHECK(launch_embed(m->embed.parts[0], s->vtok, first_from_state ? &s->sc->last_token : nullptr, sc_ld, n, B,
                        s->x, m->embed_scale, st),
           "embedding");
    s->launches += 2;  // embedding, final norm
    if (m->pli) {
        // compute_per_layer_inputs! (Gemma4.jl:459-503) for every column: the
        // token table rows, the model projection of the scaled embedding, then
        // per layer (RMSNorm(proj) + row sqrt(pli)) 2^-1/2
        const int64_t lp = (int64_t)c.n_layers * m->pli;
        ECHECK(launch_embed(m->pli_token_embd.parts[0], s->vtok, first_from_state ? &s->sc->last_token : nullptr, sc_ld,
                            n, B, s->pli_emb, 1.0f, st),
               "per-layer input table");
        int rc = gemv(s, CAT_LAYER_GEMV, m->pli_model_proj, s->x, nc, s->pli_tmp, false, st);
        if (rc) return rc;
        ECHECK(ifr::pli_inputs(s->pli_tmp, s->pli_emb, m->pli_proj_norm, m->pli, c.n_layers, nc, c.rms_eps,
                               s->pli_in, st),
               "per-layer inputs");
        (void)lp;
        s->launches += 2;
    }
    if (n > kNMax) {
        ifr::chunk_positions(s->chunk_pos, s->sc, (n + kNMax - 1) / kNMax, kNMax, st);
        s->launches++;
    }
    const int64_t kv_ld = (int64_t)s->max_ctx * m->nkv * c.head_dim;
    if (fused_on(s, n)) {
        ProfScope ps(s, CAT_FUSED, 0, st);
        if (s->prof)
            ECHECK(cudaMemsetAsync(s->fused_trace, 0,
                                   (4 * (size_t)s->fused_np[n] * (ifr::fused_ctas() + 1) + 1) * sizeof(unsigned long long), st),
                   "fused trace reset");
        ECHECK(ifr::fused_layers(s->fused_ph[n], s->fused_np[n], s->fused_ctr, s->prof ? s->fused_trace : nullptr, st),
               "fused_layers");
        s->launches++;
        s->fused_last = n;
    } else {
        for (int li = 0; li < c.n_layers; li++) {
            int rc = layer_forward(s, m->layers[li], li, n, s->kc[li], s->vc[li], &s->sc->pos, sc_ld, kv_ld, false, st);
            if (rc) return rc;
        }
    }
    ifr::rmsnorm(s->x, m->final_norm, s->hid, nc, c.hidden, c.rms_eps, c.hidden, c.hidden, st);
    if (logits) {
        ifr::XForm f;
        f.am = am;
        int rc = gemv(s, CAT_LM_HEAD, m->lm_head, s->hid, nc, s->logits, false, st, f);
        if (rc) return rc;
        if (m->final_softcap > 0.f) {  // get_logits (Gemma4.jl:678-693): logit_softcap!
            ifr::softcap(s->logits, (int64_t)nc * m->vocab, m->final_softcap, st);
            s->launches++;
        }
    }
    s->last_n = n;
    return IFR_OK;
}

__global__ void set_pos_kernel(int32_t *dst, const ifr::EngineScalars *sc, int add) {
    ifr::pdl_trigger();
    ifr::pdl_wait();
    *dst = sc->pos + add;
}
// after the prompt's last token (one column per request, b = blockIdx.x):
// its greedy token is emitted and fed next, its hidden feeds the MTP head
__global__ void prefill_finish_kernel(ifr::EngineScalars *sc, const int32_t *tok, const float *hid, float *mtp_h,
                                      int d, int32_t *log, int log_cap) {
    ifr::pdl_trigger();
    ifr::pdl_wait();
    const int b = blockIdx.x;
    sc += b;
    tok += b;
    hid += (int64_t)b * d;
    mtp_h += (int64_t)b * d;
    log += (int64_t)b * log_cap;
    if (threadIdx.x == 0) {
        sc->last_token = *tok;
        if (sc->n_log < log_cap) log[sc->n_log++] = *tok;
    }
    for (int i = threadIdx.x; i < d; i += blockDim.x) mtp_h[i] = hid[i];
}

// the lm_head of nc columns can make the greedy decision in its own epilogue:
// one small-N launch over an unsharded, single-part lm_head
bool lm_head_decides(const ifr_state *s, int nc) {
    const ifr_model *m = s->m;
    return !m->comm && !(m->final_softcap > 0.f) && m->lm_head.parts.size() == 1 && nc <= kNMax &&
           !(nc >= ifr_ctx_dense_min(m->ctx) && s->dense) && m->lm_head.parts[0].rows <= 0x7FFFFFFF;
}

// MTP draft of gamma tokens into vtok[b * kNMax + 1 .. gamma] of every request
int mtp_draft(ifr_state *s, int gamma, cudaStream_t st) {
    ifr_model *m = s->m;
    const ifr_model_info &c = m->info;
    const int d = c.hidden, B = s->B;
    const int sc_ld = (int)(sizeof(ifr::EngineScalars) / sizeof(int32_t));
    const int64_t kv_ld = (int64_t)s->max_ctx * m->nkv * c.head_dim;
    ifr::XForm norm_out;  // the MTP head's final norm, applied inside the lm_head GEMV
    norm_out.kind = 1;
    norm_out.w = m->mtp_norm;
    norm_out.eps = c.rms_eps;
    for (int j = 1; j <= gamma; j++) {
        const int32_t *tok = j == 1 ? &s->sc->last_token : s->vtok + (j - 1);
        const int tok_ld = j == 1 ? sc_ld : kNMax;
        // the previous draft's layer output stays in s->x until the fc GEMV below
        // overwrites it, after the prep kernel has read it
        const float *hin = j == 1 ? s->mtp_h : s->x;
        ECHECK(launch_mtp_prep(m->embed.parts[0], tok, tok_ld, hin, m->mtp_norm_e, m->mtp_norm_h, c.rms_eps, d,
                               s->mtp_cat, s->mtp_pos, s->sc, j - 1, B, st),
               "mtp prep");
        int rc = gemv(s, CAT_DRAFT_GEMV, m->mtp_fc, s->mtp_cat, B, s->x, false, st);
        if (rc) return rc;
        if ((rc = layer_forward(s, m->mtp_layer, -1, 1, s->mtp_kc, s->mtp_vc, s->mtp_pos, 1, kv_ld, true, st)))
            return rc;
        // greedy draft token straight into the verify tokens: in the lm_head's
        // epilogue when it runs as one small-N launch, else a separate argmax
        ifr::GemvArgmax am;
        am.cand = s->am_cand;
        am.counter = s->am_count;
        am.out = s->vtok + j;
        am.out_ld = kNMax;
        const bool fused = lm_head_decides(s, B);
        ifr::XForm f = norm_out;
        if (fused) f.am = &am;
        f.rev = j % 2 == 0;  // alternate directions: a draft starts on the rows the previous one left in L2
        if ((rc = gemv(s, CAT_DRAFT_LM_HEAD, m->lm_head, s->x, B, s->logits, false, st, f))) return rc;
        if (!fused) {
            ECHECK(ifr::accept_greedy_fused(s->logits, nullptr, B, 0, c.vocab, s->acc, s->vtok + j, s->acc_scratch,
                                            s->gcount, st, 1, kNMax),
                   "draft argmax");
            s->launches++;
        }
        s->launches++;  // prep
    }
    return IFR_OK;
}

}  // namespace

// ------------------------------------------------------------- C ABI --------
extern "C" {

int ifr_model_load_gguf(ifr_ctx *ctx, const char *path, ifr_model **out) {
    return ifr_model_load_gguf_tp(ctx, path, nullptr, out);
}

int ifr_model_load_gguf_tp(ifr_ctx *ctx, const char *path, ifr_comm *comm, ifr_model **out) {
    if (!ctx || !path || !out) return ifr_fail(IFR_ERR_ARG, "NULL argument");
    *out = nullptr;
    int dev = ifr_ctx_device(ctx), prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(dev);
    Gguf g;
    std::string err;
    if (!g.open_file(path, err)) {
        cudaSetDevice(prev);
        return ifr_fail(IFR_ERR_ARG, "%s: %s", path, err.c_str());
    }
    ifr_model *m = new ifr_model();
    m->ctx = ctx;
    // get_config (LoaderCPU.jl:439-469): "{arch}.key", then "key", then the default
    const std::string arch = g.str.count("general.architecture") ? g.str["general.architecture"] : "qwen";
    auto md = [&](const char *k, double def) {
        std::string a = arch + "." + k;
        if (g.num.count(a)) return g.num[a];
        if (g.num.count(k)) return g.num[k];
        return def;
    };
    ifr_model_info &c = m->info;
    c.hidden = (int)md("embedding_length", 1024);
    c.ffn = (int)md("feed_forward_length", 3584);
    c.n_layers = (int)md("block_count", 24);
    c.n_head = (int)md("attention.head_count", 8);
    c.n_kv_head = (int)md("attention.head_count_kv", 2);
    c.head_dim = (int)md("attention.key_length", 256);
    c.rms_eps = (float)md("attention.layer_norm_rms_epsilon", 1e-6);
    c.rope_theta = (float)md("rope.freq_base", 10000000.0);
    c.context_length = (int)md("context_length", 4096);
    c.conv_kernel = (int)md("ssm.conv_kernel", 4);
    c.rotary_dim = (int)std::lround(c.head_dim * (float)md("rope.partial_rotary_factor", 0.25));  // LoaderCPU.jl:421
    int rc = IFR_OK;
    if (arch == "gemma4") {
        // Gemma4Loader.jl:60-123 (our GGUF keys): sliding window and its layer
        // pattern, softcaps, the two RoPE bases, embed_scale = Float32(sqrt(hidden))
        m->gemma = true;
        m->window = (int)md("attention.sliding_window", 512);
        m->sliding_pattern = (int)md("attention.sliding_window_pattern", 6);
        m->attn_softcap = (float)md("attn_logit_softcapping", 0.0);
        m->final_softcap = (float)md("final_logit_softcapping", 0.0);
        m->rope_theta_swa = (float)md("rope.freq_base_swa", 10000.0);
        c.rope_theta = (float)md("rope.freq_base", 1000000.0);
        m->partial_rotary = (float)md("rope.partial_rotary_factor", 0.25);
        m->embed_scale = (float)std::sqrt((double)c.hidden);
        m->pli = (int)md("embedding_length_per_layer_input", 0);
        if (g.has("mtp.fc.weight")) rc = ifr_fail(IFR_ERR_UNSUPPORTED, "gemma4 models have no MTP head here");
        if (!rc && (m->pli < 0 || m->pli % 32)) rc = ifr_fail(IFR_ERR_ARG, "per-layer input size %d", m->pli);
    }
    auto te = g.t.find("token_embd.weight");
    if (te == g.t.end() || te->second.dims.size() != 2) rc = ifr_fail(IFR_ERR_ARG, "token_embd.weight missing");
    if (!rc) {
        c.vocab = (int)te->second.dims[1];  // actual vocab from the embedding (LoaderCPU.jl:321-322)
        if ((int)te->second.dims[0] != c.hidden) rc = ifr_fail(IFR_ERR_ARG, "embedding width != embedding_length");
    }
    // SSM dims from the first SSM layer (LoaderCPU.jl:549-567)
    for (int i = 0; !rc && i < c.n_layers; i++) {
        const std::string pre = "blk." + std::to_string(i) + ".";
        if (!g.has(pre + "ssm_a")) continue;
        const int heads = (int)g.t[pre + "ssm_a"].nel();
        const int inner = (int)g.t[pre + "attn_gate.weight"].dims[1];
        const int C = (int)g.t[pre + "attn_qkv.weight"].dims[1];
        c.ssm_heads = heads;
        c.ssm_head_dim = inner / heads;
        m->inner = inner;
        m->conv_channels = C;
        if ((C - inner) / (2 * heads) != c.ssm_head_dim)
            rc = ifr_fail(IFR_ERR_UNSUPPORTED, "SSM head k dim != v dim is not supported");
        break;
    }
    if (!rc && m->inner && c.ssm_head_dim != 128 && c.ssm_head_dim != 64)
        rc = ifr_fail(IFR_ERR_UNSUPPORTED, "SSM head dim %d (supported: 64, 128)", c.ssm_head_dim);
    if (!rc && c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256)
        rc = ifr_fail(IFR_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128, 256)", c.head_dim);
    // this rank's share (the whole model for one rank)
    m->comm = comm;
    m->tp_rank = comm_rank(comm);
    m->tp_world = comm_world(comm);
    const int W = m->tp_world, r = m->tp_rank;
    if (!rc && (c.n_head % W || c.n_kv_head % W))
        rc = ifr_fail(IFR_ERR_ARG, "%d query / %d KV heads do not split over %d ranks", c.n_head, c.n_kv_head, W);
    if (!rc && W > 1 && m->inner)
        rc = ifr_fail(IFR_ERR_UNSUPPORTED, "tensor parallelism covers attention-only models (this one has SSM layers)");
    if (!rc && W > 1 && g.has("mtp.fc.weight"))
        rc = ifr_fail(IFR_ERR_UNSUPPORTED, "tensor parallelism with an MTP head is not supported (use a draft model)");
    if (!rc && W > 1 && (c.n_head / W * c.head_dim) % 256)
        rc = ifr_fail(IFR_ERR_ARG, "per-rank attention width %d is not a multiple of 256", c.n_head / W * c.head_dim);
    if (!rc && W > 1 && c.ffn % 256) rc = ifr_fail(IFR_ERR_ARG, "FFN width %d is not a multiple of 256", c.ffn);
    if (!rc) {
        m->nh = c.n_head / W;
        m->nkv = c.n_kv_head / W;
        const int nuf = c.ffn / (W > 1 ? 256 : 1);  // FFN units (256 columns) split as evenly as possible
        const int u0 = (int)((int64_t)r * nuf / W), u1 = (int)((int64_t)(r + 1) * nuf / W);
        const int unit = W > 1 ? 256 : 1;
        m->ffn_off = u0 * unit;
        m->ffn = (u1 - u0) * unit;
        m->vocab_off = (int)((int64_t)r * c.vocab / W);
        m->vocab = (int)((int64_t)(r + 1) * c.vocab / W) - m->vocab_off;
    }
    if (!rc) rc = upload_proj(m, g, {"token_embd.weight"}, &m->embed);
    if (!rc) {
        const std::string lm = g.has("output.weight") ? "output.weight" : "token_embd.weight";
        if (W > 1) {
            Slice sv;
            sv.r0 = m->vocab_off;
            sv.r1 = m->vocab_off + m->vocab;
            rc = upload_proj(m, g, {lm}, &m->lm_head, {sv});
        } else if (g.has("output.weight")) {
            rc = upload_proj(m, g, {"output.weight"}, &m->lm_head);
        } else {
            m->lm_head = m->embed;  // tied (LoaderCPU.jl:411-417)
        }
    }
    if (!rc && m->embed.parts.size() != 1) rc = ifr_fail(IFR_ERR_ARG, "bad embedding");
    if (!rc && m->pli) {
        // per-layer input tables (Gemma4Loader.jl:142-151), whole on every rank
        rc = upload_proj(m, g, {"pli_token_embd.weight"}, &m->pli_token_embd);
        if (!rc) rc = upload_proj(m, g, {"pli_model_proj.weight"}, &m->pli_model_proj);
        if (!rc) rc = upload_f32(m, g, "pli_proj_norm.weight", m->pli, &m->pli_proj_norm);
        const int64_t lp = (int64_t)c.n_layers * m->pli;
        if (!rc && (m->pli_token_embd.parts.size() != 1 || m->pli_token_embd.cols != lp ||
                    m->pli_model_proj.rows != lp || m->pli_model_proj.cols != c.hidden))
            rc = ifr_fail(IFR_ERR_ARG, "per-layer input tables do not match the config");
    }
    if (!rc) rc = upload_f32(m, g, "output_norm.weight", c.hidden, &m->final_norm);
    m->layers.resize(c.n_layers);
    for (int i = 0; !rc && i < c.n_layers; i++) {
        rc = load_layer(m, g, "blk." + std::to_string(i) + ".", m->layers[i], i);
        if (!rc && !m->layers[i].ssm) c.n_attention_layers++;
    }
    if (!rc && g.has("mtp.fc.weight")) {
        m->has_mtp = true;
        rc = upload_proj(m, g, {"mtp.fc.weight"}, &m->mtp_fc);
        if (!rc) rc = upload_f32(m, g, "mtp.pre_fc_norm_embedding.weight", c.hidden, &m->mtp_norm_e);
        if (!rc) rc = upload_f32(m, g, "mtp.pre_fc_norm_hidden.weight", c.hidden, &m->mtp_norm_h);
        if (!rc) rc = upload_f32(m, g, "mtp.norm.weight", c.hidden, &m->mtp_norm);
        if (!rc) rc = load_layer(m, g, "mtp.blk.0.", m->mtp_layer);
        if (!rc && m->mtp_layer.ssm) rc = ifr_fail(IFR_ERR_UNSUPPORTED, "the MTP layer must be an attention layer");
    }
    if (!rc) {
        c.has_mtp = m->has_mtp ? 1 : 0;
        int64_t wb = proj_bytes(m->lm_head);
        for (auto &L : m->layers) wb += proj_bytes(L.proj) + proj_bytes(L.out) + proj_bytes(L.gate_up) + proj_bytes(L.down);
        c.weight_bytes = wb;
    }
    cudaSetDevice(prev);
    if (rc) {
        delete m;
        return rc;
    }
    ifr_ctx_retain(ctx);
    *out = m;
    return IFR_OK;
}

static int model_destroy(ifr_model *m) {
    int prev = 0;
    cudaGetDevice(&prev);
    ifr_ctx *c = m->ctx;
    cudaSetDevice(ifr_ctx_device(c));
    delete m;
    cudaSetDevice(prev);
    ifr_ctx_release(c);
    return IFR_OK;
}

// a model outlives the states built on it: freeing it while states are alive
// only marks it, and the last ifr_state_free completes the destruction
int ifr_model_free(ifr_model *m) {
    if (!m) return IFR_OK;
    m->closing = true;
    return m->states == 0 ? model_destroy(m) : IFR_OK;
}

int ifr_model_get_shard(const ifr_model *m, int32_t *sh) {
    if (!m || !sh) return ifr_fail(IFR_ERR_ARG, "NULL argument");
    const int32_t v[8] = {m->tp_rank, m->tp_world, m->nh, m->nkv, m->ffn, m->ffn_off, m->vocab, m->vocab_off};
    memcpy(sh, v, sizeof v);
    return IFR_OK;
}

int ifr_model_get_info(const ifr_model *m, ifr_model_info *info) {
    if (!m || !info) return ifr_fail(IFR_ERR_ARG, "NULL argument");
    *info = m->info;
    return IFR_OK;
}

int ifr_state_create(ifr_model *m, int max_ctx, ifr_state **out) { return ifr_state_create_batch(m, max_ctx, 1, out); }

int ifr_state_create_batch(ifr_model *m, int max_ctx, int batch, ifr_state **out) {
    if (!m || !out) return ifr_fail(IFR_ERR_ARG, "NULL argument");
    const ifr_model_info &c = m->info;
    if (max_ctx < 1 || max_ctx > c.context_length)
        return ifr_fail(IFR_ERR_ARG, "max_ctx %d outside 1..context_length (%d)", max_ctx, c.context_length);
    if (batch < 1 || batch > IFR_MAX_BATCH) return ifr_fail(IFR_ERR_ARG, "batch %d outside 1..%d", batch, IFR_MAX_BATCH);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(m->ctx));
    ifr_state *s = new ifr_state();
    s->m = m;
    s->B = batch;
    s->max_ctx = max_ctx;
    s->log_cap = max_ctx + 16;
    // one request: columns for a prefill chunk of kPrefillChunk tokens
    const int d = c.hidden, N = batch == 1 ? ifr::kPrefillChunk : kNMax * batch, B = batch;
    int64_t maxproj = (int64_t)(2 * m->nh + 2 * m->nkv) * c.head_dim;
    if (m->conv_channels + m->inner > maxproj) maxproj = m->conv_channels + m->inner;
    const int64_t ymax = std::max<int64_t>(m->inner, (int64_t)m->nh * c.head_dim);
    int rc = IFR_OK;
    auto chk = [&](int r) { if (!rc) rc = r; };
    chk(dalloc(s, &s->sc, B));
    chk(dalloc(s, &s->vtok, N));
    chk(dalloc(s, &s->prompt, (size_t)B * max_ctx));
    chk(dalloc(s, &s->acc, B + 4));
    chk(dalloc(s, &s->outtok, N + B));
    chk(dalloc(s, &s->mtp_pos, B + 4));
    chk(dalloc(s, &s->chunk_pos, 32));
    chk(dalloc(s, &s->log, (size_t)B * s->log_cap));
    chk(dalloc(s, &s->x, (size_t)N * d));
    chk(dalloc(s, &s->xn, (size_t)N * d));
    chk(dalloc(s, &s->proj, (size_t)N * maxproj));
    chk(dalloc(s, &s->y, (size_t)N * ymax));
    chk(dalloc(s, &s->gu, (size_t)N * 2 * m->ffn));
    chk(dalloc(s, &s->hmid, (size_t)N * m->ffn));
    chk(dalloc(s, &s->hid, (size_t)N * d));
    chk(dalloc(s, &s->logits, (size_t)N * m->vocab));
    chk(dalloc(s, &s->cand, (size_t)2 * N * (m->tp_world + 1)));
    chk(dalloc(s, &s->mtp_h, (size_t)B * d));
    chk(dalloc(s, &s->mtp_cat, (size_t)B * 2 * d));
    chk(dalloc(s, &s->gcount, B + 4));
    chk(dalloc(s, &s->am_cand, (size_t)8 * 1024));
    chk(dalloc(s, &s->am_count, 4));
    const int half = m->gemma ? c.head_dim / 2 : c.rotary_dim / 2;
    chk(dalloc(s, &s->rope_cos, (size_t)max_ctx * half));
    chk(dalloc(s, &s->rope_sin, (size_t)max_ctx * half));
    if (m->gemma) {
        chk(dalloc(s, &s->rope_cos_full, (size_t)max_ctx * half));
        chk(dalloc(s, &s->rope_sin_full, (size_t)max_ctx * half));
    }
    if (m->pli) {
        const size_t lp = (size_t)c.n_layers * m->pli;
        chk(dalloc(s, &s->pli_emb, (size_t)N * lp));
        chk(dalloc(s, &s->pli_tmp, (size_t)N * lp));
        chk(dalloc(s, &s->pli_in, (size_t)N * lp));
        chk(dalloc(s, &s->pli_g, (size_t)N * m->pli));
    }
    s->S.assign(c.n_layers, nullptr);
    s->hist.assign(c.n_layers, nullptr);
    s->rq.assign(c.n_layers, nullptr);
    s->rkv.assign(c.n_layers, nullptr);
    s->kc.assign(c.n_layers, nullptr);
    s->vc.assign(c.n_layers, nullptr);
    // bf16 caches (split-KV states only): half the floats, read as uint16
    s->kv16 = ifr_ctx_kv_bf16(m->ctx) && (B > 1 || max_ctx >= kSplitMinCtx);
    const size_t kvn = (size_t)B * max_ctx * m->nkv * c.head_dim / (s->kv16 ? 2 : 1);
    for (int i = 0; !rc && i < c.n_layers; i++) {
        if (m->layers[i].ssm) {
            const int hd = c.ssm_head_dim;
            chk(dalloc(s, &s->S[i], (size_t)B * c.ssm_heads * hd * hd));
            chk(dalloc(s, &s->hist[i], (size_t)B * (c.conv_kernel - 1) * m->conv_channels));
            chk(dalloc(s, &s->rq[i], (size_t)N * m->conv_channels));
            chk(dalloc(s, &s->rkv[i], (size_t)c.ssm_heads * N * (2 * hd + 2)));
        } else {
            chk(dalloc(s, &s->kc[i], kvn));
            chk(dalloc(s, &s->vc[i], kvn));
        }
    }
    // batches and long caches: split-KV attention (key slices spread over the
    // GPU, partial softmax states merged by a second kernel); one request with
    // a short cache keeps the single-launch cluster kernel
    if (B > 1 || max_ctx >= kSplitMinCtx)
        chk(dalloc(s, &s->attn_part, (size_t)ifr::attn_part_floats(m->nh, m->nkv, c.head_dim, B, max_ctx)));
    if (m->has_mtp) {
        chk(dalloc(s, &s->mtp_kc, kvn));
        chk(dalloc(s, &s->mtp_vc, kvn));
    }
    const int64_t accb = ifr::accept_greedy_scratch_bytes(B, kNMax, m->vocab);
    if (!rc) {
        void *p = nullptr;
        cudaError_t e = cudaMalloc(&p, accb);
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "cudaMalloc(accept scratch)");
        else { s->allocs.push_back(p); s->acc_scratch = p; }
    }
    if (!rc && N > kNMax) {
        // dense tensor-core GEMMs of up to B * kNMax columns: the largest plan of all projections
        int64_t need = 0;
        auto plan = [&](const Proj &p) {
            for (auto &q : p.parts) need = std::max(need, ifr::qgemm_dense_scratch_bytes(q, N));
        };
        for (auto &L : m->layers) {
            plan(L.proj);
            plan(L.out);
            plan(L.gate_up);
            plan(L.down);
        }
        plan(m->lm_head);
        if (m->has_mtp) {
            plan(m->mtp_fc);
            plan(m->mtp_layer.proj);
            plan(m->mtp_layer.out);
            plan(m->mtp_layer.gate_up);
            plan(m->mtp_layer.down);
        }
        void *p = nullptr;
        cudaError_t e = cudaMalloc(&p, need);
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "cudaMalloc(dense scratch)");
        else { s->allocs.push_back(p); s->dense = p; s->dense_bytes = need; }
    }
    if (!rc && cudaMallocHost((void **)&s->h_tok, sizeof(int32_t) * (N + 64)) != cudaSuccess)
        rc = ifr_fail(IFR_ERR_NOMEM, "cudaMallocHost failed");
    if (!rc) rc = fused_build(s);
    if (!rc && B > 1 && ifr_ctx_dense_f16(m->ctx)) rc = model_prepare_f16(m, ifr_ctx_stream_of(m->ctx));
    if (!rc && m->gemma) {
        // precompute_rope (Gemma4.jl:205-249): frequencies and angles in
        // Float64, cos / sin as Float32; sliding layers: every pair, theta_swa;
        // full layers: the first gemma_full_pairs pairs, frequencies over head_dim
        const int hd = c.head_dim, np = gemma_full_pairs(m);
        std::vector<float> cs((size_t)max_ctx * half), sn(cs.size()), cf(cs.size()), sf(cs.size());
        for (int k = 0; k < half; k++) {
            const double fs = 1.0 / std::pow((double)m->rope_theta_swa, 2.0 * k / (double)hd);
            const double ff = k < np ? 1.0 / std::pow((double)c.rope_theta, 2.0 * k / (double)hd) : 0.0;
            for (int p = 0; p < max_ctx; p++) {
                cs[(size_t)p * half + k] = (float)std::cos(p * fs);
                sn[(size_t)p * half + k] = (float)std::sin(p * fs);
                cf[(size_t)p * half + k] = (float)std::cos(p * ff);
                sf[(size_t)p * half + k] = (float)std::sin(p * ff);
            }
        }
        if (cudaMemcpy(s->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(s->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(s->rope_cos_full, cf.data(), cf.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(s->rope_sin_full, sf.data(), sf.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            rc = ifr_fail(IFR_ERR_CUDA, "H2D rope tables");
    } else if (!rc) {
        // RoPE tables as the reference builds them (ModelCPU.jl:136-154):
        // inv_freq = Float32(1/theta^(2(i-1)/rd)) in f64; angle = inv_freq * pos in f32
        std::vector<float> cs((size_t)max_ctx * half), sn((size_t)max_ctx * half);
        for (int i = 0; i < half; i++) {
            const float inv = (float)(1.0 / std::pow((double)c.rope_theta, (double)(2 * i) / (double)c.rotary_dim));
            for (int p = 0; p < max_ctx; p++) {
                const float ang = inv * (float)p;
                cs[(size_t)p * half + i] = std::cos(ang);
                sn[(size_t)p * half + i] = std::sin(ang);
            }
        }
        if (cudaMemcpy(s->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(s->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            rc = ifr_fail(IFR_ERR_CUDA, "H2D rope tables");
    }
    if (!rc) {
        ifr::EngineScalars init{};
        init.a_prev = -1;
        std::vector<ifr::EngineScalars> all(B, init);
        if (cudaMemcpy(s->sc, all.data(), sizeof(init) * B, cudaMemcpyHostToDevice) != cudaSuccess)
            rc = ifr_fail(IFR_ERR_CUDA, "H2D scalars");
    }
    cudaSetDevice(prev);
    if (rc) {
        delete s;
        return rc;
    }
    m->states++;
    *out = s;
    return IFR_OK;
}

int ifr_state_free(ifr_state *s) {
    if (!s) return IFR_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(s->m->ctx));
    cudaStreamSynchronize(ifr_ctx_stream_of(s->m->ctx));
    ifr_model *m = s->m;
    delete s;
    cudaSetDevice(prev);
    if (--m->states == 0 && m->closing) return model_destroy(m);
    return IFR_OK;
}

int ifr_state_reset(ifr_state *s) {
    if (!s) return ifr_fail(IFR_ERR_ARG, "NULL argument");
    const ifr_model_info &c = s->m->info;
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    ifr::EngineScalars init{};
    init.a_prev = -1;
    std::vector<ifr::EngineScalars> all(s->B, init);
    ECHECK(cudaStreamSynchronize(st), "reset");
    s->pending = -1;
    ECHECK(cudaMemcpy(s->sc, all.data(), sizeof(init) * s->B, cudaMemcpyHostToDevice), "reset scalars");
    for (int i = 0; i < c.n_layers; i++)
        if (s->S[i]) {
            const int hd = c.ssm_head_dim;
            ECHECK(cudaMemsetAsync(s->S[i], 0, (size_t)s->B * c.ssm_heads * hd * hd * 4, st), "reset state");
            ECHECK(cudaMemsetAsync(s->hist[i], 0, (size_t)s->B * (c.conv_kernel - 1) * s->m->conv_channels * 4, st),
                   "reset conv");
        }
    // the MTP layer attends over positions that only its drafts write: they
    // read as zeros until then, as after creation
    if (s->mtp_kc) {
        const size_t kvb = (size_t)s->B * s->max_ctx * s->m->nkv * c.head_dim * (s->kv16 ? 2 : 4);
        ECHECK(cudaMemsetAsync(s->mtp_kc, 0, kvb, st), "reset mtp cache");
        ECHECK(cudaMemsetAsync(s->mtp_vc, 0, kvb, st), "reset mtp cache");
    }
    ECHECK(cudaStreamSynchronize(st), "reset");
    return IFR_OK;
}

int ifr_prefill(ifr_state *s, const int32_t *tokens, int n, int32_t *first_token) {
    if (!s) return ifr_fail(IFR_ERR_ARG, "NULL state");
    if (s->B != 1) return ifr_fail(IFR_ERR_ARG, "batched state: use ifr_prefill_batch");
    return ifr_prefill_batch(s, tokens, n, first_token);
}

// every request's prompt (n tokens each, row-major [batch][n]) in chunks of up
// to kNMax tokens per request; the last token alone, with logits
int ifr_prefill_batch(ifr_state *s, const int32_t *tokens, int n, int32_t *first_tokens) {
    if (!s || !tokens || n < 1) return ifr_fail(IFR_ERR_ARG, "invalid prefill arguments");
    if (s->pending >= 0) return ifr_fail(IFR_ERR_ARG, "a verify awaits ifr_rollback");
    const ifr_model_info &c = s->m->info;
    const int B = s->B;
    for (int64_t i = 0; i < (int64_t)B * n; i++)
        if (tokens[i] < 0 || tokens[i] >= c.vocab) return ifr_fail(IFR_ERR_ARG, "token %d out of range", tokens[i]);
    if (n + kNMax > s->max_ctx) return ifr_fail(IFR_ERR_ARG, "prompt of %d tokens does not fit max_ctx=%d", n, s->max_ctx);
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(s->m->ctx));
    int rc = IFR_OK;
    // the whole prompt goes to the device once; every chunk's tokens are a
    // device-to-device copy, so the chunks queue without host round trips
    cudaError_t e0 = cudaMemcpyAsync(s->prompt, tokens, sizeof(int32_t) * B * n, cudaMemcpyHostToDevice, st);
    if (e0 != cudaSuccess) rc = ifr_cuda_fail(e0, "H2D prompt");
    // one request: chunks of kPrefillChunk tokens (the SSM layers scan and
    // commit a chunk in one launch); a batch: kNMax tokens per request
    const int chunk = B == 1 ? ifr::kPrefillChunk : kNMax;
    for (int i0 = 0; !rc && i0 < n;) {
        const bool last = i0 == n - 1;
        const int k = last ? 1 : std::min(chunk, n - 1 - i0);
        cudaError_t e = B == 1 ? cudaMemcpyAsync(s->vtok, s->prompt + i0, sizeof(int32_t) * k,
                                                 cudaMemcpyDeviceToDevice, st)
                               : cudaMemcpy2DAsync(s->vtok, sizeof(int32_t) * kNMax, s->prompt + i0,
                                                   sizeof(int32_t) * n, sizeof(int32_t) * k, B,
                                                   cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) { rc = ifr_cuda_fail(e, "prompt chunk"); break; }
        s->prefill_chunk = k > kNMax;
        rc = target_forward(s, k, last, false, st);
        s->prefill_chunk = false;
        if (!rc)
            ifr::commit(s->sc, s->acc, s->outtok, k, k > kNMax ? 2 : 1, nullptr, nullptr, c.hidden, s->log,
                        s->log_cap, B, st);
        if (!rc && last) {
            rc = greedy_accept(s, nullptr, 0, B, 0, s->outtok, 1, st);
            if (rc) break;
            e = ifr::launch_k(prefill_finish_kernel, dim3(B), dim3(256), 0, st, s->sc, (const int32_t *)s->outtok,
                              (const float *)s->hid, s->mtp_h, (int)c.hidden, s->log, (int)s->log_cap);
            if (e != cudaSuccess) { rc = ifr_cuda_fail(e, "prefill finish"); break; }
        }
        i0 += k;
    }
    if (!rc && cudaStreamSynchronize(st) != cudaSuccess) rc = ifr_cuda_fail(cudaGetLastError(), "prefill");
    if (!rc && first_tokens) {
        cudaError_t e = cudaMemcpy(first_tokens, s->outtok, sizeof(int32_t) * B, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "D2H first token");
    }
    cudaSetDevice(prev);
    return rc;
}

}  // extern "C"

namespace {

// draft-model steps: request b's token j of the target's verify tokens becomes
// the draft state's next input
__global__ void copy_token_kernel(int32_t *dst, const int32_t *src, int B) {
    ifr::pdl_trigger();
    ifr::pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) dst[(int64_t)b * kNMax] = src[(int64_t)b * kNMax];
}
// the draft state follows the target: its last token and position (positions
// past the committed ones are overwritten by the next step; attention only)
__global__ void draft_sync_kernel(ifr::EngineScalars *draft, const ifr::EngineScalars *target, int B) {
    ifr::pdl_trigger();
    ifr::pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) {
        draft[b].last_token = target[b].last_token;
        draft[b].pos = target[b].pos;
        draft[b].a_prev = -1;
    }
}

int spec_step_device(ifr_state *s, int gamma, bool mtp, cudaStream_t st);

// one speculative step with a separate draft model (SpeculativeDecoding.jl's
// draft -> verify -> accept loop with the draft model's greedy tokens): the
// draft feeds [last, d1 .. d_gamma] (gamma + 1 single-token forwards, so that
// its cache holds every token the target may commit), its argmaxes d1..d_gamma
// go into the target's verify tokens; then verify, accept, commit, and the
// draft is re-synced to the target's position and last token
int draft_step_device(ifr_state *t, ifr_state *d, int gamma, cudaStream_t st) {
    const int B = t->B;
    const ifr_model_info &dc = d->m->info;
    ECHECK(ifr::launch_k(draft_sync_kernel, dim3((B + 127) / 128), dim3(128), 0, st, d->sc,
                         (const ifr::EngineScalars *)t->sc, B),
           "draft sync");
    for (int j = 1; j <= gamma + 1; j++) {
        if (j > 1)
            ECHECK(ifr::launch_k(copy_token_kernel, dim3((B + 127) / 128), dim3(128), 0, st, d->vtok,
                                 (const int32_t *)(t->vtok + (j - 1)), B),
                   "draft input");
        int rc = target_forward(d, 1, j <= gamma, j == 1, st);
        if (rc) return rc;
        if (j <= gamma) {
            rc = greedy_accept(d, nullptr, 0, B, 0, t->vtok + j, kNMax, st);
            if (rc) return rc;
        }
        ifr::commit(d->sc, d->acc, d->outtok, 1, true, nullptr, nullptr, dc.hidden, d->log, d->log_cap, B, st);
        d->launches += 2;
    }
    int rc = spec_step_device(t, gamma, false, st);
    if (rc) return rc;
    ECHECK(ifr::launch_k(draft_sync_kernel, dim3((B + 127) / 128), dim3(128), 0, st, d->sc,
                         (const ifr::EngineScalars *)t->sc, B),
           "draft sync");
    return IFR_OK;
}

// the device work of one spec step (capturable): MTP drafts (or drafts
// already in vtok[b * kNMax + 1 .. gamma]), verify, greedy accept, commit
int spec_step_device(ifr_state *s, int gamma, bool mtp, cudaStream_t st) {
    const ifr_model_info &c = s->m->info;
    const int B = s->B;
    int rc = IFR_OK;
    if (gamma > 0 && mtp) rc = mtp_draft(s, gamma, st);
    // greedy acceptance in the lm_head's epilogue when it runs as one small-N
    // launch (one request), else its own launch
    ifr::GemvArgmax am;
    am.cand = s->am_cand;
    am.counter = s->am_count;
    am.drafts = s->vtok + 1;
    am.draft_ld = kNMax;
    am.G = gamma;
    am.acc = s->acc;
    am.out = s->outtok;
    am.out_ld = gamma + 1;
    const bool fused = lm_head_decides(s, B * (gamma + 1));
    if (!rc) rc = target_forward(s, gamma + 1, true, true, st, fused ? &am : nullptr);
    if (!rc && !fused) {
        rc = greedy_accept(s, s->vtok + 1, kNMax, B, gamma, s->outtok, gamma + 1, st);
        s->launches++;
    }
    if (!rc)
        ifr::commit(s->sc, s->acc, s->outtok, gamma + 1, false, s->hid, s->mtp_h, c.hidden, s->log, s->log_cap, B, st);
    s->launches++;  // commit
    return rc;
}
}  // namespace

extern "C" {

int ifr_spec_step(ifr_state *s, int gamma, const int32_t *drafts) {
    if (!s) return ifr_fail(IFR_ERR_ARG, "NULL state");
    if (s->pending >= 0) return ifr_fail(IFR_ERR_ARG, "a verify awaits ifr_rollback");
    if (gamma < 0 || gamma + 1 > kNMax) return ifr_fail(IFR_ERR_ARG, "gamma must be in 0..%d", kNMax - 1);
    if (gamma > 0 && !drafts && !s->m->has_mtp) return ifr_fail(IFR_ERR_ARG, "no drafts given and the model has no MTP head");
    const ifr_model_info &c = s->m->info;
    const int B = s->B;
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(s->m->ctx));
    int rc = IFR_OK;
    if (gamma > 0 && drafts) {
        for (int64_t i = 0; i < (int64_t)B * gamma; i++)
            if (drafts[i] < 0 || drafts[i] >= c.vocab) { cudaSetDevice(prev); return ifr_fail(IFR_ERR_ARG, "draft token out of range"); }
        cudaError_t e = cudaStreamSynchronize(st);  // staging buffer reuse
        if (e == cudaSuccess) {
            // drafts [batch][gamma] into vtok[b * kNMax + 1 ..]; slot 0 is set on the device
            for (int b = 0; b < B; b++) memcpy(s->h_tok + (int64_t)b * kNMax + 1, drafts + (int64_t)b * gamma, sizeof(int32_t) * gamma);
            for (int b = 0; b < B && e == cudaSuccess; b++)
                e = cudaMemcpyAsync(s->vtok + (int64_t)b * kNMax + 1, s->h_tok + (int64_t)b * kNMax + 1,
                                    sizeof(int32_t) * gamma, cudaMemcpyHostToDevice, st);
        }
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "H2D drafts");
        if (!rc) rc = spec_step_device(s, gamma, false, st);
    } else {
        rc = spec_step_device(s, gamma, true, st);
    }
    if (!rc) {
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "spec step launch");
    }
    cudaSetDevice(prev);
    return rc;
}

namespace {
int check_draft_pair(ifr_state *t, ifr_state *d, int gamma) {
    if (!t || !d) return ifr_fail(IFR_ERR_ARG, "NULL state");
    if (gamma < 1 || gamma + 1 > kNMax) return ifr_fail(IFR_ERR_ARG, "gamma must be in 1..%d", kNMax - 1);
    if (t->B != d->B) return ifr_fail(IFR_ERR_ARG, "target batch %d != draft batch %d", t->B, d->B);
    if (t->m->ctx != d->m->ctx) return ifr_fail(IFR_ERR_ARG, "target and draft must share a context");
    if (d->m->inner || d->m->comm) return ifr_fail(IFR_ERR_UNSUPPORTED, "the draft model must be attention-only and unsharded");
    if (d->m->info.vocab != t->m->info.vocab) return ifr_fail(IFR_ERR_ARG, "draft and target vocabularies differ");
    return IFR_OK;
}
}  // namespace

int ifr_spec_step_draft(ifr_state *t, ifr_state *d, int gamma) {
    int rc = check_draft_pair(t, d, gamma);
    if (rc) return rc;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(t->m->ctx));
    rc = draft_step_device(t, d, gamma, ifr_ctx_stream_of(t->m->ctx));
    if (!rc) {
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "draft step launch");
    }
    cudaSetDevice(prev);
    return rc;
}

int ifr_spec_graph_draft(ifr_state *t, ifr_state *d, int gamma, int steps) {
    int rc = check_draft_pair(t, d, gamma);
    if (rc) return rc;
    if (steps < 1) return ifr_fail(IFR_ERR_ARG, "steps must be >= 1");
    cudaStream_t st = ifr_ctx_stream_of(t->m->ctx);
    if (st == nullptr) return ifr_fail(IFR_ERR_ARG, "the context stream is the legacy default stream, which cannot be captured");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(t->m->ctx));
    if (t->graph_exec) { cudaGraphExecDestroy(t->graph_exec); t->graph_exec = nullptr; }
    if (t->graph) { cudaGraphDestroy(t->graph); t->graph = nullptr; }
    cudaError_t e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) rc = ifr_cuda_fail(e, "begin capture");
    for (int i = 0; !rc && i < steps; i++) rc = draft_step_device(t, d, gamma, st);
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(st, &g);
    if (!rc && e != cudaSuccess) rc = ifr_cuda_fail(e, "end capture");
    if (!rc) {
        t->graph = g;
        e = cudaGraphInstantiate(&t->graph_exec, g, 0);
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "graph instantiate");
    } else if (g) {
        cudaGraphDestroy(g);
    }
    cudaSetDevice(prev);
    return rc;
}

// ---- the step in parts: draft, verify, acceptance by the caller, commit ----
int ifr_draft_mtp(ifr_state *s, int gamma, int32_t *drafts_out) {
    if (!s) return ifr_fail(IFR_ERR_ARG, "NULL state");
    if (gamma < 1 || gamma + 1 > kNMax) return ifr_fail(IFR_ERR_ARG, "gamma must be in 1..%d", kNMax - 1);
    if (!s->m->has_mtp) return ifr_fail(IFR_ERR_ARG, "the model has no MTP head");
    if (s->pending >= 0) return ifr_fail(IFR_ERR_ARG, "a verify awaits ifr_rollback");
    const int B = s->B;
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(s->m->ctx));
    int rc = mtp_draft(s, gamma, st);
    if (!rc && drafts_out) {
        cudaError_t e = cudaMemcpy2DAsync(drafts_out, sizeof(int32_t) * gamma, s->vtok + 1, sizeof(int32_t) * kNMax,
                                          sizeof(int32_t) * gamma, B, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "D2H drafts");
    }
    cudaSetDevice(prev);
    return rc;
}

int ifr_verify_step(ifr_state *s, int gamma, const int32_t *drafts, float *logits_out) {
    if (!s) return ifr_fail(IFR_ERR_ARG, "NULL state");
    if (gamma < 0 || gamma + 1 > kNMax) return ifr_fail(IFR_ERR_ARG, "gamma must be in 0..%d", kNMax - 1);
    if (s->pending >= 0) return ifr_fail(IFR_ERR_ARG, "a verify awaits ifr_rollback");
    const ifr_model_info &c = s->m->info;
    const int B = s->B;
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(s->m->ctx));
    int rc = IFR_OK;
    if (gamma > 0 && drafts) {
        for (int64_t i = 0; i < (int64_t)B * gamma; i++)
            if (drafts[i] < 0 || drafts[i] >= c.vocab) { cudaSetDevice(prev); return ifr_fail(IFR_ERR_ARG, "draft token out of range"); }
        cudaError_t e = cudaStreamSynchronize(st);  // staging buffer reuse
        for (int b = 0; b < B && e == cudaSuccess; b++) {
            memcpy(s->h_tok + (int64_t)b * kNMax + 1, drafts + (int64_t)b * gamma, sizeof(int32_t) * gamma);
            e = cudaMemcpyAsync(s->vtok + (int64_t)b * kNMax + 1, s->h_tok + (int64_t)b * kNMax + 1,
                                sizeof(int32_t) * gamma, cudaMemcpyHostToDevice, st);
        }
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "H2D drafts");
    }
    if (!rc) rc = target_forward(s, gamma + 1, true, true, st);
    if (!rc && logits_out) {
        cudaError_t e = cudaMemcpyAsync(logits_out, s->logits, sizeof(float) * B * (gamma + 1) * s->m->vocab,
                                        cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "logits copy");
    }
    if (!rc) s->pending = gamma;
    cudaSetDevice(prev);
    return rc;
}

int ifr_rollback(ifr_state *s, const int32_t *accept_count, const int32_t *tokens) {
    if (!s || !accept_count || !tokens) return ifr_fail(IFR_ERR_ARG, "NULL argument");
    if (s->pending < 0) return ifr_fail(IFR_ERR_ARG, "no verify awaits ifr_rollback");
    const ifr_model_info &c = s->m->info;
    const int B = s->B, G = s->pending;
    for (int b = 0; b < B; b++) {
        const int a = accept_count[b];
        if (a < 0 || a > G) return ifr_fail(IFR_ERR_ARG, "accept count %d of request %d outside 0..%d", a, b, G);
        for (int i = 0; i <= a; i++) {
            const int t = tokens[(int64_t)b * (G + 1) + i];
            if (t < 0 || t >= c.vocab) return ifr_fail(IFR_ERR_ARG, "token %d out of range", t);
        }
    }
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(s->m->ctx));
    int rc = IFR_OK;
    // staged through the pinned buffer (B * kNMax + 64 ints): tokens, then counts
    cudaError_t e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) {
        memcpy(s->h_tok, tokens, sizeof(int32_t) * B * (G + 1));
        e = cudaMemcpyAsync(s->outtok, s->h_tok, sizeof(int32_t) * B * (G + 1), cudaMemcpyHostToDevice, st);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) {
        memcpy(s->h_tok, accept_count, sizeof(int32_t) * B);
        e = cudaMemcpyAsync(s->acc, s->h_tok, sizeof(int32_t) * B, cudaMemcpyHostToDevice, st);
    }
    if (e != cudaSuccess) rc = ifr_cuda_fail(e, "H2D acceptance");
    if (!rc) {
        ifr::commit(s->sc, s->acc, s->outtok, G + 1, false, s->hid, s->mtp_h, c.hidden, s->log, s->log_cap, B, st);
        e = cudaGetLastError();
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "commit");
        else s->pending = -1;
    }
    cudaSetDevice(prev);
    return rc;
}

int ifr_spec_graph(ifr_state *s, int gamma, int steps) {
    if (!s || steps < 1) return ifr_fail(IFR_ERR_ARG, "invalid graph arguments");
    if (gamma < 0 || gamma + 1 > kNMax) return ifr_fail(IFR_ERR_ARG, "gamma must be in 0..%d", kNMax - 1);
    if (gamma > 0 && !s->m->has_mtp) return ifr_fail(IFR_ERR_ARG, "the model has no MTP head");
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    if (st == nullptr) return ifr_fail(IFR_ERR_ARG, "the context stream is the legacy default stream, which cannot be captured");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(s->m->ctx));
    if (s->graph_exec) { cudaGraphExecDestroy(s->graph_exec); s->graph_exec = nullptr; }
    if (s->graph) { cudaGraphDestroy(s->graph); s->graph = nullptr; }
    int rc = IFR_OK;
    cudaError_t e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) rc = ifr_cuda_fail(e, "begin capture");
    for (int i = 0; !rc && i < steps; i++) rc = spec_step_device(s, gamma, true, st);
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(st, &g);
    if (!rc && e != cudaSuccess) rc = ifr_cuda_fail(e, "end capture");
    if (!rc) {
        s->graph = g;
        e = cudaGraphInstantiate(&s->graph_exec, g, 0);
        if (e != cudaSuccess) rc = ifr_cuda_fail(e, "graph instantiate");
    } else if (g) {
        cudaGraphDestroy(g);
    }
    cudaSetDevice(prev);
    return rc;
}

int ifr_spec_graph_launch(ifr_state *s) {
    if (!s || !s->graph_exec) return ifr_fail(IFR_ERR_ARG, "no captured graph (call ifr_spec_graph first)");
    if (s->pending >= 0) return ifr_fail(IFR_ERR_ARG, "a verify awaits ifr_rollback");
    ECHECK(cudaGraphLaunch(s->graph_exec, ifr_ctx_stream_of(s->m->ctx)), "graph launch");
    return IFR_OK;
}

int ifr_state_profile(ifr_state *s, int enable) {
    if (!s) return ifr_fail(IFR_ERR_ARG, "NULL state");
    s->prof = enable != 0;
    s->recs.clear();
    s->ev_next = 0;
    return IFR_OK;
}

int ifr_state_profile_read(ifr_state *s, double *ms, int64_t *bytes, int *count, int64_t *launches) {
    if (!s) return ifr_fail(IFR_ERR_ARG, "NULL state");
    ECHECK(cudaStreamSynchronize(ifr_ctx_stream_of(s->m->ctx)), "sync");
    for (int k = 0; k < CAT_NCAT; k++) {
        if (ms) ms[k] = 0;
        if (bytes) bytes[k] = 0;
        if (count) count[k] = 0;
    }
    int failed = 0;
    for (auto &r : s->recs) {
        float t = 0.f;
        if (cudaEventElapsedTime(&t, s->ev_pool[r.ev0], s->ev_pool[r.ev0 + 1]) != cudaSuccess) {
            failed++;
            continue;
        }
        if (ms) ms[r.cat] += t;
        if (bytes) bytes[r.cat] += r.bytes;
        if (count) count[r.cat] += 1;
    }
    cudaGetLastError();  // a failed elapsed-time query must not surface in a later launch check
    if (launches) *launches = s->launches;
    if (failed) return ifr_fail(IFR_ERR_UNSUPPORTED, "%d timings unavailable (events recorded inside a CUDA graph cannot be timed); profile eagerly", failed);
    return IFR_OK;
}

int ifr_state_fused_trace(ifr_state *s, int max_phases, int *kinds, double *us, int *n_phases) {
    if (!s || !n_phases) return ifr_fail(IFR_ERR_ARG, "NULL argument");
    *n_phases = 0;
    const int n = s->fused_last;
    if (!s->prof || n < 1 || !s->fused_ph[n]) return IFR_OK;  // nothing traced
    const int np = s->fused_np[n], nc = ifr::fused_ctas();
    std::vector<unsigned long long> t(4 * (size_t)np * (nc + 1) + 1);
    ECHECK(cudaStreamSynchronize(ifr_ctx_stream_of(s->m->ctx)), "fused trace sync");
    ECHECK(cudaMemcpy(t.data(), s->fused_trace, t.size() * sizeof(t[0]), cudaMemcpyDeviceToHost), "fused trace D2H");
    const int k = std::min(np, max_phases);
    auto d = [](unsigned long long a, unsigned long long b) { return (double)(long long)(b - a) * 1e-3; };
    const unsigned long long *bar = t.data() + 4 * (size_t)np * nc, end = t[4 * (size_t)np * nc + 4 * np];
    for (int i = 0; i < k; i++) {
        const unsigned long long *c0 = t.data() + 4 * (size_t)i * nc;
        const unsigned long long next = i + 1 < np ? t[4 * (size_t)(i + 1) * nc] : end;
        // the slowest CTA of the phase (its own start to its end)
        int w = 0;
        for (int c = 1; c < nc; c++)
            if (c0[4 * c + 3] - c0[4 * c] > c0[4 * w + 3] - c0[4 * w]) w = c;
        const unsigned long long *cw = c0 + 4 * w;
        if (kinds) kinds[i] = s->fused_kinds[n][i];
        if (us) {
            us[6 * i] = d(c0[0], next);
            us[6 * i + 1] = d(cw[0], cw[1]);
            us[6 * i + 2] = d(cw[1], cw[2]);
            us[6 * i + 3] = d(cw[2], cw[3]);
            us[6 * i + 4] = d(cw[3], next);
            us[6 * i + 5] = d(cw[0], cw[3]);
        }
        if (us && max_phases >= 2 * np) {
            const unsigned long long *b = bar + 4 * i;
            double *o = us + 6 * np + 4 * i;
            if (b[0] && b[3]) {
                o[0] = d(b[0], b[3]);
                o[1] = d(b[3], b[1]);
                o[2] = d(b[1], b[2]);
                o[3] = d(b[2], next);
            } else {
                o[0] = o[1] = o[2] = o[3] = 0;
            }
        }
    }
    *n_phases = k;
    return IFR_OK;
}

int ifr_gemv_pass(ifr_state *s, int ncols) {
    if (!s || ncols < 1 || ncols > kNMax * s->B) return ifr_fail(IFR_ERR_ARG, "ncols must be in 1..%d", kNMax * s->B);
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ifr_ctx_device(s->m->ctx));
    int rc = IFR_OK;
    const ifr_model_info &c = s->m->info;
    ifr::XForm norm;
    norm.kind = 1;
    norm.eps = c.rms_eps;
    ifr::XForm swiglu;
    swiglu.kind = 2;
    swiglu.ldx = 2 * (int64_t)s->m->ffn;
    // the verify's GEMVs with their fused input transforms; outputs go to
    // buffers a spec step rewrites before it reads them (proj, gu, hid): the
    // caches, SSM states and residual stream are not changed
    for (auto &L : s->m->layers) {
        norm.w = L.attn_norm;
        if (!rc) rc = gemv(s, CAT_LAYER_GEMV, L.proj, s->xn, ncols, s->proj, false, st, norm);
        if (!rc) rc = gemv(s, CAT_LAYER_GEMV, L.out, s->y, ncols, s->hid, false, st);
        norm.w = L.post_norm;
        if (L.gate_up.glu) {
            ifr::XForm glu = norm;
            glu.ep = 1;
            if (!rc) rc = gemv(s, CAT_LAYER_GEMV, L.gate_up, s->xn, ncols, s->hmid, false, st, glu);
            if (!rc) rc = gemv(s, CAT_LAYER_GEMV, L.down, s->hmid, ncols, s->hid, false, st);
        } else {
            if (!rc) rc = gemv(s, CAT_LAYER_GEMV, L.gate_up, s->xn, ncols, s->gu, false, st, norm);
            if (!rc) rc = gemv(s, CAT_LAYER_GEMV, L.down, s->gu, ncols, s->hid, false, st, swiglu);
        }
    }
    if (!rc) rc = gemv(s, CAT_LM_HEAD, s->m->lm_head, s->hid, ncols, s->logits, false, st);
    cudaSetDevice(prev);
    return rc;
}

int ifr_state_read(ifr_state *s, int32_t *tokens, int max_tokens, int *n_tokens, int32_t *scalars) {
    return ifr_state_read_request(s, 0, tokens, max_tokens, n_tokens, scalars);
}

int ifr_state_read_request(ifr_state *s, int b, int32_t *tokens, int max_tokens, int *n_tokens, int32_t *scalars) {
    if (!s) return ifr_fail(IFR_ERR_ARG, "NULL state");
    if (b < 0 || b >= s->B) return ifr_fail(IFR_ERR_ARG, "request %d outside 0..%d", b, s->B - 1);
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    ECHECK(cudaStreamSynchronize(st), "sync");
    ifr::EngineScalars h{};
    ECHECK(cudaMemcpy(&h, s->sc + b, sizeof h, cudaMemcpyDeviceToHost), "D2H scalars");
    if (n_tokens) *n_tokens = h.n_log;
    if (tokens && max_tokens > 0 && h.n_log > 0)
        ECHECK(cudaMemcpy(tokens, s->log + (int64_t)b * s->log_cap, sizeof(int32_t) * std::min(max_tokens, h.n_log),
                          cudaMemcpyDeviceToHost),
               "D2H log");
    if (scalars) {
        scalars[0] = h.pos;
        scalars[1] = h.last_accept;
        scalars[2] = h.steps;
        scalars[3] = h.last_token;
    }
    return IFR_OK;
}

int ifr_state_last_verify(ifr_state *s, float *logits, float *hidden, int32_t *tokens, int *n_cols) {
    if (!s) return ifr_fail(IFR_ERR_ARG, "NULL state");
    const ifr_model_info &c = s->m->info;
    cudaStream_t st = ifr_ctx_stream_of(s->m->ctx);
    ECHECK(cudaStreamSynchronize(st), "sync");
    const int n = s->last_n, B = s->B;
    if (n_cols) *n_cols = n;
    if (logits)
        ECHECK(cudaMemcpy(logits, s->logits, sizeof(float) * B * n * s->m->vocab, cudaMemcpyDeviceToHost), "D2H logits");
    if (hidden)
        ECHECK(cudaMemcpy(hidden, s->hid, sizeof(float) * B * n * c.hidden, cudaMemcpyDeviceToHost), "D2H hidden");
    for (int b = 0; tokens && b < B; b++)
        ECHECK(cudaMemcpy(tokens + (int64_t)b * n, s->vtok + (int64_t)b * kNMax, sizeof(int32_t) * n,
                          cudaMemcpyDeviceToHost),
               "D2H tokens");
    return IFR_OK;
}

}  // extern "C"
