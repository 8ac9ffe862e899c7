/* .mlb loading for the CUDA build, written from the format's specification
 * (reference docs/file-format.md: the header table, the body's array order,
 * the loader's validation table) with the reference's status codes
 * (core/ml.h:7-14).
 *
 * Two tables drive it. HEADER lists every header field with its offset, its
 * type, where it lands in kc_config and the check the specification gives
 * it; the checks that tie several fields together follow in cross_checks().
 * body_schedule() then lists the arrays the header implies, in file order,
 * and one walker places them on their 64-byte boundaries, checks that the
 * file holds them and that no Q8 quant is -128. The arrays stay host views
 * into the mapping until kc_model_upload. */
#include <cmath>
#include <cstddef>
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "kc_internal.h"

namespace kc {

namespace {

constexpr uint32_t DIM_LIMIT = 65536;        /* dim, n_layers, heads, hidden_dim, head_dim, q_dim */
constexpr uint32_t TOKEN_LIMIT = 1u << 24;   /* vocab, max_seq, sliding_window */
constexpr size_t ALIGN = 64;                 /* every array starts on this boundary */
constexpr size_t HEADER_BYTES = 256;
constexpr unsigned LAYER_SLIDING = 1, LAYER_LOCAL_ROPE = 2;   /* per-layer flag bits */

/* What a field's check accepts; the status a failure returns is in the row. */
enum Rule {
    ANY,          /* no check of its own */
    DIM,          /* 1 .. DIM_LIMIT */
    TOKENS,       /* 1 .. TOKEN_LIMIT */
    TOKENS0,      /* 0 .. TOKEN_LIMIT */
    DIM0,         /* 0 .. DIM_LIMIT */
    FLAG,         /* 0 or 1 */
    WTYPE,        /* 1 (Q8_0) or 2 (Q4_0) */
    ROPE,         /* 0 .. 3 */
    MASK,         /* bits of the seven matrix classes only */
    POSITIVE,     /* finite and > 0 */
    NONNEG,       /* finite and >= 0 */
};

struct Field {
    uint32_t offset;
    bool is_float;
    int kc_config::*i;      /* integer destination, or nullptr */
    float kc_config::*f;    /* float destination, or nullptr */
    Rule rule;
    int status;             /* status when the rule fails */
};

/* Header fields in offset order (file-format.md, "Header"). */
const Field HEADER[] = {
    { 8, false, &kc_config::dim, nullptr, DIM, KC_E_SHAPE },
    { 12, false, &kc_config::n_layers, nullptr, DIM, KC_E_SHAPE },
    { 16, false, &kc_config::n_heads, nullptr, DIM, KC_E_SHAPE },
    { 20, false, &kc_config::n_kv_heads, nullptr, DIM, KC_E_SHAPE },
    { 24, false, &kc_config::hidden_dim, nullptr, DIM, KC_E_SHAPE },
    { 28, false, &kc_config::vocab, nullptr, TOKENS, KC_E_SHAPE },
    { 32, false, &kc_config::max_seq, nullptr, TOKENS, KC_E_SHAPE },
    { 36, true, nullptr, &kc_config::rope_theta, POSITIVE, KC_E_FORMAT },
    { 40, true, nullptr, &kc_config::norm_eps, NONNEG, KC_E_FORMAT },
    { 44, false, &kc_config::wtype, nullptr, WTYPE, KC_E_FORMAT },
    { 52, false, &kc_config::rope_type, nullptr, ROPE, KC_E_FORMAT },
    { 56, true, nullptr, &kc_config::rope_factor, ANY, KC_E_FORMAT },
    { 60, true, nullptr, &kc_config::rope_low_freq_factor, ANY, KC_E_FORMAT },
    { 64, true, nullptr, &kc_config::rope_high_freq_factor, ANY, KC_E_FORMAT },
    { 68, false, &kc_config::rope_orig_max_seq, nullptr, ANY, KC_E_FORMAT },
    { 72, false, nullptr, nullptr, MASK, KC_E_FORMAT },   /* q8_mask: unsigned, stored below */
    { 76, false, &kc_config::qkv_bias, nullptr, FLAG, KC_E_FORMAT },
    { 80, false, &kc_config::head_dim, nullptr, DIM0, KC_E_SHAPE },
    { 84, false, &kc_config::qk_norm, nullptr, FLAG, KC_E_FORMAT },
    { 88, true, nullptr, &kc_config::rope_attn_factor, NONNEG, KC_E_FORMAT },
    { 92, false, &kc_config::sliding_window, nullptr, TOKENS0, KC_E_FORMAT },
    { 96, false, &kc_config::layer_flags, nullptr, FLAG, KC_E_FORMAT },
    { 100, true, nullptr, &kc_config::rope_local_theta, NONNEG, KC_E_FORMAT },
    { 104, false, &kc_config::act, nullptr, FLAG, KC_E_FORMAT },
    { 108, false, &kc_config::post_norms, nullptr, FLAG, KC_E_FORMAT },
    { 112, true, nullptr, &kc_config::embed_scale, NONNEG, KC_E_FORMAT },
    { 116, true, nullptr, &kc_config::attn_scale, NONNEG, KC_E_FORMAT },
    { 120, false, &kc_config::scale_f16, nullptr, FLAG, KC_E_FORMAT },
    { 124, true, nullptr, &kc_config::attn_softcap, NONNEG, KC_E_FORMAT },
    { 128, true, nullptr, &kc_config::final_softcap, NONNEG, KC_E_FORMAT },
};

uint32_t le32(const uint8_t *p) {
    return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}

float lef(const uint8_t *p) {
    const uint32_t u = le32(p);
    float v;
    std::memcpy(&v, &u, sizeof v);
    return v;
}

/* Finite and below a bound that keeps every derived product finite. */
bool sane(float v) { return std::isfinite(v) && std::fabs(v) < 1e30f; }

bool accepts(Rule r, uint32_t u, float f) {
    switch (r) {
    case ANY: return true;
    case DIM: return u >= 1 && u <= DIM_LIMIT;
    case TOKENS: return u >= 1 && u <= TOKEN_LIMIT;
    case TOKENS0: return u <= TOKEN_LIMIT;
    case DIM0: return u <= DIM_LIMIT;
    case FLAG: return u <= 1;
    case WTYPE: return u == KC_Q8_0 || u == KC_Q4_0;
    case ROPE: return u <= 3;
    case MASK: return (u & ~127u) == 0;
    case POSITIVE: return sane(f) && f > 0.0f;
    case NONNEG: return sane(f) && f >= 0.0f;
    }
    return false;
}

/* Rules over several fields (file-format.md, "Validation done by the loader"),
 * after every field passed its own. */
int cross_checks(kc_config &c) {
    if (c.vocab < 3) return KC_E_SHAPE;   /* ids 1 and 2 are BOS and EOS */
    if (c.wtype == KC_Q8_0 && c.q8_mask) return KC_E_FORMAT;
    /* RoPE scaling parameters per kind; rope_attn_factor belongs to yarn alone */
    const float f = c.rope_factor, lo = c.rope_low_freq_factor, hi = c.rope_high_freq_factor;
    if (c.rope_type != KC_ROPE_YARN && c.rope_attn_factor != 0.0f) return KC_E_FORMAT;
    switch (c.rope_type) {
    case KC_ROPE_LLAMA3:
        if (!(sane(f) && f > 0.0f && sane(lo) && lo > 0.0f && sane(hi) && hi > lo && c.rope_orig_max_seq > 0))
            return KC_E_FORMAT;
        break;
    case KC_ROPE_LINEAR:
        if (!(sane(f) && f > 0.0f)) return KC_E_FORMAT;
        break;
    case KC_ROPE_YARN:   /* lo holds beta_fast, hi beta_slow */
        if (!(sane(f) && f > 0.0f && sane(hi) && hi > 0.0f && sane(lo) && lo > hi && c.rope_orig_max_seq > 0 &&
              c.rope_attn_factor > 0.0f))
            return KC_E_FORMAT;
        break;
    default: break;
    }
    /* shapes */
    if (c.dim % KC_QK || c.hidden_dim % KC_QK) return KC_E_SHAPE;
    if (c.n_heads % c.n_kv_heads) return KC_E_SHAPE;
    if (c.head_dim == 0) {
        if (c.dim % c.n_heads) return KC_E_SHAPE;
        c.head_dim = c.dim / c.n_heads;
    }
    const uint64_t q_dim = (uint64_t)c.head_dim * (uint64_t)c.n_heads;
    if (c.head_dim % 2 || q_dim % KC_QK || q_dim > DIM_LIMIT) return KC_E_SHAPE;
    c.q_dim = (int)q_dim;
    c.kv_dim = c.head_dim * c.n_kv_heads;
    /* defaults the specification gives for a zero field */
    if (c.embed_scale == 0.0f) c.embed_scale = 1.0f;
    if (c.attn_scale == 0.0f) c.attn_scale = 1.0f / std::sqrt((float)c.head_dim);
    return KC_OK;
}

/* ---- the body */

enum Kind { BYTES, FLOATS, MATRIX };

struct Entry {
    Kind kind;
    size_t count;              /* BYTES / FLOATS: elements */
    int rows, cols;            /* MATRIX */
    unsigned cls;              /* MATRIX: q8_mask class bits */
    const void **dst;          /* BYTES / FLOATS */
    HostMat *mat;              /* MATRIX */
};

Entry bytes(size_t n, const void **dst) { return Entry{ BYTES, n, 0, 0, 0, dst, nullptr }; }
Entry floats(size_t n, const float **dst) { return Entry{ FLOATS, n, 0, 0, 0, (const void **)dst, nullptr }; }
Entry matrix(int rows, int cols, unsigned cls, HostMat *m) { return Entry{ MATRIX, 0, rows, cols, cls, nullptr, m }; }

/* The arrays of the file in order (file-format.md, "Body"). */
std::vector<Entry> body_schedule(const kc_config &c, int shared, const uint8_t **lflags, HostMat &tok_emb,
                                 HostMat &wcls, const float *&final_norm, std::vector<HostLayer> &layers) {
    std::vector<Entry> s;
    const size_t d = (size_t)c.dim;
    if (c.layer_flags) s.push_back(bytes((size_t)c.n_layers, (const void **)lflags));
    /* a shared table is Q8_0 when either the embedding or the classifier class is */
    s.push_back(matrix(c.vocab, c.dim, shared ? 1u | 2u : 1u, &tok_emb));
    for (HostLayer &L : layers) {
        s.push_back(floats(d, &L.attn_norm));
        s.push_back(matrix(c.q_dim, c.dim, 4, &L.wq));
        s.push_back(matrix(c.kv_dim, c.dim, 4, &L.wk));
        s.push_back(matrix(c.kv_dim, c.dim, 8, &L.wv));
        s.push_back(matrix(c.dim, c.q_dim, 16, &L.wo));
        if (c.qkv_bias) {
            s.push_back(floats((size_t)c.q_dim, &L.bq));
            s.push_back(floats((size_t)c.kv_dim, &L.bk));
            s.push_back(floats((size_t)c.kv_dim, &L.bv));
        }
        if (c.qk_norm) {
            s.push_back(floats((size_t)c.head_dim, &L.q_norm));
            s.push_back(floats((size_t)c.head_dim, &L.k_norm));
        }
        s.push_back(floats(d, &L.ffn_norm));
        s.push_back(matrix(c.hidden_dim, c.dim, 32, &L.w1));
        s.push_back(matrix(c.dim, c.hidden_dim, 64, &L.w2));
        s.push_back(matrix(c.hidden_dim, c.dim, 32, &L.w3));
        if (c.post_norms) {
            s.push_back(floats(d, &L.post_attn_norm));
            s.push_back(floats(d, &L.post_ffn_norm));
        }
    }
    s.push_back(floats(d, &final_norm));
    if (!shared) s.push_back(matrix(c.vocab, c.dim, 2, &wcls));
    return s;
}

/* Places one array at `off` (aligned) if the file holds its n bytes; the next
 * array starts at the following boundary. The padding after the last array
 * may be missing. */
const uint8_t *place(const uint8_t *base, size_t size, size_t &off, size_t n) {
    if (off > size || n > size - off) return nullptr;
    const uint8_t *p = base + off;
    off += n;
    off = off % ALIGN ? off + (ALIGN - off % ALIGN) : off;
    return p;
}

}  // namespace

int parse_header(kc_config *cfg, int *shared, const uint8_t *h) {
    kc_config c{};
    if (std::memcmp(h, "MLB1", 4) != 0 || le32(h + 4) != 1) return KC_E_FORMAT;
    for (const Field &F : HEADER) {
        const uint32_t u = le32(h + F.offset);
        const float f = F.is_float ? lef(h + F.offset) : 0.0f;
        if (!accepts(F.rule, u, f)) return F.status;
        if (F.i) c.*F.i = (int)u;
        if (F.f) c.*F.f = f;
    }
    c.q8_mask = le32(h + 72);
    const uint32_t sh = le32(h + 48);
    const int s = cross_checks(c);
    if (s != KC_OK) return s;
    *cfg = c;
    *shared = sh != 0;
    return KC_OK;
}

int take_arrays(const kc_config &c, int shared, const uint8_t *data, size_t size, HostMat &tok_emb, HostMat &wcls,
                const float *&final_norm, std::vector<HostLayer> &layers) {
    layers.assign((size_t)c.n_layers, HostLayer{});
    const uint8_t *lflags = nullptr;
    const std::vector<Entry> sched = body_schedule(c, shared, &lflags, tok_emb, wcls, final_norm, layers);
    size_t off = HEADER_BYTES;
    for (const Entry &e : sched) {
        if (e.kind != MATRIX) {
            const uint8_t *p = place(data, size, off, e.kind == FLOATS ? e.count * sizeof(float) : e.count);
            if (!p) return KC_E_FORMAT;
            *e.dst = p;
            continue;
        }
        HostMat &M = *e.mat;
        M.rows = e.rows;
        M.cols = e.cols;
        M.type = c.wtype == KC_Q8_0 || (c.q8_mask & e.cls) ? KC_Q8_0 : KC_Q4_0;
        M.d16 = c.scale_f16;
        M.q = place(data, size, off, M.qbytes());
        M.d = M.q ? place(data, size, off, M.dbytes()) : nullptr;
        if (!M.q || !M.d) return KC_E_FORMAT;
        /* Q8_0 quants lie in [-127, 127]: -128 has no int8 negation */
        if (M.type == KC_Q8_0 && std::memchr(M.q, 0x80, M.qbytes())) return KC_E_FORMAT;
    }
    /* per-layer flags: bit 0 sliding window, bit 1 local RoPE (which needs its base) */
    for (int l = 0; l < c.n_layers; l++) {
        const unsigned fl = lflags ? lflags[l] : LAYER_SLIDING;   /* no flags: the window, if any, everywhere */
        if ((fl & ~(LAYER_SLIDING | LAYER_LOCAL_ROPE)) || ((fl & LAYER_LOCAL_ROPE) && !(c.rope_local_theta > 0.0f)))
            return KC_E_FORMAT;
        layers[(size_t)l].window = fl & LAYER_SLIDING ? c.sliding_window : 0;
        layers[(size_t)l].local_rope = (fl & LAYER_LOCAL_ROPE) != 0;
    }
    if (shared) wcls = tok_emb;
    return KC_OK;
}

}  // namespace kc

extern "C" int kc_model_load(kc_model **out, const char *path) {
    *out = nullptr;
    kc::clear_error();
    const int fd = open(path, O_RDONLY);
    if (fd < 0) { kc::set_error(std::string("cannot open ") + path); return KC_E_IO; }
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); return KC_E_IO; }
    if ((size_t)st.st_size < kc::HEADER_BYTES) { close(fd); return KC_E_FORMAT; }
    void *p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return KC_E_IO;
    kc_model *m = new (std::nothrow) kc_model();
    if (!m) { munmap(p, (size_t)st.st_size); return KC_E_NOMEM; }
    m->map = p;
    m->map_size = (size_t)st.st_size;
    int s = kc::parse_header(&m->cfg, &m->shared, (const uint8_t *)p);
    if (s == KC_OK)
        s = kc::take_arrays(m->cfg, m->shared, (const uint8_t *)p, m->map_size, m->tok_emb, m->wcls, m->final_norm,
                            m->layers);
    if (s != KC_OK) { kc_model_free(m); return s; }
    *out = m;
    return KC_OK;
}
