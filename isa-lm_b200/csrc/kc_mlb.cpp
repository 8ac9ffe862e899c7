/* .mlb loading for the CUDA build: the reference's header rules and array
 * walk (model/mlb.c:80-218), written for this library, with the same status
 * codes. The arrays stay host views into the mapping until kc_model_upload. */
#include <cmath>
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "kc_internal.h"

namespace kc {

static const uint32_t MAX_DIM = 1u << 16;      /* model/mlb.c:5 */
static const uint32_t MAX_TOKENS = 1u << 24;   /* model/mlb.c:6 */

static uint32_t rd32(const uint8_t *p) { uint32_t v; std::memcpy(&v, p, 4); return v; }
static float rdf(const uint8_t *p) { float v; std::memcpy(&v, p, 4); return v; }

int parse_header(kc_config *cfg, int *shared, const uint8_t *h) {
    std::memset(cfg, 0, sizeof *cfg);
    if (std::memcmp(h, "MLB1", 4) != 0 || rd32(h + 4) != 1) return KC_E_FORMAT;
    uint32_t v[7];
    for (int i = 0; i < 7; i++) v[i] = rd32(h + 8 + 4 * i);
    for (int i = 0; i < 7; i++)
        if (v[i] == 0 || v[i] > (i == 5 || i == 6 ? MAX_TOKENS : MAX_DIM)) return KC_E_SHAPE;
    if (v[5] < 3) return KC_E_SHAPE;   /* ids 1 and 2 are BOS / EOS */
    cfg->dim = (int)v[0]; cfg->n_layers = (int)v[1]; cfg->n_heads = (int)v[2];
    cfg->n_kv_heads = (int)v[3]; cfg->hidden_dim = (int)v[4]; cfg->vocab = (int)v[5];
    cfg->max_seq = (int)v[6];
    cfg->rope_theta = rdf(h + 36);
    cfg->norm_eps = rdf(h + 40);
    cfg->wtype = (int)rd32(h + 44);
    *shared = rd32(h + 48) != 0;
    if (cfg->wtype != KC_Q8_0 && cfg->wtype != KC_Q4_0) return KC_E_FORMAT;
    cfg->q8_mask = rd32(h + 72);
    if ((cfg->q8_mask & ~127u) || (cfg->wtype == KC_Q8_0 && cfg->q8_mask)) return KC_E_FORMAT;
    const uint32_t bias = rd32(h + 76);
    if (bias > 1) return KC_E_FORMAT;
    cfg->qkv_bias = (int)bias;
    if (cfg->dim % KC_QK || cfg->hidden_dim % KC_QK) return KC_E_SHAPE;
    if (cfg->n_heads % cfg->n_kv_heads) return KC_E_SHAPE;
    const uint32_t hd = rd32(h + 80);
    if (hd > MAX_DIM || (!hd && cfg->dim % cfg->n_heads)) return KC_E_SHAPE;
    cfg->head_dim = hd ? (int)hd : cfg->dim / cfg->n_heads;
    if ((uint64_t)cfg->head_dim * (uint64_t)cfg->n_heads > MAX_DIM) return KC_E_SHAPE;
    cfg->q_dim = cfg->head_dim * cfg->n_heads;
    cfg->kv_dim = cfg->head_dim * cfg->n_kv_heads;
    if (cfg->head_dim % 2 || cfg->q_dim % KC_QK) return KC_E_SHAPE;
    const uint32_t qkn = rd32(h + 84), win = rd32(h + 92);
    if (qkn > 1 || win > MAX_TOKENS) return KC_E_FORMAT;
    cfg->qk_norm = (int)qkn;
    cfg->sliding_window = (int)win;
    const uint32_t lflags = rd32(h + 96);
    if (lflags > 1) return KC_E_FORMAT;
    cfg->layer_flags = (int)lflags;
    cfg->rope_local_theta = rdf(h + 100);
    if (!(cfg->rope_local_theta >= 0.0f && cfg->rope_local_theta < 1e30f)) return KC_E_FORMAT;
    const uint32_t act = rd32(h + 104), pn = rd32(h + 108);
    if (act > 1 || pn > 1) return KC_E_FORMAT;
    cfg->act = (int)act;
    cfg->post_norms = (int)pn;
    cfg->embed_scale = rdf(h + 112);
    cfg->attn_scale = rdf(h + 116);
    if (!(cfg->embed_scale >= 0.0f && cfg->embed_scale < 1e6f) || !(cfg->attn_scale >= 0.0f && cfg->attn_scale < 1e6f))
        return KC_E_FORMAT;
    if (cfg->embed_scale == 0.0f) cfg->embed_scale = 1.0f;
    if (cfg->attn_scale == 0.0f) cfg->attn_scale = 1.0f / std::sqrt((float)cfg->head_dim);
    const uint32_t f16 = rd32(h + 120);
    if (f16 > 1) return KC_E_FORMAT;
    cfg->scale_f16 = (int)f16;
    cfg->attn_softcap = rdf(h + 124);
    cfg->final_softcap = rdf(h + 128);
    if (!(cfg->attn_softcap >= 0.0f && cfg->attn_softcap < 1e6f) || !(cfg->final_softcap >= 0.0f && cfg->final_softcap < 1e6f))
        return KC_E_FORMAT;
    if (!(cfg->rope_theta > 0.0f) || !(cfg->norm_eps >= 0.0f)) return KC_E_FORMAT;
    cfg->rope_type = (int)rd32(h + 52);
    cfg->rope_factor = rdf(h + 56);
    cfg->rope_low_freq_factor = rdf(h + 60);
    cfg->rope_high_freq_factor = rdf(h + 64);
    cfg->rope_orig_max_seq = (int)rd32(h + 68);
    cfg->rope_attn_factor = rdf(h + 88);
    if (cfg->rope_type != 3 && cfg->rope_attn_factor != 0.0f) return KC_E_FORMAT;
    if (cfg->rope_type == 1) {
        if (!(cfg->rope_factor > 0.0f && cfg->rope_factor < 1e6f) || !(cfg->rope_low_freq_factor > 0.0f) ||
            !(cfg->rope_high_freq_factor > cfg->rope_low_freq_factor && cfg->rope_high_freq_factor < 1e6f) ||
            cfg->rope_orig_max_seq <= 0)
            return KC_E_FORMAT;
    } else if (cfg->rope_type == 2) {
        if (!(cfg->rope_factor > 0.0f && cfg->rope_factor < 1e6f)) return KC_E_FORMAT;
    } else if (cfg->rope_type == 3) {
        if (!(cfg->rope_factor > 0.0f && cfg->rope_factor < 1e6f) || !(cfg->rope_high_freq_factor > 0.0f) ||
            !(cfg->rope_low_freq_factor > cfg->rope_high_freq_factor && cfg->rope_low_freq_factor < 1e6f) ||
            cfg->rope_orig_max_seq <= 0 || !(cfg->rope_attn_factor > 0.0f && cfg->rope_attn_factor < 1e3f))
            return KC_E_FORMAT;
    } else if (cfg->rope_type != 0) {
        return KC_E_FORMAT;
    }
    return KC_OK;
}

namespace {
struct Cursor {
    const uint8_t *base;
    size_t off, size;
    bool ok;
    /* model/mlb.c:24-31: each array starts 64 B aligned; a missing final pad is tolerated */
    const void *take(size_t n) {
        if (!ok || n > size - off) { ok = false; return nullptr; }
        const void *p = base + off;
        off += n;
        off = (off + 63) & ~(size_t)63;
        if (off > size) off = size;
        return p;
    }
    HostMat take_mat(int rows, int cols, int type, int f16) {
        HostMat t;
        t.rows = rows; t.cols = cols; t.type = type; t.d16 = f16;
        const size_t n = (size_t)rows * (size_t)cols;
        t.q = take(type == KC_Q4_0 ? n / 2 : n);
        t.d = take(n / KC_QK * (f16 ? 2 : 4));
        /* Q8 quants must be in [-127, 127] (model/mlb.c:34-36) */
        if (ok && type == KC_Q8_0 && std::memchr(t.q, 0x80, n)) ok = false;
        return t;
    }
};
}  // namespace

int take_arrays(const kc_config &c, int shared, const uint8_t *data, size_t size, HostMat &tok_emb, HostMat &wcls,
                const float *&final_norm, std::vector<HostLayer> &layers) {
    auto WT = [&](unsigned bits) { return c.wtype == KC_Q8_0 || (c.q8_mask & bits) ? KC_Q8_0 : KC_Q4_0; };
    Cursor cur{ data, 256, size, true };
    const size_t normsz = (size_t)c.dim * sizeof(float);
    const uint8_t *lf = c.layer_flags ? (const uint8_t *)cur.take((size_t)c.n_layers) : nullptr;
    for (int l = 0; lf && cur.ok && l < c.n_layers; l++)
        if ((lf[l] & ~3) || ((lf[l] & 2) && !(c.rope_local_theta > 0.0f))) return KC_E_FORMAT;
    layers.assign((size_t)c.n_layers, HostLayer{});
    tok_emb = cur.take_mat(c.vocab, c.dim, WT(1u | (shared ? 2u : 0u)), c.scale_f16);
    for (int l = 0; l < c.n_layers; l++) {
        HostLayer &L = layers[(size_t)l];
        L.window = !lf || (lf[l] & 1) ? c.sliding_window : 0;
        L.local_rope = lf && (lf[l] & 2);
        L.attn_norm = (const float *)cur.take(normsz);
        L.wq = cur.take_mat(c.q_dim, c.dim, WT(4), c.scale_f16);
        L.wk = cur.take_mat(c.kv_dim, c.dim, WT(4), c.scale_f16);
        L.wv = cur.take_mat(c.kv_dim, c.dim, WT(8), c.scale_f16);
        L.wo = cur.take_mat(c.dim, c.q_dim, WT(16), c.scale_f16);
        if (c.qkv_bias) {
            L.bq = (const float *)cur.take((size_t)c.q_dim * 4);
            L.bk = (const float *)cur.take((size_t)c.kv_dim * 4);
            L.bv = (const float *)cur.take((size_t)c.kv_dim * 4);
        }
        if (c.qk_norm) {
            L.q_norm = (const float *)cur.take((size_t)c.head_dim * 4);
            L.k_norm = (const float *)cur.take((size_t)c.head_dim * 4);
        }
        L.ffn_norm = (const float *)cur.take(normsz);
        L.w1 = cur.take_mat(c.hidden_dim, c.dim, WT(32), c.scale_f16);
        L.w2 = cur.take_mat(c.dim, c.hidden_dim, WT(64), c.scale_f16);
        L.w3 = cur.take_mat(c.hidden_dim, c.dim, WT(32), c.scale_f16);
        if (c.post_norms) {
            L.post_attn_norm = (const float *)cur.take(normsz);
            L.post_ffn_norm = (const float *)cur.take(normsz);
        }
    }
    final_norm = (const float *)cur.take(normsz);
    wcls = shared ? tok_emb : cur.take_mat(c.vocab, c.dim, WT(2), c.scale_f16);
    return cur.ok ? KC_OK : KC_E_FORMAT;
}

}  // namespace kc

extern "C" int kc_model_load(kc_model **out, const char *path) {
    *out = nullptr;
    kc::clear_error();
    const int fd = open(path, O_RDONLY);
    if (fd < 0) { kc::set_error(std::string("cannot open ") + path); return KC_E_IO; }
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); return KC_E_IO; }
    if ((size_t)st.st_size < 256) { close(fd); return KC_E_FORMAT; }
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
