/* TEST INFRASTRUCTURE ONLY — CPU restatement of the reference's scalar token
 * loop. See krafla_oracle.h. Built with -ffp-contract=off like the reference
 * (Makefile:18 of the reference) so every float operation rounds as its scalar
 * build does. Each function cites the reference file:line it follows. */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "krafla_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#define QK ORC_QK
#define QUANT_TINY 1e-30f   /* core/ml.h:22 */

/* ---------------------------------------------------------------- numerics */

/* IEEE binary16 from binary32, round to nearest even; the same values as
 * core/ml.c:39-53 (written here from the IEEE definition). */
uint16_t orc_f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7e00u;            /* NaN */
    if (a >= 0x477ff000u) return sign | 0x7c00u;           /* overflows to inf */
    if (a < 0x38800000u) {                                 /* result subnormal or zero */
        float m;
        memcpy(&m, &a, 4);
        return sign | (uint16_t)lrintf(m * 16777216.0f);  /* multiples of 2^-24, RNE */
    }
    const uint32_t r = a + 0xfffu + ((a >> 13) & 1u);      /* RNE on the 13 dropped bits */
    return sign | (uint16_t)((r >> 13) - (112u << 10));
}

/* core/ml.c:55-62 */
float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) return (sign ? -1.0f : 1.0f) * (float)m * (1.0f / 16777216.0f);
    const uint32_t x = sign | (e == 31 ? 0x7f800000u | (m << 13) : ((e + 112u) << 23) | (m << 13));
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* kernels/scalar/k_scalar.c:39-57: d = amax/127, q = trunc(x*(127/amax) + copysign(.5, x)). */
void orc_quantize_q8(int8_t *q, float *d, const float *x, int k) {
    for (int b = 0; b < k / QK; b++) {
        const float *xb = x + b * QK;
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) amax = fmaxf(amax, fabsf(xb[j]));
        if (amax < QUANT_TINY) {
            d[b] = 0.0f;
            memset(q + b * QK, 0, QK);
            continue;
        }
        const float id = 127.0f / amax;
        d[b] = amax / 127.0f;
        for (int j = 0; j < QK; j++) {
            float v = truncf(xb[j] * id + copysignf(0.5f, xb[j]));
            v = fminf(fmaxf(v, -127.0f), 127.0f);
            q[b * QK + j] = (int8_t)v;
        }
    }
}

/* ops/ops.c:81-96 */
void orc_quantize_row(int8_t *q, float *d, const float *x, int n) {
    float amax = 0.0f;
    for (int i = 0; i < n; i++) amax = fmaxf(amax, fabsf(x[i]));
    if (amax < QUANT_TINY) {
        *d = 0.0f;
        memset(q, 0, (size_t)n);
        return;
    }
    const float id = 127.0f / amax;
    *d = amax / 127.0f;
    for (int i = 0; i < n; i++) {
        float v = truncf(x[i] * id + copysignf(0.5f, x[i]));
        v = fminf(fmaxf(v, -127.0f), 127.0f);
        q[i] = (int8_t)v;
    }
}

/* int32 dot of weight row r, block b with the activation block. Q4 bytes hold
 * element j (low nibble) and j+16 (high nibble), value nibble - 8
 * (kernels/scalar/k_scalar.c:19-37, core/quant_ref.c:11-18). */
static int32_t block_dot(int type, const void *wq, int cols, int r, int b, const int8_t *xq) {
    int32_t s = 0;
    if (type == ORC_Q8_0) {
        const int8_t *w = (const int8_t *)wq + (size_t)r * cols + (size_t)b * QK;
        for (int j = 0; j < QK; j++) s += w[j] * xq[b * QK + j];
    } else {
        const uint8_t *p = (const uint8_t *)wq + ((size_t)r * (cols / QK) + b) * (QK / 2);
        for (int j = 0; j < QK / 2; j++) {
            s += ((p[j] & 0xF) - 8) * xq[b * QK + j];
            s += ((p[j] >> 4) - 8) * xq[b * QK + j + QK / 2];
        }
    }
    return s;
}

/* k_scalar.c:4-37: sum += (float)s * wd * xd, blocks in order. */
void orc_matvec(float *y, int type, const void *wq, const float *wd, int rows, int cols,
                const int8_t *xq, const float *xd, int r0, int r1) {
    (void)rows;
    const int nb = cols / QK;
    for (int r = r0; r < r1; r++) {
        float sum = 0.0f;
        for (int b = 0; b < nb; b++)
            sum += (float)block_dot(type, wq, cols, r, b, xq) * wd[(size_t)r * nb + b] * xd[b];
        y[r] = sum;
    }
}

void orc_block_sums(int32_t *s, int type, const void *wq, int rows, int cols, const int8_t *xq) {
    const int nb = cols / QK;
    for (int r = 0; r < rows; r++)
        for (int b = 0; b < nb; b++) s[(size_t)r * nb + b] = block_dot(type, wq, cols, r, b, xq);
}

/* k_scalar.c:59-64 */
void orc_rmsnorm(float *o, const float *x, const float *w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) o[i] = x[i] * inv * w[i];
}

/* k_scalar.c:66-77 */
void orc_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) mx = fmaxf(mx, x[i]);
    if (mx == -INFINITY) {
        for (int i = 0; i < n; i++) x[i] = 1.0f / (float)n;
        return;
    }
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    const float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* k_scalar.c:79-94: rotate adjacent pairs (2i, 2i+1). */
static void rope_heads(float *v, const float *c, const float *s, int hd, int nh) {
    for (int h = 0; h < nh; h++) {
        float *p = v + h * hd;
        for (int i = 0; i < hd / 2; i++) {
            const float a = p[2 * i], b = p[2 * i + 1];
            p[2 * i] = a * c[i] - b * s[i];
            p[2 * i + 1] = a * s[i] + b * c[i];
        }
    }
}

void orc_rope(float *q, float *k, const float *cs, const float *sn, int hd, int nh, int nkv) {
    rope_heads(q, cs, sn, hd, nh);
    rope_heads(k, cs, sn, hd, nkv);
}

/* k_scalar.c:96-98 */
void orc_silu_mul(float *g, const float *u, int n) {
    for (int i = 0; i < n; i++) g[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

/* k_scalar.c:100-105 */
void orc_gelu_mul(float *g, const float *u, int n) {
    for (int i = 0; i < n; i++) {
        const float x = g[i];
        g[i] = 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x))) * u[i];
    }
}

/* core/quant_ref.c:4-19 */
void orc_dequant_row(float *out, int type, const void *wq, const float *wd, int cols, int row) {
    const int nb = cols / QK;
    const float *d = wd + (size_t)row * nb;
    if (type == ORC_Q8_0) {
        const int8_t *q = (const int8_t *)wq + (size_t)row * cols;
        for (int i = 0; i < cols; i++) out[i] = q[i] * d[i / QK];
        return;
    }
    const uint8_t *q = (const uint8_t *)wq + (size_t)row * nb * (QK / 2);
    for (int b = 0; b < nb; b++)
        for (int j = 0; j < QK / 2; j++) {
            const uint8_t v = q[b * (QK / 2) + j];
            out[b * QK + j] = ((v & 0xF) - 8) * d[b];
            out[b * QK + j + QK / 2] = ((v >> 4) - 8) * d[b];
        }
}

/* ------------------------------------------------------------------ model */

typedef struct {
    const void *q;
    float *d;     /* float scales (converted from f16 when the file has f16) */
    int rows, cols, type;
} omat;

typedef struct {
    const float *attn_norm, *ffn_norm, *bq, *bk, *bv, *q_norm, *k_norm, *post_attn_norm, *post_ffn_norm;
    omat wq, wk, wv, wo, w1, w2, w3;
    int window, local_rope;
} olayer;

struct orc_model {
    /* header (model/mlb.h:9-32) */
    int dim, n_layers, n_heads, n_kv_heads, hidden_dim, vocab, max_seq, head_dim, kv_dim, q_dim;
    float rope_theta, norm_eps;
    int wtype, q8_mask, qkv_bias, qk_norm, sliding_window, layer_flags, act, post_norms, scale_f16, shared;
    float rope_local_theta, embed_scale, attn_scale, attn_softcap, final_softcap;
    int rope_type, rope_orig;
    float rope_factor, rope_lo, rope_hi, rope_attn_factor;
    /* arrays */
    uint8_t *data;
    size_t size;
    omat tok_emb, wcls;
    const float *final_norm;
    olayer *layers;
};

static uint32_t rd32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }
static float rdf(const uint8_t *p) { float v; memcpy(&v, p, 4); return v; }

typedef struct { const uint8_t *base; size_t off, size; int ok; } cur_t;

/* model/mlb.c:24-31: arrays are 64 B aligned. */
static const void *take(cur_t *c, size_t n) {
    if (!c->ok || n > c->size - c->off) { c->ok = 0; return NULL; }
    const void *p = c->base + c->off;
    c->off += n;
    c->off = (c->off + 63) & ~(size_t)63;
    if (c->off > c->size) c->off = c->size;
    return p;
}

static omat take_mat(cur_t *c, int rows, int cols, int type, int f16) {
    omat t = { NULL, NULL, rows, cols, type };
    const size_t n = (size_t)rows * cols, nb = n / QK;
    t.q = take(c, type == ORC_Q4_0 ? n / 2 : n);
    const void *dp = take(c, nb * (f16 ? 2 : 4));
    if (!c->ok) return t;
    t.d = malloc(nb * sizeof(float));
    if (!t.d) { c->ok = 0; return t; }
    for (size_t i = 0; i < nb; i++)
        t.d[i] = f16 ? orc_f16_to_f32(((const uint16_t *)dp)[i]) : ((const float *)dp)[i];
    return t;
}

/* model/mlb.c:80-159 (the fields the forward reads) and :161-218. */
int orc_model_load(orc_model **out, const char *path) {
    *out = NULL;
    int fd = open(path, O_RDONLY);
    if (fd < 0) return ORC_E_IO;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 256) { close(fd); return ORC_E_FORMAT; }
    void *mp = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (mp == MAP_FAILED) return ORC_E_IO;
    orc_model *m = calloc(1, sizeof *m);
    if (!m) { munmap(mp, (size_t)st.st_size); return ORC_E_NOMEM; }
    m->data = mp;
    m->size = (size_t)st.st_size;
    const uint8_t *h = m->data;
    if (memcmp(h, "MLB1", 4) != 0 || rd32(h + 4) != 1) { orc_model_free(m); return ORC_E_FORMAT; }
    m->dim = (int)rd32(h + 8); m->n_layers = (int)rd32(h + 12); m->n_heads = (int)rd32(h + 16);
    m->n_kv_heads = (int)rd32(h + 20); m->hidden_dim = (int)rd32(h + 24); m->vocab = (int)rd32(h + 28);
    m->max_seq = (int)rd32(h + 32);
    m->rope_theta = rdf(h + 36); m->norm_eps = rdf(h + 40);
    m->wtype = (int)rd32(h + 44); m->shared = rd32(h + 48) != 0;
    m->rope_type = (int)rd32(h + 52); m->rope_factor = rdf(h + 56); m->rope_lo = rdf(h + 60);
    m->rope_hi = rdf(h + 64); m->rope_orig = (int)rd32(h + 68);
    m->q8_mask = (int)rd32(h + 72); m->qkv_bias = (int)rd32(h + 76);
    const int hd = (int)rd32(h + 80);
    m->qk_norm = (int)rd32(h + 84); m->rope_attn_factor = rdf(h + 88);
    m->sliding_window = (int)rd32(h + 92); m->layer_flags = (int)rd32(h + 96);
    m->rope_local_theta = rdf(h + 100); m->act = (int)rd32(h + 104); m->post_norms = (int)rd32(h + 108);
    m->embed_scale = rdf(h + 112); m->attn_scale = rdf(h + 116); m->scale_f16 = (int)rd32(h + 120);
    m->attn_softcap = rdf(h + 124); m->final_softcap = rdf(h + 128);
    if (m->n_heads <= 0 || m->n_kv_heads <= 0 || m->dim <= 0) { orc_model_free(m); return ORC_E_SHAPE; }
    m->head_dim = hd ? hd : m->dim / m->n_heads;
    m->q_dim = m->head_dim * m->n_heads;
    m->kv_dim = m->head_dim * m->n_kv_heads;
    if (m->embed_scale == 0.0f) m->embed_scale = 1.0f;
    if (m->attn_scale == 0.0f) m->attn_scale = 1.0f / sqrtf((float)m->head_dim);   /* model/mlb.c:126 */

    const int f16 = m->scale_f16;
#define WT(bits) (m->wtype == ORC_Q8_0 || (m->q8_mask & (bits)) ? ORC_Q8_0 : ORC_Q4_0)
    cur_t c = { m->data, 256, m->size, 1 };
    const uint8_t *lf = m->layer_flags ? take(&c, (size_t)m->n_layers) : NULL;
    m->layers = calloc((size_t)m->n_layers, sizeof(olayer));
    if (!m->layers) { orc_model_free(m); return ORC_E_NOMEM; }
    const size_t normsz = (size_t)m->dim * 4;
    m->tok_emb = take_mat(&c, m->vocab, m->dim, WT(1 | (m->shared ? 2 : 0)), f16);
    for (int l = 0; l < m->n_layers; l++) {
        olayer *L = &m->layers[l];
        L->window = !lf || (lf[l] & 1) ? m->sliding_window : 0;
        L->local_rope = lf && (lf[l] & 2);
        L->attn_norm = take(&c, normsz);
        L->wq = take_mat(&c, m->q_dim, m->dim, WT(4), f16);
        L->wk = take_mat(&c, m->kv_dim, m->dim, WT(4), f16);
        L->wv = take_mat(&c, m->kv_dim, m->dim, WT(8), f16);
        L->wo = take_mat(&c, m->dim, m->q_dim, WT(16), f16);
        if (m->qkv_bias) {
            L->bq = take(&c, (size_t)m->q_dim * 4);
            L->bk = take(&c, (size_t)m->kv_dim * 4);
            L->bv = take(&c, (size_t)m->kv_dim * 4);
        }
        if (m->qk_norm) {
            L->q_norm = take(&c, (size_t)m->head_dim * 4);
            L->k_norm = take(&c, (size_t)m->head_dim * 4);
        }
        L->ffn_norm = take(&c, normsz);
        L->w1 = take_mat(&c, m->hidden_dim, m->dim, WT(32), f16);
        L->w2 = take_mat(&c, m->dim, m->hidden_dim, WT(64), f16);
        L->w3 = take_mat(&c, m->hidden_dim, m->dim, WT(32), f16);
        if (m->post_norms) {
            L->post_attn_norm = take(&c, normsz);
            L->post_ffn_norm = take(&c, normsz);
        }
    }
    m->final_norm = take(&c, normsz);
    if (m->shared) {
        m->wcls = m->tok_emb;
    } else {
        m->wcls = take_mat(&c, m->vocab, m->dim, WT(2), f16);
    }
#undef WT
    if (!c.ok) { orc_model_free(m); return ORC_E_FORMAT; }
    *out = m;
    return ORC_OK;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    if (m->layers) {
        for (int l = 0; l < m->n_layers; l++) {
            olayer *L = &m->layers[l];
            free(L->wq.d); free(L->wk.d); free(L->wv.d); free(L->wo.d);
            free(L->w1.d); free(L->w2.d); free(L->w3.d);
        }
        free(m->layers);
    }
    if (!m->shared) free(m->wcls.d);
    free(m->tok_emb.d);
    if (m->data) munmap(m->data, m->size);
    free(m);
}

void orc_model_config(const orc_model *m, int *f) {
    const int v[20] = { m->dim, m->n_layers, m->n_heads, m->n_kv_heads, m->hidden_dim, m->vocab, m->max_seq,
                        m->head_dim, m->kv_dim, m->q_dim, m->wtype, m->q8_mask, m->qkv_bias, m->qk_norm,
                        m->sliding_window, m->act, m->post_norms, m->scale_f16, m->shared, m->rope_type };
    memcpy(f, v, sizeof v);
}

/* ------------------------------------------------------------------ state */

struct orc_state {
    orc_model *m;
    int kv_type, nthreads;
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *ao, *att, *logits;
    int8_t *qa, *qh, *qq;   /* quantized inputs: max(dim, q_dim), hidden_dim; Q8 KV query */
    float *da, *dh, *qd;
    float *kc, *vc;         /* F32 [L][max_seq][kv_dim] */
    uint16_t *kh, *vh;      /* F16 */
    int8_t *kq, *vq;        /* Q8 */
    float *kd, *vd;         /* Q8 scales [L][max_seq][n_kv_heads] */
    float *rcos, *rsin, *lcos, *lsin;   /* [max_seq][hd/2] */
};

/* model/transformer.c:16-38 */
static double rope_inv_freq(const orc_model *c, int i) {
    const double inv = pow((double)c->rope_theta, -2.0 * i / c->head_dim);
    if (c->rope_type == 2) return inv / c->rope_factor;
    if (c->rope_type == 3) {
        const double hd = c->head_dim, orig = c->rope_orig, lb = 2.0 * log((double)c->rope_theta);
        const double pi2 = 2.0 * 3.14159265358979323846;
        double lo = floor(hd * log(orig / ((double)c->rope_lo * pi2)) / lb);
        double hi = ceil(hd * log(orig / ((double)c->rope_hi * pi2)) / lb);
        if (lo < 0.0) lo = 0.0;
        if (hi > hd - 1.0) hi = hd - 1.0;
        if (lo == hi) hi += 0.001;
        double ramp = (i - lo) / (hi - lo);
        ramp = ramp < 0.0 ? 0.0 : (ramp > 1.0 ? 1.0 : ramp);
        return inv / c->rope_factor * ramp + inv * (1.0 - ramp);
    }
    if (c->rope_type != 1) return inv;
    const double f = c->rope_factor, lo = c->rope_lo, hi = c->rope_hi;
    const double orig = c->rope_orig, wavelen = 2.0 * 3.14159265358979323846 / inv;
    if (wavelen < orig / hi) return inv;
    if (wavelen > orig / lo) return inv / f;
    const double smooth = (orig / wavelen - lo) / (hi - lo);
    return (1.0 - smooth) * inv / f + smooth * inv;
}

int orc_state_new(orc_state **out, orc_model *m, int kv_type, int nthreads) {
    *out = NULL;
    if (kv_type != ORC_F32 && kv_type != ORC_F16 && kv_type != ORC_Q8_0) return ORC_E_SHAPE;
    orc_state *s = calloc(1, sizeof *s);
    if (!s) return ORC_E_NOMEM;
    s->m = m;
    s->kv_type = kv_type;
    s->nthreads = nthreads < 1 ? 1 : nthreads;
    const size_t D = m->dim, QD = m->q_dim, KV = m->kv_dim, H = m->hidden_dim, T = m->max_seq;
    const size_t big = D > QD ? D : QD, h2 = m->head_dim / 2;
    const size_t kvn = (size_t)m->n_layers * T * KV;
    s->x = calloc(D, 4); s->xb = calloc(D, 4); s->xb2 = calloc(D, 4);
    s->hb = calloc(H, 4); s->hb2 = calloc(H, 4);
    s->q = calloc(QD, 4); s->k = calloc(KV, 4); s->v = calloc(KV, 4); s->ao = calloc(QD, 4);
    s->att = calloc((size_t)m->n_heads * T, 4);
    s->logits = calloc((size_t)m->vocab, 4);
    s->qa = calloc(big, 1); s->da = calloc(big / QK + 1, 4);
    s->qh = calloc(H, 1); s->dh = calloc(H / QK + 1, 4);
    s->qq = calloc(QD, 1); s->qd = calloc((size_t)m->n_heads, 4);
    if (kv_type == ORC_F32) { s->kc = calloc(kvn, 4); s->vc = calloc(kvn, 4); }
    else if (kv_type == ORC_F16) { s->kh = calloc(kvn, 2); s->vh = calloc(kvn, 2); }
    else {
        s->kq = calloc(kvn, 1); s->vq = calloc(kvn, 1);
        s->kd = calloc((size_t)m->n_layers * T * m->n_kv_heads, 4);
        s->vd = calloc((size_t)m->n_layers * T * m->n_kv_heads, 4);
    }
    s->rcos = calloc(T * h2, 4); s->rsin = calloc(T * h2, 4);
    if (m->rope_local_theta > 0.0f) { s->lcos = calloc(T * h2, 4); s->lsin = calloc(T * h2, 4); }
    if (!s->x || !s->att || !s->logits || !s->rcos || !s->rsin || !s->qq ||
        (kv_type == ORC_F32 && (!s->kc || !s->vc)) || (kv_type == ORC_F16 && (!s->kh || !s->vh)) ||
        (kv_type == ORC_Q8_0 && (!s->kq || !s->vq || !s->kd || !s->vd))) {
        orc_state_free(s);
        return ORC_E_NOMEM;
    }
    /* model/transformer.c:146-162: tables in double, stored as float */
    const double af = m->rope_type == 3 ? m->rope_attn_factor : 1.0;
    for (size_t i = 0; i < h2; i++) {
        const double freq = rope_inv_freq(m, (int)i);
        const double lfreq = s->lcos ? pow((double)m->rope_local_theta, -2.0 * (double)i / m->head_dim) : 0.0;
        for (size_t p = 0; p < T; p++) {
            const double ang = (double)p * freq;
            s->rcos[p * h2 + i] = (float)(cos(ang) * af);
            s->rsin[p * h2 + i] = (float)(sin(ang) * af);
            if (s->lcos) {
                s->lcos[p * h2 + i] = (float)cos((double)p * lfreq);
                s->lsin[p * h2 + i] = (float)sin((double)p * lfreq);
            }
        }
    }
    *out = s;
    return ORC_OK;
}

void orc_state_free(orc_state *s) {
    if (!s) return;
    free(s->x); free(s->xb); free(s->xb2); free(s->hb); free(s->hb2); free(s->q); free(s->k); free(s->v);
    free(s->ao); free(s->att); free(s->logits); free(s->qa); free(s->da); free(s->qh); free(s->dh);
    free(s->qq); free(s->qd); free(s->kc); free(s->vc); free(s->kh); free(s->vh); free(s->kq); free(s->vq);
    free(s->kd); free(s->vd); free(s->rcos); free(s->rsin); free(s->lcos); free(s->lsin);
    free(s);
}

const float *orc_state_x(const orc_state *s) { return s->x; }
/* 0 x, 1 q (after RoPE), 2 ao, 3 hb (after the activation), 4 F32 K cache, 5 F32 V cache */
const float *orc_state_buf(const orc_state *s, int which) {
    switch (which) {
    case 0: return s->x;
    case 1: return s->q;
    case 2: return s->ao;
    case 3: return s->hb;
    case 4: return s->kc;
    case 5: return s->vc;
    }
    return NULL;
}
const float *orc_rope_cos(const orc_state *s) { return s->rcos; }
const float *orc_rope_sin(const orc_state *s) { return s->rsin; }

/* Matvec rows split across threads; each row is computed in the scalar order,
 * so the result does not depend on the split (ops/ops.c:16-42). */
typedef struct { float *y; const omat *W; const int8_t *xq; const float *xd; int r0, r1; } mv_job;

static void *mv_run(void *p) {
    const mv_job *j = p;
    orc_matvec(j->y, j->W->type, j->W->q, j->W->d, j->W->rows, j->W->cols, j->xq, j->xd, j->r0, j->r1);
    return NULL;
}

static void matvec(const orc_state *s, float *y, const omat *W, const int8_t *xq, const float *xd) {
    int nt = s->nthreads;
    if ((size_t)W->rows * W->cols < (1u << 20) || nt <= 1) {
        orc_matvec(y, W->type, W->q, W->d, W->rows, W->cols, xq, xd, 0, W->rows);
        return;
    }
    if (nt > 64) nt = 64;
    pthread_t th[64];
    mv_job jobs[64];
    int started[64] = { 0 };
    for (int t = 0; t < nt; t++) {
        jobs[t] = (mv_job){ y, W, xq, xd, (int)((long long)W->rows * t / nt), (int)((long long)W->rows * (t + 1) / nt) };
        if (t > 0) started[t] = pthread_create(&th[t], NULL, mv_run, &jobs[t]) == 0;
    }
    mv_run(&jobs[0]);
    for (int t = 1; t < nt; t++) {
        if (started[t]) pthread_join(th[t], NULL);
        else mv_run(&jobs[t]);
    }
}

static void add(float *y, const float *x, int n) { for (int i = 0; i < n; i++) y[i] += x[i]; }

/* model/transformer.c:240-243 */
static void residual_add(const orc_model *m, float *x, float *y, const float *post_norm) {
    if (post_norm) orc_rmsnorm(y, y, post_norm, m->dim, m->norm_eps);
    add(x, y, m->dim);
}

/* ops/ops.c:124-155 with the scalar dot/axpy kernels (k_scalar.c:111-155),
 * for heads [0, n_heads) at position pos of layer l. */
static void attention(orc_state *s, int l, int pos) {
    const orc_model *m = s->m;
    const int hd = m->head_dim, group = m->n_heads / m->n_kv_heads, win = m->layers[l].window;
    const int first = win && pos >= win ? pos + 1 - win : 0, n = pos + 1 - first;
    const size_t ld = (size_t)m->kv_dim, ldd = (size_t)m->n_kv_heads, T = (size_t)m->max_seq;
    const size_t lrow = (size_t)l * T;
    const float scale = m->attn_scale;
    if (s->kv_type == ORC_Q8_0)   /* ops/ops.c:170-173: quantized query heads */
        for (int h = 0; h < m->n_heads; h++) orc_quantize_row(s->qq + h * hd, s->qd + h, s->q + h * hd, hd);
    for (int h = 0; h < m->n_heads; h++) {
        const int kvh = h / group;
        float *a = s->att + (size_t)h * T;
        const float *qh = s->q + h * hd;
        for (int t = 0; t < n; t++) {
            const size_t row = lrow + first + t;
            if (s->kv_type == ORC_F32) {
                const float *kr = s->kc + row * ld + (size_t)kvh * hd;
                float acc = 0.0f;
                for (int i = 0; i < hd; i++) acc += qh[i] * kr[i];
                a[t] = acc * scale;
            } else if (s->kv_type == ORC_F16) {
                const uint16_t *kr = s->kh + row * ld + (size_t)kvh * hd;
                float acc = 0.0f;
                for (int i = 0; i < hd; i++) acc += qh[i] * orc_f16_to_f32(kr[i]);
                a[t] = acc * scale;
            } else {
                const int8_t *kr = s->kq + row * ld + (size_t)kvh * hd;
                const int8_t *qq = s->qq + h * hd;
                int32_t sum = 0;
                for (int i = 0; i < hd; i++) sum += qq[i] * kr[i];
                const float c = s->qd[h] * scale;
                a[t] = (float)sum * c * s->kd[row * ldd + kvh];
            }
        }
        if (m->attn_softcap > 0.0f)
            for (int t = 0; t < n; t++) a[t] = m->attn_softcap * tanhf(a[t] / m->attn_softcap);
        orc_softmax(a, n);
        float *o = s->ao + h * hd;
        memset(o, 0, sizeof(float) * hd);
        for (int t = 0; t < n; t++) {
            const size_t row = lrow + first + t;
            if (s->kv_type == ORC_F32) {
                const float *vr = s->vc + row * ld + (size_t)kvh * hd;
                for (int i = 0; i < hd; i++) o[i] += a[t] * vr[i];
            } else if (s->kv_type == ORC_F16) {
                const uint16_t *vr = s->vh + row * ld + (size_t)kvh * hd;
                for (int i = 0; i < hd; i++) o[i] += a[t] * orc_f16_to_f32(vr[i]);
            } else {
                const int8_t *vr = s->vq + row * ld + (size_t)kvh * hd;
                const float w = a[t] * s->vd[row * ldd + kvh];
                for (int i = 0; i < hd; i++) o[i] += w * (float)vr[i];
            }
        }
    }
}

/* model/transformer.c:246-248 */
static void heads_norm(float *x, const float *w, int n, const orc_model *m) {
    for (int h = 0; h < n; h++) orc_rmsnorm(x + (size_t)h * m->head_dim, x + (size_t)h * m->head_dim, w, m->head_dim, m->norm_eps);
}

/* model/transformer.c:257-306 */
int orc_forward(orc_state *s, int token, int pos, float *logits) {
    const orc_model *m = s->m;
    if (pos < 0 || pos >= m->max_seq || token < 0 || token >= m->vocab) return ORC_E_SHAPE;
    const int D = m->dim, QD = m->q_dim, KV = m->kv_dim, H = m->hidden_dim, hd = m->head_dim;
    const size_t h2 = (size_t)hd / 2, T = (size_t)m->max_seq;
    orc_dequant_row(s->x, m->tok_emb.type, m->tok_emb.q, m->tok_emb.d, D, token);   /* embed :226-230 */
    if (m->embed_scale != 1.0f)
        for (int i = 0; i < D; i++) s->x[i] *= m->embed_scale;
    for (int l = 0; l < m->n_layers; l++) {
        const olayer *L = &m->layers[l];
        const size_t row = (size_t)l * T + pos;
        float *k = s->kv_type == ORC_F32 ? s->kc + row * KV : s->k;
        float *v = s->kv_type == ORC_F32 ? s->vc + row * KV : s->v;
        const float *cs = (L->local_rope ? s->lcos : s->rcos) + pos * h2;
        const float *sn = (L->local_rope ? s->lsin : s->rsin) + pos * h2;

        orc_rmsnorm(s->xb, s->x, L->attn_norm, D, m->norm_eps);
        orc_quantize_q8(s->qa, s->da, s->xb, D);
        matvec(s, s->q, &L->wq, s->qa, s->da);
        matvec(s, k, &L->wk, s->qa, s->da);
        matvec(s, v, &L->wv, s->qa, s->da);
        if (L->bq) { add(s->q, L->bq, QD); add(k, L->bk, KV); add(v, L->bv, KV); }
        if (L->q_norm) { heads_norm(s->q, L->q_norm, m->n_heads, m); heads_norm(k, L->k_norm, m->n_kv_heads, m); }
        orc_rope(s->q, k, cs, sn, hd, m->n_heads, m->n_kv_heads);
        if (s->kv_type == ORC_F16) {   /* store_kv :188-205 */
            for (int i = 0; i < KV; i++) { s->kh[row * KV + i] = orc_f32_to_f16(k[i]); s->vh[row * KV + i] = orc_f32_to_f16(v[i]); }
        } else if (s->kv_type == ORC_Q8_0) {
            for (int h = 0; h < m->n_kv_heads; h++) {
                const size_t o = (size_t)h * hd;
                orc_quantize_row(s->kq + row * KV + o, s->kd + row * m->n_kv_heads + h, k + o, hd);
                orc_quantize_row(s->vq + row * KV + o, s->vd + row * m->n_kv_heads + h, v + o, hd);
            }
        }
        attention(s, l, pos);
        orc_quantize_q8(s->qa, s->da, s->ao, QD);
        matvec(s, s->xb2, &L->wo, s->qa, s->da);
        residual_add(m, s->x, s->xb2, L->post_attn_norm);
        orc_rmsnorm(s->xb, s->x, L->ffn_norm, D, m->norm_eps);
        orc_quantize_q8(s->qa, s->da, s->xb, D);
        matvec(s, s->hb, &L->w1, s->qa, s->da);
        matvec(s, s->hb2, &L->w3, s->qa, s->da);
        if (m->act == 1) orc_gelu_mul(s->hb, s->hb2, H);
        else orc_silu_mul(s->hb, s->hb2, H);
        orc_quantize_q8(s->qh, s->dh, s->hb, H);
        matvec(s, s->xb2, &L->w2, s->qh, s->dh);
        residual_add(m, s->x, s->xb2, L->post_ffn_norm);
    }
    if (!logits) return ORC_OK;
    orc_rmsnorm(s->xb, s->x, m->final_norm, D, m->norm_eps);
    orc_quantize_q8(s->qa, s->da, s->xb, D);
    matvec(s, logits, &m->wcls, s->qa, s->da);
    if (m->final_softcap > 0.0f)
        for (int i = 0; i < m->vocab; i++) logits[i] = m->final_softcap * tanhf(logits[i] / m->final_softcap);
    return ORC_OK;
}

int orc_prefill(orc_state *s, const int *tokens, int n, int pos0, float *logits) {
    const orc_model *m = s->m;
    if (n < 0 || pos0 < 0 || pos0 + n > m->max_seq) return ORC_E_SHAPE;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= m->vocab) return ORC_E_SHAPE;
    for (int i = 0; i < n; i++) {
        const int st = orc_forward(s, tokens[i], pos0 + i, logits ? logits + (size_t)i * m->vocab : NULL);
        if (st != ORC_OK) return st;
    }
    return ORC_OK;
}

/* ------------------------------------------------------------------ sampler
 * model/sampler.c restated: penalty (:30-42), xorshift64* (:44-49), argmax
 * (:51-55), softmax (kernels/scalar/k_scalar.c:66-77), the multinomial draw
 * (:57-64), top-k (:80-106; the k best in (p desc, id asc) order), sample_sorted
 * (:108-131), sample_topp (:133-155). Each call also reports how close the
 * draw came to a boundary between two tokens (relative to the mass it was
 * drawn from), so that a test can tell an implementation whose float sums
 * differ by rounding from one that picks another token. */
struct orc_sampler {
    orc_sampler_opts o;
    uint64_t rng;
    int vocab, n_recent, recent_at;
    int *recent;
    float *probs;
    int *order;
};

int orc_sampler_new(orc_sampler **out, int vocab, const orc_sampler_opts *o) {
    orc_sampler *s = calloc(1, sizeof *s);
    if (!s) return 4;
    s->o = *o;
    if (s->o.repeat_last_n < 0) s->o.repeat_last_n = 0;
    s->vocab = vocab;
    s->rng = o->seed ? o->seed : 0x9E3779B97F4A7C15ull;
    s->recent = calloc((size_t)(s->o.repeat_last_n > 0 ? s->o.repeat_last_n : 1), sizeof(int));
    s->probs = malloc(sizeof(float) * (size_t)vocab);
    s->order = malloc(sizeof(int) * (size_t)vocab);
    if (!s->recent || !s->probs || !s->order) { orc_sampler_free(s); return 4; }
    *out = s;
    return 0;
}

void orc_sampler_free(orc_sampler *s) {
    if (!s) return;
    free(s->recent);
    free(s->probs);
    free(s->order);
    free(s);
}

void orc_sampler_accept(orc_sampler *s, int token) {
    if (s->o.repeat_last_n <= 0 || token < 0 || token >= s->vocab) return;
    s->recent[s->recent_at] = token;
    s->recent_at = (s->recent_at + 1) % s->o.repeat_last_n;
    if (s->n_recent < s->o.repeat_last_n) s->n_recent++;
}

uint64_t orc_sampler_rng(const orc_sampler *s) { return s->rng; }

static float orc_coin(uint64_t *st) {
    uint64_t x = *st;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *st = x;
    return (float)((uint32_t)((x * 0x2545F4914F6CDD1Dull) >> 32) >> 8) / 16777216.0f;
}

static const float *g_sort_p;
static int by_prob_then_id(const void *a, const void *b) {
    const int x = *(const int *)a, y = *(const int *)b;
    if (g_sort_p[x] > g_sort_p[y]) return -1;
    if (g_sort_p[x] < g_sort_p[y]) return 1;
    return x - y;
}

/* distance of r from the two boundaries of the interval it falls in (the
 * cumulative sums of `seq`, ids into p, m of them, in order), over mass */
static float draw_margin(const float *p, const int *seq, int m, float r, float mass) {
    float lo = 0.0f, hi = 0.0f;
    for (int i = 0; i < m; i++) {
        hi = lo + p[seq ? seq[i] : i];
        if (r < hi) break;
        lo = hi;
    }
    const float d = fminf(fabsf(r - lo), fabsf(hi - r));
    return mass > 0.0f ? d / mass : d;
}

/* One ml_sample over logits[vocab] (overwritten by the penalty, as the
 * reference's are); *margin: see above (INFINITY for greedy). */
int orc_sample(orc_sampler *s, float *logits, float *margin) {
    const int n = s->vocab;
    *margin = INFINITY;
    if (s->o.repeat_penalty != 1.0f)
        for (int i = 0; i < s->n_recent; i++) {
            const int t = s->recent[i];
            int seen = 0;
            for (int j = 0; j < i; j++) seen |= s->recent[j] == t;
            if (seen || t >= n) continue;
            logits[t] = logits[t] > 0.0f ? logits[t] / s->o.repeat_penalty : logits[t] * s->o.repeat_penalty;
        }
    if (s->o.temperature == 0.0f) {
        int best = 0;
        for (int i = 1; i < n; i++) if (logits[i] > logits[best]) best = i;
        return best;
    }
    float *p = s->probs;
    for (int i = 0; i < n; i++) p[i] = logits[i] / s->o.temperature;
    orc_softmax(p, n);
    const float coin = orc_coin(&s->rng);
    const float topp = s->o.topp;
    if (s->o.topk > 0 && s->o.topk < n) {
        for (int i = 0; i < n; i++) s->order[i] = i;
        g_sort_p = p;
        qsort(s->order, (size_t)n, sizeof(int), by_prob_then_id);
        const int m = s->o.topk;
        float total = 0.0f;
        for (int i = 0; i < m; i++) total += p[s->order[i]];
        int last = m - 1;
        if (topp > 0.0f && topp < 1.0f) {
            float cum = 0.0f;
            for (int i = 0; i < m; i++) {
                cum += p[s->order[i]];
                if (cum > topp * total) { last = i; break; }
            }
            total = cum;
        }
        const float r = coin * total;
        *margin = draw_margin(p, s->order, last + 1, r, total);
        float cdf = 0.0f;
        for (int i = 0; i <= last; i++) {
            cdf += p[s->order[i]];
            if (r < cdf) return s->order[i];
        }
        return s->order[last];
    }
    if (topp <= 0.0f || topp >= 1.0f) {
        *margin = draw_margin(p, NULL, n, coin, 1.0f);
        float cdf = 0.0f;
        for (int i = 0; i < n; i++) {
            cdf += p[i];
            if (coin < cdf) return i;
        }
        return n - 1;
    }
    const float cutoff = n > 1 ? (1.0f - topp) / (float)(n - 1) : 0.0f;
    int m = 0;
    for (int i = 0; i < n; i++)
        if (p[i] >= cutoff) s->order[m++] = i;
    if (m == 0) {
        int best = 0;
        for (int i = 1; i < n; i++) if (p[i] > p[best]) best = i;
        return best;
    }
    g_sort_p = p;
    qsort(s->order, (size_t)m, sizeof(int), by_prob_then_id);
    float cum = 0.0f;
    int last = m - 1;
    for (int i = 0; i < m; i++) {
        cum += p[s->order[i]];
        if (cum > topp) { last = i; break; }
    }
    const float r = coin * cum;
    *margin = draw_margin(p, s->order, last + 1, r, cum);
    float cdf = 0.0f;
    for (int i = 0; i <= last; i++) {
        cdf += p[s->order[i]];
        if (r < cdf) return s->order[i];
    }
    return s->order[last];
}
