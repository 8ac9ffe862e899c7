/* Synthetic .mlb model writer: seeded N(0, sigma) weights, quantized by the
 * reference's rules, written in the reference's file format.
 *
 * Format: the 256-byte header and 64 B-aligned arrays of
 * docs/file-format.md and tools/mlb.py:326-379 (write_mlb); tensor order of
 * tools/mlb.py:295-312 (_order). Quantization restates tools/mlb.py:125-142
 * (quantize_q8, f32 or f16 scales) and tools/mlb.py:145-198 + 226-280
 * (the fitted Q4_0 rule, without an importance matrix), with float32
 * arithmetic in numpy's order so that the bytes equal what write_mlb writes
 * for the same float weights (checked against fixtures written by the
 * reference, tests/golden/).
 *
 * Weights come from a counter-based generator (SplitMix64 + Box-Muller), so a
 * tensor's values depend only on (seed, tensor id, index) and not on the
 * thread count. Compiled with -ffp-contract=off: every float op rounds alone.
 */
#define _GNU_SOURCE
#include <errno.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "mlb_writer.h"

#define QK 32
#define TINY 1e-30f    /* tools/mlb.py:15 */
#define SMALL 1e-6f    /* tools/mlb.py:152 */

/* ------------------------------------------------------------ f16 rounding */

/* IEEE binary16 from binary32, round to nearest even (numpy astype(float16)). */
static uint16_t f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7e00u;
    if (a >= 0x477ff000u) return sign | 0x7c00u;
    if (a < 0x38800000u) {
        float m;
        memcpy(&m, &a, 4);
        return sign | (uint16_t)lrintf(m * 16777216.0f);
    }
    const uint32_t r = a + 0xfffu + ((a >> 13) & 1u);
    return sign | (uint16_t)((r >> 13) - (112u << 10));
}

static float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) return (sign ? -1.0f : 1.0f) * (float)m * (1.0f / 16777216.0f);
    const uint32_t x = sign | (e == 31 ? 0x7f800000u | (m << 13) : ((e + 112u) << 23) | (m << 13));
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------ quantizers */

static float round_half_away(float v) { return truncf(v + copysignf(0.5f, v)); }

/* One block of 32: tools/mlb.py:125-142. d16: store the scale as f16 (the
 * quants are then taken against the rounded scale). Returns 0, or -1 when an
 * f16 scale would overflow (mlb.py:117-122 refuses those files). */
static int q8_block(const float *x, int8_t *q, float *d32, uint16_t *d16) {
    float amax = 0.0f;
    for (int j = 0; j < QK; j++) amax = fmaxf(amax, fabsf(x[j]));
    if (amax < TINY) amax = 0.0f;
    const float d = amax / 127.0f;
    float idv;
    if (d16) {
        const uint16_t h = f32_to_f16(d);
        if ((h & 0x7c00u) == 0x7c00u) return -1;
        *d16 = h;
        const float df = f16_to_f32(h);
        idv = df != 0.0f ? 1.0f / df : 0.0f;
    } else {
        *d32 = d;
        idv = amax != 0.0f ? 127.0f / amax : 0.0f;
    }
    for (int j = 0; j < QK; j++) {
        float v = round_half_away(x[j] * idv);
        v = fminf(fmaxf(v, -127.0f), 127.0f);
        q[j] = (int8_t)v;
    }
    return 0;
}

/* Sum of 32 values in numpy's _sum32 tree (tools/mlb.py:156-163). */
static float sum32(float *a) {
    for (int h = QK / 2; h >= 1; h /= 2)
        for (int i = 0; i < h; i++) a[i] = a[i] + a[i + h];
    return a[0];
}

/* One block: tools/mlb.py:166-198 (_q4_search without weights). levels in
 * -8..7 into lv, the fitted scale returned. */
static float q4_block_fit(const float *xin, float *lv) {
    int am = 0;
    float amx = fabsf(xin[0]);
    for (int j = 1; j < QK; j++)
        if (fabsf(xin[j]) > amx) { amx = fabsf(xin[j]); am = j; }   /* first index of the max |x| */
    const float mx = xin[am];
    const int zero = fabsf(mx) < TINY;
    const float inv = 1.0f / (zero ? 1.0f : mx);
    float y[QK], b[QK], w[QK], wb[QK], t[QK];
    for (int j = 0; j < QK; j++) y[j] = xin[j] * inv;
    const int small = fabsf(mx) < SMALL && !zero;
    const float up = small ? 1.0f / fabsf(mx) : 1.0f;
    for (int j = 0; j < QK; j++) {
        b[j] = xin[j] * up;
        w[j] = b[j] * b[j];
        wb[j] = w[j] * b[j];
    }
    float best = 0.0f, step = 0.0f;
    for (int k = -10; k < 3; k++) {
        const float s = (float)k * 0.2f;   /* Q4_STEPS: arange(-10, 3) * 0.2 in float32 */
        const float f = -(8.0f + s);
        float l[QK];
        for (int j = 0; j < QK; j++) l[j] = fminf(fmaxf(rintf(y[j] * f), -8.0f), 7.0f);
        for (int j = 0; j < QK; j++) t[j] = wb[j] * l[j];
        const float num = sum32(t);
        for (int j = 0; j < QK; j++) t[j] = w[j] * l[j] * l[j];
        const float den = sum32(t);
        const float score = num * num / (den > 0.0f ? den : 1.0f);
        if (k == -10 || score > best) { best = score; step = s; }
    }
    const float f = -(8.0f + step);
    for (int j = 0; j < QK; j++) lv[j] = fminf(fmaxf(rintf(y[j] * f), -8.0f), 7.0f);
    for (int j = 0; j < QK; j++) t[j] = w[j] * lv[j] * lv[j];
    const float den = sum32(t);
    float d;
    if (den > 0.0f) {
        for (int j = 0; j < QK; j++) t[j] = wb[j] * lv[j];
        d = sum32(t) / den / up;
    } else {
        d = 0.0f / up;
    }
    if (zero) {
        for (int j = 0; j < QK; j++) lv[j] = 0.0f;
        d = 0.0f;
    }
    return d;
}

/* tools/mlb.py:145-149: byte j = level j + 8 (low) | level j+16 + 8 (high). */
static int q4_block(const float *x, uint8_t *q, float *d32, uint16_t *d16) {
    float lv[QK];
    const float d = q4_block_fit(x, lv);
    for (int j = 0; j < QK / 2; j++)
        q[j] = (uint8_t)(((int)lv[j] + 8) | (((int)lv[j + QK / 2] + 8) << 4));
    if (d16) {
        const uint16_t h = f32_to_f16(d);
        if ((h & 0x7c00u) == 0x7c00u) return -1;
        *d16 = h;
    } else {
        *d32 = d;
    }
    return 0;
}

/* Quantizes nblocks blocks of x. type 1: Q8_0 (q: nblocks*32 bytes), 2: Q4_0
 * (nblocks*16 bytes). d: float[nblocks], or uint16 f16 [nblocks] when f16. */
int kw_quantize(int type, int f16, const float *x, long nblocks, void *q, void *d) {
    for (long b = 0; b < nblocks; b++) {
        int st;
        if (type == 1)
            st = q8_block(x + b * QK, (int8_t *)q + b * QK, f16 ? NULL : (float *)d + b, f16 ? (uint16_t *)d + b : NULL);
        else
            st = q4_block(x + b * QK, (uint8_t *)q + b * (QK / 2), f16 ? NULL : (float *)d + b,
                          f16 ? (uint16_t *)d + b : NULL);
        if (st) return -1;
    }
    return 0;
}

/* ------------------------------------------------------------ generator */

static uint64_t splitmix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* Uniform in (0, 1) with 53 random bits, never 0. */
static double unif(uint64_t seed, uint64_t tid, uint64_t i) {
    const uint64_t r = splitmix64(splitmix64(seed * 0x100000001b3ull ^ tid) ^ i);
    return ((double)(r >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

/* out[i] = sigma * N(0,1) for i in [i0, i0+n) of tensor `tid` (Box-Muller on
 * index pairs), rounded to float32. */
void kw_normal(uint64_t seed, uint64_t tid, uint64_t i0, long n, double sigma, float *out) {
    for (long k = 0; k < n; k++) {
        const uint64_t i = i0 + (uint64_t)k, pair = i >> 1;
        const double u1 = unif(seed, tid, 2 * pair), u2 = unif(seed, tid, 2 * pair + 1);
        const double r = sqrt(-2.0 * log(u1)), th = 6.283185307179586 * u2;
        out[k] = (float)(sigma * r * ((i & 1) ? sin(th) : cos(th)));
    }
}

/* ------------------------------------------------------------ writer */

typedef struct {
    FILE *f;
    int err;
} wctx;

static void put(wctx *w, const void *p, size_t n) {
    if (w->err) return;
    if (n && fwrite(p, 1, n, w->f) != n) { w->err = EIO; return; }
    static const uint8_t zeros[64] = { 0 };
    const size_t pad = (64 - n % 64) % 64;
    if (pad && fwrite(zeros, 1, pad, w->f) != pad) w->err = EIO;
}

typedef struct {
    const kw_config *c;
    uint64_t tid;
    int type, f16;
    long rows_per_chunk, cols;
    long row0, nrows;
    uint8_t *q;
    uint8_t *d;
    float *scratch;
    int err;
} mat_job;

/* Generates and quantizes rows [row0, row0 + nrows). */
static void *mat_run(void *p) {
    mat_job *j = p;
    const long nb = j->cols / QK;
    const size_t qrow = j->type == 1 ? (size_t)j->cols : (size_t)j->cols / 2;
    const size_t drow = (size_t)nb * (j->f16 ? 2 : 4);
    for (long r = 0; r < j->nrows; r++) {
        const long row = j->row0 + r;
        kw_normal(j->c->seed, j->tid, (uint64_t)row * (uint64_t)j->cols, j->cols, j->c->sigma, j->scratch);
        if (kw_quantize(j->type, j->f16, j->scratch, nb, j->q + (size_t)r * qrow, j->d + (size_t)r * drow)) {
            j->err = 1;
            return NULL;
        }
    }
    return NULL;
}

/* Writes a rows x cols matrix of tensor id `tid`, chunk by chunk of rows,
 * quants first and then scales, each padded to 64 bytes. The quants and
 * scales of the whole matrix are staged in memory (at most rows*cols bytes). */
static void put_matrix(wctx *w, const kw_config *c, uint64_t tid, long rows, long cols, int type) {
    if (w->err) return;
    const int f16 = c->scale_f16;
    const long nb = cols / QK;
    const size_t qbytes = (size_t)rows * (type == 1 ? (size_t)cols : (size_t)cols / 2);
    const size_t dbytes = (size_t)rows * nb * (f16 ? 2 : 4);
    uint8_t *q = malloc(qbytes ? qbytes : 1), *d = malloc(dbytes ? dbytes : 1);
    int nt = c->nthreads > 0 ? c->nthreads : 1;
    if (nt > 256) nt = 256;
    if (nt > rows) nt = (int)rows;
    if (nt < 1) nt = 1;
    mat_job jobs[256];
    pthread_t th[256];
    int started[256] = { 0 };
    if (!q || !d) { free(q); free(d); w->err = ENOMEM; return; }
    for (int t = 0; t < nt; t++) {
        const long r0 = rows * t / nt, r1 = rows * (t + 1) / nt;
        jobs[t] = (mat_job){ c, tid, type, f16, 0, cols, r0, r1 - r0,
                             q + (size_t)r0 * (type == 1 ? (size_t)cols : (size_t)cols / 2),
                             d + (size_t)r0 * nb * (f16 ? 2 : 4), malloc(sizeof(float) * (size_t)cols), 0 };
        if (!jobs[t].scratch) { w->err = ENOMEM; continue; }
        if (t > 0) started[t] = pthread_create(&th[t], NULL, mat_run, &jobs[t]) == 0;
    }
    if (!w->err) {
        mat_run(&jobs[0]);
        for (int t = 1; t < nt; t++) {
            if (started[t]) pthread_join(th[t], NULL);
            else if (jobs[t].scratch) mat_run(&jobs[t]);
        }
    } else {
        for (int t = 1; t < nt; t++) if (started[t]) pthread_join(th[t], NULL);
    }
    for (int t = 0; t < nt; t++) {
        if (jobs[t].err) w->err = EDOM;
        free(jobs[t].scratch);
    }
    put(w, q, qbytes);
    put(w, d, dbytes);
    free(q);
    free(d);
}

static void put_f32(wctx *w, const kw_config *c, uint64_t tid, long n, int normal) {
    float *v = malloc(sizeof(float) * (size_t)(n ? n : 1));
    if (!v) { w->err = ENOMEM; return; }
    if (normal) kw_normal(c->seed, tid, 0, n, c->bias_sigma, v);
    else for (long i = 0; i < n; i++) v[i] = 1.0f;   /* norm weights 1.0 */
    put(w, v, sizeof(float) * (size_t)n);
    free(v);
}

static void w32(uint8_t *h, int off, uint32_t v) { memcpy(h + off, &v, 4); }
static void wf(uint8_t *h, int off, float v) { memcpy(h + off, &v, 4); }

/* Matrix storage type by class bit (model/mlb.c:172, tools/mlb.py:69-74). */
static int mtype(const kw_config *c, int bits) { return c->wtype == 1 || (c->q8_mask & bits) ? 1 : 2; }

/* Tensor ids of the generator: tok_emb 1, wcls 2, final_norm 3, layer l
 * tensors 100 + 16 l + k. */
int kw_write_model(const char *path, const kw_config *c) {
    if (c->dim % QK || c->hidden_dim % QK || c->n_heads <= 0 || c->n_kv_heads <= 0 || c->n_heads % c->n_kv_heads)
        return EINVAL;
    const int hd = c->head_dim ? c->head_dim : c->dim / c->n_heads;
    const int qd = hd * c->n_heads, kvd = hd * c->n_kv_heads;
    if (qd % QK || kvd % QK) return EINVAL;
    wctx w = { fopen(path, "wb"), 0 };
    if (!w.f) return errno ? errno : EIO;
    uint8_t h[256];
    memset(h, 0, sizeof h);
    memcpy(h, "MLB1", 4);
    w32(h, 4, 1);
    w32(h, 8, (uint32_t)c->dim); w32(h, 12, (uint32_t)c->n_layers); w32(h, 16, (uint32_t)c->n_heads);
    w32(h, 20, (uint32_t)c->n_kv_heads); w32(h, 24, (uint32_t)c->hidden_dim); w32(h, 28, (uint32_t)c->vocab);
    w32(h, 32, (uint32_t)c->max_seq); wf(h, 36, c->rope_theta); wf(h, 40, c->norm_eps);
    w32(h, 44, (uint32_t)c->wtype); w32(h, 48, (uint32_t)(c->shared != 0));
    w32(h, 52, (uint32_t)c->rope_type); wf(h, 56, c->rope_factor); wf(h, 60, c->rope_lo); wf(h, 64, c->rope_hi);
    w32(h, 68, (uint32_t)c->rope_orig);
    w32(h, 72, (uint32_t)(c->wtype == 2 ? c->q8_mask : 0)); w32(h, 76, (uint32_t)(c->qkv_bias != 0));
    /* explicit head_dim only when it differs from dim / n_heads (tools/mlb.py:340) */
    w32(h, 80, (uint32_t)(hd != c->dim / c->n_heads || c->dim % c->n_heads ? hd : 0));
    w32(h, 120, (uint32_t)(c->scale_f16 != 0));
    if (fwrite(h, 1, sizeof h, w.f) != sizeof h) w.err = EIO;
    put_matrix(&w, c, 1, c->vocab, c->dim, mtype(c, 1 | (c->shared ? 2 : 0)));
    for (int l = 0; l < c->n_layers; l++) {
        const uint64_t b = 100 + 16 * (uint64_t)l;
        put_f32(&w, c, b + 0, c->dim, 0);                      /* attn_norm */
        put_matrix(&w, c, b + 1, qd, c->dim, mtype(c, 4));      /* wq */
        put_matrix(&w, c, b + 2, kvd, c->dim, mtype(c, 4));     /* wk */
        put_matrix(&w, c, b + 3, kvd, c->dim, mtype(c, 8));     /* wv */
        put_matrix(&w, c, b + 4, c->dim, qd, mtype(c, 16));     /* wo */
        if (c->qkv_bias) {
            put_f32(&w, c, b + 5, qd, 1);
            put_f32(&w, c, b + 6, kvd, 1);
            put_f32(&w, c, b + 7, kvd, 1);
        }
        put_f32(&w, c, b + 8, c->dim, 0);                      /* ffn_norm */
        put_matrix(&w, c, b + 9, c->hidden_dim, c->dim, mtype(c, 32));    /* w1 (gate) */
        put_matrix(&w, c, b + 10, c->dim, c->hidden_dim, mtype(c, 64));   /* w2 (down) */
        put_matrix(&w, c, b + 11, c->hidden_dim, c->dim, mtype(c, 32));   /* w3 (up) */
    }
    put_f32(&w, c, 3, c->dim, 0);                               /* final_norm */
    if (!c->shared) put_matrix(&w, c, 2, c->vocab, c->dim, mtype(c, 2));
    if (fclose(w.f) != 0 && !w.err) w.err = EIO;
    if (w.err) unlink(path);
    return w.err;
}

size_t kw_config_size(void) { return sizeof(kw_config); }
