/* model/transformer.c of the reference's `cuda` ISA build: the API of
 * model/transformer.h (ml_state_init, ml_prefill, ml_forward, ml_state_free,
 * ml_imatrix_size, ml_imatrix_enable, ml_prof_names) over the B200 token loop
 * of libkrafla_cuda.so (include/krafla_cuda.h).
 *
 * make -C isa-lm_b200/ref_shim REF=<reference tree> copies the reference,
 * applies isa_cuda.patch (the ISA in mk/isa.mk, this file in place of
 * transformer.c and the library on the link line in the Makefile, its name in
 * config/ml_config.h), places this file as model/transformer_cuda.c and builds
 * the reference's own apps with ISA=cuda.
 *
 * The model stays the reference's: ml_model_load maps and validates the file
 * as before, and ml_state_init hands the loaded arrays to kc_model_from_host
 * and uploads them to HBM, once per model (the states of one model share the
 * device copy; it goes with the last of them). ml_model_pack has nothing to
 * do in this build (no packed CPU kernels), so the arrays stay the file's.
 * The state's arena holds this build's handles; the pointer ml_forward
 * returns is the device state's host logits buffer, valid until the next
 * call, as the reference's is. Status codes are the same values on both
 * sides; a failure also prints the library's message on stderr. */
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "config/ml_config.h"
#include "core/threads.h"
#include "model/transformer.h"
#include "krafla_cuda.h"

_Static_assert(sizeof(kc_config) == sizeof(ml_config), "kc_config mirrors ml_config field for field");
_Static_assert((int)KC_E_ISA == (int)ML_E_ISA && (int)KC_E_NOMEM == (int)ML_E_NOMEM &&
                   (int)KC_E_SHAPE == (int)ML_E_SHAPE && (int)KC_E_IO == (int)ML_E_IO,
               "status codes are the same values");

const char *const ml_prof_names[ML_PROF_COUNT] = { "qkv", "attention", "wo", "ffn", "classifier", "other" };

/* The state's device side, at the start of its arena. */
typedef struct {
    kc_model *km;
    kc_state *ks;
    int batch;   /* the s->batch last given to kc_set_batch (0: none yet) */
} cuda_side;

static cuda_side *side(const ml_state *s) { return (cuda_side *)s->arena.base; }

/* Device copies of loaded models, shared by their states. */
typedef struct dev_model {
    const ml_model *m;
    kc_model *km;
    int refs;
    struct dev_model *next;
} dev_model;
static dev_model *g_models;
static pthread_mutex_t g_lock = PTHREAD_MUTEX_INITIALIZER;

static ml_status report(int st, const char *what) {
    if (st != KC_OK) {
        const char *why = kc_last_error();
        fprintf(stderr, "cuda: %s: %s%s%s\n", what, kc_status_str(st), why[0] ? ": " : "", why);
    }
    return (ml_status)st;
}

/* A matrix as the device library takes it: the scales as stored in the file
 * (f16 when the file has f16 scales), else the floats. */
static kc_tensor tensor(const ml_qtensor *t) {
    kc_tensor k;
    k.q = t->q;
    k.d = t->dh ? (const void *)t->dh : (const void *)t->d;
    k.rows = t->rows;
    k.cols = t->cols;
    k.type = t->type;
    k.d_f16 = t->dh != NULL;
    return k;
}

static ml_status upload(const ml_model *m, kc_model **out) {
    const ml_config *c = &m->cfg;
    kc_config kc;
    memcpy(&kc, c, sizeof kc);
    kc_layer_desc *L = calloc((size_t)c->n_layers, sizeof *L);
    if (!L) return ML_E_NOMEM;
    for (int l = 0; l < c->n_layers; l++) {
        const ml_layer *r = &m->layers[l];
        L[l].attn_norm = r->attn_norm;
        L[l].ffn_norm = r->ffn_norm;
        L[l].wq = tensor(&r->wq);
        L[l].wk = tensor(&r->wk);
        L[l].wv = tensor(&r->wv);
        L[l].wo = tensor(&r->wo);
        L[l].w1 = tensor(&r->w1);
        L[l].w2 = tensor(&r->w2);
        L[l].w3 = tensor(&r->w3);
        L[l].bq = r->bq;
        L[l].bk = r->bk;
        L[l].bv = r->bv;
        L[l].q_norm = r->q_norm;
        L[l].k_norm = r->k_norm;
        L[l].post_attn_norm = r->post_attn_norm;
        L[l].post_ffn_norm = r->post_ffn_norm;
        L[l].window = r->window;
        L[l].local_rope = r->local_rope;
    }
    const kc_tensor emb = tensor(&m->tok_emb), cls = tensor(&m->wcls);
    kc_model *km = NULL;
    int st = kc_model_from_host(&km, &kc, &emb, &cls, m->final_norm, L);
    free(L);
    if (st != KC_OK) return report(st, "model");
    st = kc_model_upload(km);
    if (st != KC_OK) {
        kc_model_free(km);
        return report(st, "upload");
    }
    *out = km;
    return ML_OK;
}

static ml_status acquire_model(const ml_model *m, kc_model **out) {
    pthread_mutex_lock(&g_lock);
    ml_status st = ML_OK;
    dev_model *d = g_models;
    while (d && d->m != m) d = d->next;
    if (!d) {
        d = calloc(1, sizeof *d);
        if (!d) st = ML_E_NOMEM;
        else if ((st = upload(m, &d->km)) != ML_OK) {
            free(d);
            d = NULL;
        } else {
            d->m = m;
            d->next = g_models;
            g_models = d;
        }
    }
    if (d) {
        d->refs++;
        *out = d->km;
    }
    pthread_mutex_unlock(&g_lock);
    return st;
}

static void release_model(kc_model *km) {
    pthread_mutex_lock(&g_lock);
    for (dev_model **p = &g_models; *p; p = &(*p)->next) {
        if ((*p)->km != km) continue;
        dev_model *d = *p;
        if (--d->refs == 0) {
            *p = d->next;
            kc_model_free(d->km);
            free(d);
        }
        break;
    }
    pthread_mutex_unlock(&g_lock);
}

size_t ml_imatrix_size(const ml_config *c) {
    return (size_t)c->n_layers * (2 * (size_t)c->dim + c->q_dim + c->hidden_dim) + c->dim;
}

ml_status ml_state_init(ml_state *s, ml_model *m, int nthreads, int kv_type) {
    memset(s, 0, sizeof *s);
    s->m = m;
    if (kv_type != ML_F32 && kv_type != ML_Q8_0 && kv_type != ML_F16) return ML_E_SHAPE;
    s->kv_type = kv_type;
    int st = kc_device_check();
    if (st != KC_OK) return report(st, "no B200 (sm_100) GPU for ISA=cuda");
    ml_status ms = ml_arena_init(&s->arena, sizeof(cuda_side));
    if (ms != ML_OK) return ms;
    cuda_side *d = side(s);
    memset(d, 0, sizeof *d);
    if ((ms = acquire_model(m, &d->km)) != ML_OK) goto fail;
    st = kc_state_init(&d->ks, d->km, nthreads, kv_type);
    if (st != KC_OK) {
        ms = report(st, "state");
        goto fail;
    }
    s->batch = ML_BATCH_MAX;
    /* the CPU pool of the API (callers read its size); the GPU result does not depend on it */
    if ((ms = ml_pool_create(&s->pool, nthreads)) != ML_OK) goto fail;
    return ML_OK;
fail:
    if (d->ks) kc_state_free(d->ks);
    if (d->km) release_model(d->km);
    ml_arena_free(&s->arena);
    memset(s, 0, sizeof *s);
    return ms;
}

ml_status ml_prefill(ml_state *s, const int *tokens, int n, int pos0, float *logits) {
    const ml_config *c = &s->m->cfg;
    if (n < 0 || pos0 < 0 || pos0 + n > c->max_seq) return ML_E_SHAPE;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= c->vocab) return ML_E_SHAPE;
    cuda_side *d = side(s);
    const int B = s->batch < 1 ? 1 : (s->batch > ML_BATCH_MAX ? ML_BATCH_MAX : s->batch);
    if (B != d->batch) {
        const int st = kc_set_batch(d->ks, B);
        if (st != KC_OK) return report(st, "batch");
        d->batch = B;
    }
    return report(kc_prefill(d->ks, tokens, n, pos0, logits), "prefill");
}

float *ml_forward(ml_state *s, int token, int pos) {
    const ml_config *c = &s->m->cfg;
    if (pos < 0 || pos >= c->max_seq || token < 0 || token >= c->vocab) return NULL;
    float *lg = kc_forward(side(s)->ks, token, pos);
    if (!lg) report(KC_E_IO, "forward");
    s->logits = lg;
    return lg;
}

/* The importance matrix sums the inputs of every matrix on the host; this
 * build keeps them on the device and does not collect it. */
ml_status ml_imatrix_enable(ml_state *s) {
    (void)s;
    fprintf(stderr, "cuda: the importance matrix is not collected by the cuda build\n");
    return ML_E_SHAPE;
}

void ml_state_free(ml_state *s) {
    cuda_side *d = s->arena.base ? side(s) : NULL;
    if (d && d->ks) kc_state_free(d->ks);
    if (d && d->km) release_model(d->km);
    if (s->pool) ml_pool_destroy(s->pool);
    ml_arena_free(&s->arena);
    free(s->imat);
    s->pool = NULL;
    s->imat = NULL;
}
