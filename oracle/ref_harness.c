/* TEST INFRASTRUCTURE ONLY — a ctypes-friendly harness around the reference's
 * own library (JonPark0/isa-lm "Krafla"), compiled from the reference sources
 * by oracle/Makefile into oracle/_ref/libkrafla_ref_<isa>.so.
 *
 * It only calls the reference's public API: ml_model_load / ml_model_pack
 * (model/mlb.h:64, model/pack_model.h:13), ml_state_init / ml_prefill /
 * ml_forward / ml_state_free (model/transformer.h:56-65) and the bound
 * kernels of config/ml_config.h. It is used (1) to pin the oracle in
 * krafla_oracle.c bit for bit against the reference's scalar build and
 * (2) as the timed CPU baseline (the reference's best build on the host).
 */
#include <stdlib.h>
#include <string.h>
#include "config/ml_config.h"
#include "core/clock.h"
#include "core/isa_check.h"
#include "core/quant_ref.h"
#include "model/pack_model.h"
#include "model/transformer.h"
#include "ops/ops.h"

typedef struct {
    ml_model m;
    ml_state s;
} ref_ctx;

const char *ref_isa_name(void) { return ML_ISA_NAME; }

/* 0 when this CPU runs the build's ISA (core/isa_check.h). */
int ref_isa_ok(void) {
    const char *missing = NULL;
    return ml_isa_check(&missing) == ML_OK ? 0 : 1;
}

int ref_open(const char *path, int nthreads, int kv_type, int pack, ref_ctx **out) {
    *out = NULL;
    ref_ctx *c = calloc(1, sizeof *c);
    if (!c) return ML_E_NOMEM;
    ml_status st = ml_model_load(&c->m, path);
    if (st != ML_OK) { free(c); return st; }
    st = ml_state_init(&c->s, &c->m, nthreads, kv_type);
    if (st != ML_OK) { ml_model_free(&c->m); free(c); return st; }
    if (pack && (st = ml_model_pack(&c->m, c->s.pool)) != ML_OK) {
        ml_state_free(&c->s);
        ml_model_free(&c->m);
        free(c);
        return st;
    }
    *out = c;
    return ML_OK;
}

void ref_close(ref_ctx *c) {
    if (!c) return;
    ml_state_free(&c->s);
    ml_model_free(&c->m);
    free(c);
}

void ref_set_batch(ref_ctx *c, int batch) { c->s.batch = batch; }
int ref_threads(ref_ctx *c) { return ml_pool_size(c->s.pool); }

/* Copies the logits of ml_forward into out (vocab floats); -1 when it returns NULL. */
int ref_forward(ref_ctx *c, int token, int pos, float *out) {
    const float *lg = ml_forward(&c->s, token, pos);
    if (!lg) return -1;
    if (out) memcpy(out, lg, sizeof(float) * (size_t)c->m.cfg.vocab);
    return 0;
}

int ref_prefill(ref_ctx *c, const int *tokens, int n, int pos0, float *logits) {
    return ml_prefill(&c->s, tokens, n, pos0, logits);
}

/* Greedy decode of n tokens starting from `token` at `pos`: ml_forward and the
 * first-index argmax of app/ml_bench.c:126-131. Writes the tokens; returns the
 * seconds it took (wall clock, ml_now). */
double ref_decode_greedy(ref_ctx *c, int token, int pos, int n, int *out) {
    const double t0 = ml_now();
    for (int i = 0; i < n; i++) {
        const float *lg = ml_forward(&c->s, token, pos + i);
        if (!lg) return -1.0;
        int best = 0;
        for (int j = 1; j < c->m.cfg.vocab; j++) if (lg[j] > lg[best]) best = j;
        token = best;
        if (out) out[i] = best;
    }
    return ml_now() - t0;
}

/* Seconds for ml_prefill of n tokens without logits (app/ml_bench.c:120-122). */
double ref_time_prefill(ref_ctx *c, const int *tokens, int n, int pos0) {
    const double t0 = ml_now();
    if (ml_prefill(&c->s, tokens, n, pos0, NULL) != ML_OK) return -1.0;
    return ml_now() - t0;
}

/* The build's bound kernels, for the kernel-level pins. */
void ref_quantize_q8(int8_t *q, float *d, const float *x, int k) {
    ml_qact a = { q, d, k };
    ml_k_quantize_q8(&a, x, k);
}

void ref_quantize_q8_scalar(int8_t *q, float *d, const float *x, int k) {
    ml_qact a = { q, d, k };
    ml_k_quantize_q8_scalar(&a, x, k);
}

void ref_quantize_row(int8_t *q, float *d, const float *x, int n) { ml_quantize_row(q, d, x, n); }

void ref_matvec_scalar(float *y, int type, const void *wq, const float *wd, int rows, int cols,
                       const int8_t *xq, const float *xd, int r0, int r1) {
    ml_qtensor W = { (const int8_t *)wq, wd, rows, cols, (uint8_t)type, NULL, NULL, NULL, 0 };
    ml_qact x = { (int8_t *)xq, (float *)xd, cols };
    if (type == ML_Q8_0) ml_k_matvec_q8_scalar(y, &W, &x, r0, r1);
    else ml_k_matvec_q4_scalar(y, &W, &x, r0, r1);
}

void ref_rmsnorm_scalar(float *o, const float *x, const float *w, int n, float eps) { ml_k_rmsnorm_scalar(o, x, w, n, eps); }
void ref_softmax_scalar(float *x, int n) { ml_k_softmax_scalar(x, n); }
void ref_silu_mul_scalar(float *g, const float *u, int n) { ml_k_silu_mul_scalar(g, u, n); }
void ref_rope_scalar(float *q, float *k, const float *cs, const float *sn, int hd, int nh, int nkv) {
    ml_k_rope_scalar(q, k, cs, sn, hd, nh, nkv);
}
uint16_t ref_f32_to_f16(float f) { return ml_f32_to_f16(f); }
float ref_f16_to_f32(uint16_t h) { return ml_f16_to_f32(h); }

/* RoPE tables of the state: [max_seq][head_dim/2]. */
const float *ref_rope_cos(ref_ctx *c) { return c->s.rope_cos; }
const float *ref_rope_sin(ref_ctx *c) { return c->s.rope_sin; }

/* The reference's own sampler (model/sampler.h): init, accept the context
 * tokens, then for each logits row ml_sample and accept its choice. */
#include "model/sampler.h"
int ref_sample_seq(const ml_sampler_opts *o, int vocab, const int *context, int n_context, float *logits, int rows,
                   int *out, uint64_t *rng_out) {
    ml_sampler s;
    ml_status st = ml_sampler_init(&s, vocab, o);
    if (st != ML_OK) return st;
    for (int i = 0; i < n_context; i++) ml_sampler_accept(&s, context[i]);
    for (int r = 0; r < rows; r++) {
        out[r] = ml_sample(&s, logits + (size_t)r * vocab, vocab);
        ml_sampler_accept(&s, out[r]);
    }
    *rng_out = s.rng;
    ml_sampler_free(&s);
    return ML_OK;
}
