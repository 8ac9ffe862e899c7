/* TEST INFRASTRUCTURE ONLY — the CPU oracle for the Krafla token loop.
 *
 * A plain-C restatement of the reference's scalar arithmetic (JonPark0/isa-lm,
 * "Krafla"): the Q8_0 activation rule, the scalar Q8/Q4 matvec, RMSNorm, RoPE,
 * softmax, SiLU/GELU, GQA attention over F32/F16/Q8 KV caches, and the decoder
 * forward of model/transformer.c. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference arm may call it; the CUDA product never
 * links or calls it.
 *
 * Parity pin: tests/test_oracle_pin.py checks every function here against the
 * reference's own scalar build (oracle/_ref, compiled from the reference
 * sources by oracle/Makefile) bit for bit, and against golden fixtures made by
 * the reference's Python tools (tests/golden/gen_golden.py).
 */
#ifndef KRAFLA_ORACLE_H
#define KRAFLA_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK 32

/* status codes: the reference's ml_status values (core/ml.h:7-14) */
enum { ORC_OK = 0, ORC_E_IO, ORC_E_FORMAT, ORC_E_SHAPE, ORC_E_NOMEM };
/* tensor / KV types: core/ml.h:67 */
enum { ORC_F32 = 0, ORC_Q8_0 = 1, ORC_Q4_0 = 2, ORC_F16 = 3 };

typedef struct orc_model orc_model;
typedef struct orc_state orc_state;

/* f16 <-> f32, IEEE round to nearest even (core/ml.c:39-62). */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);

/* Per-32-block Q8_0 activation quantization (kernels/scalar/k_scalar.c:39-57). */
void orc_quantize_q8(int8_t *q, float *d, const float *x, int k);
/* One scale over n values (ops/ops.c:81-96). */
void orc_quantize_row(int8_t *q, float *d, const float *x, int n);
/* y[r] for r in [r0, r1): scalar matvec (k_scalar.c:4-37). wq: int8 [rows*cols]
 * (Q8) or uint8 [rows*cols/2] (Q4); wd: float scales [rows*cols/32]. */
void orc_matvec(float *y, int type, const void *wq, const float *wd, int rows, int cols,
                const int8_t *xq, const float *xd, int r0, int r1);
/* int32 block dot products s[r][b] = sum_j w[r][32b+j] * x[32b+j]. */
void orc_block_sums(int32_t *s, int type, const void *wq, int rows, int cols, const int8_t *xq);
void orc_rmsnorm(float *o, const float *x, const float *w, int n, float eps);
void orc_softmax(float *x, int n);
void orc_rope(float *q, float *k, const float *cs, const float *sn, int hd, int nh, int nkv);
void orc_silu_mul(float *g, const float *u, int n);
void orc_gelu_mul(float *g, const float *u, int n);
void orc_dequant_row(float *out, int type, const void *wq, const float *wd, int cols, int row);

/* Model: parses an .mlb file (model/mlb.c:80-218) into host arrays. */
int orc_model_load(orc_model **out, const char *path);
void orc_model_free(orc_model *m);
/* Header fields, in this order: dim n_layers n_heads n_kv_heads hidden_dim
 * vocab max_seq head_dim kv_dim q_dim wtype q8_mask qkv_bias qk_norm
 * sliding_window act post_norms scale_f16 shared rope_type (20 ints). */
void orc_model_config(const orc_model *m, int *fields);

/* State: F32, F16 or Q8_0 KV cache (model/transformer.c:51-166). nthreads
 * only splits matvec rows; results do not depend on it. */
int orc_state_new(orc_state **out, orc_model *m, int kv_type, int nthreads);
void orc_state_free(orc_state *s);
/* One decode token (model/transformer.c:257-306). logits may be NULL (the
 * classifier is skipped, as ml_prefill does without logits). Returns ORC_E_SHAPE
 * for an out-of-range token or position. */
int orc_forward(orc_state *s, int token, int pos, float *logits);
/* n tokens at pos0..: per token the arithmetic of orc_forward, which the
 * reference's batched prefill matches bit for bit (transformer.c:381-384).
 * logits: [n][vocab] or NULL. */
int orc_prefill(orc_state *s, const int *tokens, int n, int pos0, float *logits);
/* Last hidden-state vector x [dim] after the latest orc_forward. */
const float *orc_state_x(const orc_state *s);
/* Debug views: 0 x, 1 q (after RoPE), 2 ao, 3 hb, 4 F32 K cache, 5 F32 V cache. */
const float *orc_state_buf(const orc_state *s, int which);
/* RoPE tables [max_seq][head_dim/2] computed as ml_state_init does. */
const float *orc_rope_cos(const orc_state *s);
const float *orc_rope_sin(const orc_state *s);

#ifdef __cplusplus
}
#endif
/* model/sampler.h restated (test infrastructure): options field for field
 * as ml_sampler_opts. */
typedef struct {
    float temperature, topp;
    int topk;
    float repeat_penalty;
    int repeat_last_n;
    uint64_t seed;
} orc_sampler_opts;
typedef struct orc_sampler orc_sampler;
int orc_sampler_new(orc_sampler **out, int vocab, const orc_sampler_opts *o);
void orc_sampler_free(orc_sampler *s);
void orc_sampler_accept(orc_sampler *s, int token);
uint64_t orc_sampler_rng(const orc_sampler *s);
int orc_sample(orc_sampler *s, float *logits, float *margin);

#endif
