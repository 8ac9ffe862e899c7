/* krafla_cuda.h — C ABI of the B200 (sm_100a) implementation of Krafla's
 * token loop (JonPark0/isa-lm): the decoder forward of model/transformer.c
 * and the ops it binds through ops/ops.h, on HBM-resident weights.
 *
 * Plain C types only: no CUDA or torch types cross this boundary. Every entry
 * point returns a status with the reference's ml_status values
 * (core/ml.h:7-14); CUDA failures are mapped onto them (out of device memory
 * -> KC_E_NOMEM, no sm_100 device -> KC_E_ISA, any other CUDA error -> KC_E_IO)
 * and kc_last_error() gives the message. Nothing here aborts.
 *
 * Threading: one caller thread per kc_state, as the reference's ml_state.
 */
#ifndef KRAFLA_CUDA_H
#define KRAFLA_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ml_status (core/ml.h:7-14), same values */
enum { KC_OK = 0, KC_E_IO = 1, KC_E_FORMAT = 2, KC_E_SHAPE = 3, KC_E_NOMEM = 4, KC_E_ISA = 5 };
/* tensor and KV cache types (core/ml.h:67) */
enum { KC_F32 = 0, KC_Q8_0 = 1, KC_Q4_0 = 2, KC_F16 = 3 };
/* RoPE scaling kinds of the header's rope_type (model/mlb.h:34) */
enum { KC_ROPE_NONE = 0, KC_ROPE_LLAMA3 = 1, KC_ROPE_LINEAR = 2, KC_ROPE_YARN = 3 };

/* The model header, field for field in the order of ml_config
 * (model/mlb.h:9-32), so that a reference build can pass &m->cfg. */
typedef struct {
    int dim, n_layers, n_heads, n_kv_heads, hidden_dim, vocab, max_seq, head_dim, kv_dim;
    int q_dim;
    float rope_theta, norm_eps;
    int wtype;
    unsigned q8_mask;
    int qkv_bias, qk_norm, sliding_window, layer_flags;
    float rope_local_theta;
    int act, post_norms;
    float embed_scale, attn_scale;
    int scale_f16;
    float attn_softcap, final_softcap;
    int rope_type, rope_orig_max_seq;
    float rope_factor, rope_low_freq_factor, rope_high_freq_factor;
    float rope_attn_factor;
} kc_config;

/* A quantized matrix in host memory, the file's SoA layout (core/ml.h:69-83):
 * q = quants (Q8: int8 [rows*cols]; Q4: uint8 [rows*cols/2], byte j = element
 * j low nibble, j+16 high nibble), d = block scales [rows*cols/32], as f16
 * when d_f16 is set, else float. */
typedef struct {
    const void *q;
    const void *d;
    int rows, cols, type, d_f16;
} kc_tensor;

/* One decoder layer's host arrays (model/mlb.h:42-50). Optional arrays NULL. */
typedef struct {
    const float *attn_norm, *ffn_norm;
    kc_tensor wq, wk, wv, wo, w1, w2, w3;
    const float *bq, *bk, *bv;
    const float *q_norm, *k_norm;
    const float *post_attn_norm, *post_ffn_norm;
    int window, local_rope;
} kc_layer_desc;

typedef struct kc_model kc_model;
typedef struct kc_state kc_state;

/* 0 when device 0 is a Blackwell sm_100 GPU this library runs on, else
 * KC_E_ISA: the device-side counterpart of the reference's ISA guard
 * (core/isa_check.h, app/main_guard.c:8-15). */
int kc_device_check(void);
const char *kc_status_str(int status);
/* Message of the last failure on this thread ("" if none). */
const char *kc_last_error(void);

/* Replaces ml_model_load (model/mlb.h:64, model/mlb.c:161-218): maps and
 * validates an .mlb file with the reference's rules (parse_header,
 * model/mlb.c:80-159; Q8 quants of -128 refused, mlb.c:34-36), keeping host
 * views of every array. No device memory is touched. */
int kc_model_load(kc_model **out, const char *path);
/* The same from arrays the caller already holds (a reference ml_model):
 * header + tensors, copied by kc_model_upload. layers: cfg->n_layers entries.
 * For a tied classifier pass wcls == tok_emb (same q pointer). */
int kc_model_from_host(kc_model **out, const kc_config *cfg, const kc_tensor *tok_emb, const kc_tensor *wcls,
                       const float *final_norm, const kc_layer_desc *layers);
/* Replaces ml_model_pack (model/pack_model.h:13-19): the one-time upload of
 * every quantized matrix (Q4/Q8 quants + f16 or f32 block scales), norm and
 * bias to HBM, in the decode kernel's per-SM stream layout; for an unsharded
 * model also the batched prefill's tensor-core operands (int8 tiles, float
 * scales), packed on the device from that stream. Idempotent. */
int kc_model_upload(kc_model *m);
const kc_config *kc_model_config(const kc_model *m);
/* Bytes of weights held on the device (decode stream, prefill operands, float arrays). */
size_t kc_model_device_bytes(const kc_model *m);
void kc_model_free(kc_model *m);

/* Tensor parallelism (no counterpart in the reference, which runs on one
 * device): splits a loaded model, before kc_model_upload, into rank's share of
 * world ranks, one process and one GPU per rank, Megatron style: Q/K/V rows by
 * heads and the KV cache by KV head, gate/up rows, O and down by columns (the
 * ranks' partial outputs are summed on the device after each), classifier rows
 * by vocabulary (the ranks exchange their best logit). world 1..KC_TP_MAX with
 * n_heads, n_kv_heads, q_dim/32 and hidden_dim/32 divisible by world.
 * kc_model_config keeps returning the file's configuration. */
#define KC_TP_MAX 8
int kc_model_shard(kc_model *m, int rank, int world);
/* This rank's share (9 ints): rank, world, n_heads, n_kv_heads, q_dim, kv_dim,
 * hidden_dim held here, first classifier row, classifier rows. */
int kc_model_shard_info(const kc_model *m, int *out);
/* Makes `device` the current CUDA device of the calling thread (a rank's GPU). */
int kc_set_device(int device);
/* Replaces ml_state_init (model/transformer.h:56, transformer.c:51-166):
 * device buffers, the KV cache [n_layers][max_seq][kv_dim] in HBM (kv_type
 * KC_F32, KC_F16 or KC_Q8_0) and RoPE tables computed on the host in double
 * exactly as the reference does. nthreads is accepted for the API's shape and
 * ignored (the result does not depend on it, as the reference's contract
 * says). KC_E_SHAPE for model features this build does not run. */
int kc_state_init(kc_state **out, kc_model *m, int nthreads, int kv_type);
/* Replaces ml_prefill (transformer.h:60, transformer.c:427-438): n host
 * tokens at positions pos0..; logits [n][vocab] (host) or NULL (classifier
 * skipped). KC_E_SHAPE when a position or token is out of range.
 * With the state's batch > 1 (the default) the tokens go through the model in
 * chunks of up to batch tokens, each projection one int8 tensor-core GEMM
 * whose per-row float accumulation follows the reference's packed kernels;
 * with batch 1 they run one decode step each, and the logits equal those of
 * kc_forward bit for bit. */
int kc_prefill(kc_state *s, const int *tokens, int n, int pos0, float *logits);
/* Prompt tokens per batched prefill step: the ml_state.batch field
 * (model/transformer.h:30-31) that ml_run --batch sets (app/ml_run.c:274,347);
 * 1..KC_BATCH_MAX, 1 = token by token. KC_E_SHAPE outside that range. */
#define KC_BATCH_MAX 1024
int kc_set_batch(kc_state *s, int batch);
/* Replaces ml_forward (transformer.h:62, transformer.c:257-306): logits for
 * `token` at `pos` in a host buffer owned by the state, valid until the next
 * call; NULL when pos or token is out of range (or on a device error). */
float *kc_forward(kc_state *s, int token, int pos);
/* Greedy decode of n tokens from `token` at `pos`, entirely on the device:
 * each step's argmax (first index of the maximum, model/sampler.c:57-61) is
 * the next step's input. out_tokens (host, n ints) receives the n chosen
 * tokens. The ml_run -T 0 / ml_bench decode loop (app/ml_bench.c:125-131). */
int kc_generate_greedy(kc_state *s, int token, int pos, int n, int *out_tokens);
/* Sampling on the device (model/sampler.h): the options of ml_sampler_opts,
 * field for field, so a reference build can pass &opts. */
typedef struct {
    float temperature;     /* 0 = greedy */
    float topp;            /* 0 or 1 = off */
    int topk;              /* 0 = off */
    float repeat_penalty;  /* 1 = off */
    int repeat_last_n;
    uint64_t seed;         /* 0: the reference's default seed */
} kc_sampler_opts;
typedef struct kc_sampler kc_sampler;
/* Replaces ml_sampler_init (model/sampler.c:6-19) for a state: the xorshift64*
 * state and the recent-token ring live in device memory. */
int kc_sampler_init(kc_sampler **out, kc_state *s, const kc_sampler_opts *o);
/* Replaces ml_sampler_accept (:23-28): records a context token for the penalty. */
int kc_sampler_accept(kc_sampler *p, int token);
/* Replaces ml_sample (:157-165) on the logits of the state's last step, on the
 * device (the logits stay there): penalty, greedy at temperature 0, else
 * softmax, top-k / top-p / multinomial with the same random stream and tie
 * rules; records the token as accepted. */
int kc_sample(kc_sampler *p, int *token);
/* n tokens from `token` at `pos`: per step one decode step and one device
 * sample (no logits copy); out_tokens (host, n ints). */
int kc_generate_sampled(kc_state *s, kc_sampler *p, int token, int pos, int n, int *out_tokens);
/* The sampler's xorshift64* state (tests and resumption). */
int kc_sampler_rng(kc_sampler *p, uint64_t *rng);
void kc_sampler_free(kc_sampler *p);

/* Debug view of the state after the last step: copies a device buffer to the
 * host (which: 0 x [dim], 1 q|k|v before RoPE [q_dim + 2 kv_dim], 2 attention
 * output [q_dim], 3 FFN hidden [hidden_dim] (2 and 3 as the quantized
 * activation of the next matrix, dequantized: q * d), 4 / 5 the K / V cache
 * [n_layers][max_seq][kv_dim]). KC_E_SHAPE when bytes is too small. */
int kc_debug_copy(kc_state *s, int which, void *dst, size_t bytes);
/* A sharded state's exchange buffer handle (CUDA IPC, KC_TP_HANDLE_BYTES
 * bytes) for the other ranks; then kc_tp_connect with every rank's handle in
 * rank order opens them. Until connected a sharded state refuses to run
 * (KC_E_SHAPE). Every rank must then make the same sequence of calls. */
#define KC_TP_HANDLE_BYTES 64
int kc_tp_handle(kc_state *s, void *out, size_t cap);
int kc_tp_connect(kc_state *s, const void *handles);
/* Replaces ml_state_free (transformer.h:65). */
void kc_state_free(kc_state *s);

/* Timing helper for bench.py: CUDA events on the state's stream around exactly
 * `steps` greedy decode steps (one launch of the step kernel) after `warmup`
 * untimed ones, starting at position pos; *ms receives the device
 * milliseconds. */
int kc_time_decode(kc_state *s, int token, int pos, int warmup, int steps, float *ms);
/* The device clock (ns) at the start of one decode step and after each of
 * its grid barriers (as CTA 0 sees them): per layer Q/K/V, attention, O,
 * gate/up, down, then the classifier. t: cap entries; *n: entries written. */
int kc_step_timeline(kc_state *s, int token, int pos, unsigned long long *t, int cap, int *n);

/* Per-CTA trace of one decode step (diagnostics): out[(phase * nctas + cta) *
 * 3 + k] = device clock (ns) when CTA cta finished the phase's activation
 * prologue (k = 0), arrived at its barrier (1) and was released (2); phases as
 * in kc_step_timeline. cap: entries of out. */
int kc_step_trace(kc_state *s, int token, int pos, unsigned long long *out, size_t cap, int *nphases, int *nctas);

/* Event log of one decode step (diagnostics): out[(cta * 2 + who) * cap + k] =
 * SM clock << 8 | event code, the k-th event of CTA cta's consumer (who 0:
 * 2 activation ready, 3 ring stage ready, 4 stage done, 5 barrier arrival,
 * 6 release) or producer (who 1: 7 waits for a free stage, 8 issued it).
 * out holds nctas * 2 * cap entries (nctas = the SM count), zero past the end. */
int kc_step_events(kc_state *s, int token, int pos, unsigned long long *out, unsigned cap, int *nctas);

/* ---- kernel-level entry points (device pointers, stream may be NULL) ----
 * These run the exact device code of the model path, for parity tests. */

/* Replaces ml_k_quantize_q8 (kernels/scalar/k_scalar.c:39-57), bit exact. */
int kc_quantize_q8_dev(int8_t *q, float *d, const float *x, int k, void *stream);
/* RMSNorm (k_scalar.c:59-64) of x by w, then quantize_q8 of the result: the
 * activation prologue of the decode projections. xn (optional, may be NULL)
 * receives the normalized floats. */
int kc_rmsnorm_quantize_dev(int8_t *q, float *d, float *xn, const float *x, const float *w, int n, float eps,
                            void *stream);
/* Replaces ml_k_matvec_q8 / ml_k_matvec_q4 (k_scalar.c:4-37) over all rows:
 * y[r] = sum_b int32(w.x over block b) * d_w[r,b] * d_x[b]. wd holds f16
 * scales when d_f16 is set. Uses the decode GEMV kernel. Asynchronous on
 * `stream`: a device wait that gave up is reported by the next kc_dev_sync. */
int kc_matvec_dev(float *y, int type, int d_f16, const void *wq, const void *wd, int rows, int cols,
                  const int8_t *xq, const float *xd, void *stream);
/* No counterpart in the reference (its CPU kernels need no device memory).
 * y = W . quantize_q8(x) for a float activation x on the device: the
 * quantized x lives in a file-scope device scratch of the library, so the call
 * allocates nothing, for callers that cannot allocate device memory per call
 * (a serving loop whose device memory is all reserved at set-up, or a host
 * framework that owns the device allocator and lets no library allocate on
 * its own). cols <= KC_NOALLOC_MAX_COLS, else KC_E_SHAPE with no launch. The
 * first call on each device looks up the scratch's address with that device
 * current, so it should come before any stream capture. The scratch is one
 * per device: calls that overlap in time (different streams or threads) race
 * on it; calls on one stream are ordered. Same results as kc_quantize_q8_dev
 * then kc_matvec_dev. A device wait that gave up is reported by the next
 * kc_dev_sync. */
#define KC_NOALLOC_MAX_COLS 16384
int kc_matvec_f32_noalloc(float *y, int type, int d_f16, const void *wq, const void *wd, int rows, int cols,
                          const float *x, void *stream);

/* The int32 block dot products s[r][b] of the same kernel code (bit exact
 * against the scalar kernels' integer sums). */
int kc_block_sums_dev(int32_t *s, int type, const void *wq, int rows, int cols, const int8_t *xq, void *stream);

/* Device memory helpers for callers without a CUDA runtime of their own. */
/* Replaces ml_matmul (ops/ops.c:51-79, the batched products of prefill) on
 * device buffers: y[t * rows + r] = sum_b s(r, t, b) * (d_w[r][b] * d_x[t][b])
 * for n quantized activation rows xq [n][cols], xd [n][cols/32], each block dot
 * an exact int32 from the int8 tensor cores and the float sum over blocks in
 * block order as the reference's packed kernels accumulate it. The weights are
 * repacked into temporary device memory per call. */
int kc_matmul_dev(float *y, int type, int d_f16, const void *wq, const void *wd, int rows, int cols,
                  const int8_t *xq, const float *xd, int n, void *stream);
void *kc_dev_alloc(size_t bytes);
void kc_dev_free(void *p);
int kc_memcpy_htod(void *dst, const void *src, size_t bytes);
int kc_memcpy_dtoh(void *dst, const void *src, size_t bytes);
/* Waits for the current device. KC_E_IO when a kernel-level matvec call
 * (kc_matvec_dev, kc_matvec_f32_noalloc) on it had a device wait give up
 * since the last kc_dev_sync (its error word is then cleared). */
int kc_dev_sync(void);
/* Diagnostics for tests of the error path: the polls of the kernel-level
 * matvec's first wait on each chunk of weights (0: it gives up at once;
 * negative: the default of about a second). A wait that runs out flags the
 * device error word and then waits for the chunk, so the results stay
 * correct and the next kc_dev_sync returns KC_E_IO. No counterpart in the
 * reference (its CPU kernels do not wait on copies). */
int kc_debug_wait_limit(int polls);
/* Testing: how the decode kernel shares the gate|up rows of models uploaded
 * from now on: -1 by the model (default), 0 whole 32-row blocks, 1 4-row units
 * with blocks split between CTAs. Returns the previous mode. No reference
 * counterpart. */
int kc_debug_ffn_split(int mode);

#ifdef __cplusplus
}
#endif
#endif
