/* Batched prefill (kc_prefill.cu): what the runtime hands it. Host-only
 * declarations, shared by kc_runtime.cu and kc_prefill.cu. */
#ifndef KC_PREFILL_H
#define KC_PREFILL_H
#include <cuda_runtime.h>

#include "kc_internal.h"

namespace kc {

/* Shared memory the batched attention may use for its score rows. */
constexpr int PF_ATTN_SMEM_MAX = 200 * 1024;

/* One layer as the batched path sees it: device norms, this state's cache
 * rows of the layer, the RoPE tables it uses and its attention window. */
struct PfLayerRun {
    const float *attn_norm, *ffn_norm;
    void *kc, *vc;
    float *kd, *vd;
    const float *rcos, *rsin;
    int window;
    const float *q_norm, *k_norm;          /* per-head RMSNorm before RoPE, or null */
    const float *post_attn, *post_ffn;     /* RMSNorm of a block's output before the residual add, or null */
};

struct PfRun {
    kc_model *m;
    int kv_type;
    const PfLayerRun *layers;          /* [n_layers] */
    const uint8_t *emb_q;              /* the device embedding table */
    const void *emb_d;
    int emb_type, emb_d16;             /* T_Q8 / T_Q4, f16 scales */
    const float *final_norm;
    float *logits_dev;                 /* [logits_rows][vocab] */
    int logits_rows;
    unsigned *err;                     /* device error word */
    cudaStream_t st;
    PfScratch **scratch;               /* owned by the state */
    int batch;                         /* tokens per chunk */
};

/* Device byte offsets, into the weight stream, of the row records the
 * batched prefill's GEMM operands are packed from (a record: quants, then
 * block scales of the stream's type): Q|K|V [n_layers][q_dim + 2 kv_dim], O [n_layers][dim], gate
 * then up [n_layers][2 hidden], down [n_layers][dim], classifier [vocab]. */
struct PfRowTable {
    const unsigned long long *qkv, *wo, *w13, *w2, *cls;
    int d16;   /* the stream's block scales are f16 (else f32) */
};
/* Packs every GEMM operand of the model from its uploaded weight stream
 * (device to device; at upload). */
int pf_pack_model(kc_model *m, const uint8_t *stream, const PfRowTable &t, cudaStream_t st);

/* True when the batched kernels take this model and a chunk reaching
 * position last_pos. */
bool pf_fits(const kc_config &c, int kv_type, int last_pos);
/* Runs the n tokens at pos0.. (logits: host [n][vocab] or null) through the
 * operands pf_pack_model built. */
int pf_prefill(const PfRun &r, const int *tokens, int n, int pos0, float *logits);
void pf_free_model(PfModel *p);
void pf_free_scratch(PfScratch *p);
size_t pf_model_bytes(const PfModel *p);

}  // namespace kc

#endif
