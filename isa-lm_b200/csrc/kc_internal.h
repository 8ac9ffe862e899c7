/* Internal declarations shared by the host files of libkrafla_cuda. */
#ifndef KC_INTERNAL_H
#define KC_INTERNAL_H
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "krafla_cuda.h"

#define KC_QK 32

namespace kc {

/* Thread-local last error message (kc_last_error). */
void set_error(const std::string &msg);
void clear_error();

/* One host matrix: pointers into the mapped file (or the caller's arrays). */
struct HostMat {
    const void *q = nullptr;
    const void *d = nullptr;
    int rows = 0, cols = 0, type = 0, d16 = 0;
    size_t qbytes() const { return (size_t)rows * (type == KC_Q4_0 ? (size_t)cols / 2 : (size_t)cols); }
    size_t dbytes() const { return (size_t)rows * (cols / KC_QK) * (d16 ? 2 : 4); }
};

struct HostLayer {
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
    HostMat wq, wk, wv, wo, w1, w2, w3;
    const float *bq = nullptr, *bk = nullptr, *bv = nullptr;
    const float *q_norm = nullptr, *k_norm = nullptr;
    const float *post_attn_norm = nullptr, *post_ffn_norm = nullptr;
    int window = 0, local_rope = 0;
};

/* Device copy of one matrix. */
struct DevMat {
    const uint8_t *q = nullptr;
    const void *d = nullptr;
    int rows = 0, cols = 0, type = 0, d16 = 0;
};

struct DevLayer {
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
    DevMat wq, wk, wv, wo, w1, w2, w3;
    const float *bq = nullptr, *bk = nullptr, *bv = nullptr;
    const float *q_norm = nullptr, *k_norm = nullptr;
    const float *post_attn_norm = nullptr, *post_ffn_norm = nullptr;
    int window = 0, local_rope = 0;
};

struct PfModel;     /* packed weights of the batched prefill (kc_prefill.cu) */
struct PfScratch;   /* its per-state buffers */

/* Parses and validates the header of an .mlb (model/mlb.c:80-159). */
int parse_header(kc_config *cfg, int *shared, const uint8_t *h);
/* Takes the arrays of a mapped .mlb (model/mlb.c:161-218). */
int take_arrays(const kc_config &c, int shared, const uint8_t *data, size_t size, HostMat &tok_emb, HostMat &wcls,
                const float *&final_norm, std::vector<HostLayer> &layers);

}  // namespace kc

struct kc_model {
    kc_config cfg{};
    /* host side */
    void *map = nullptr;
    size_t map_size = 0;
    kc::HostMat tok_emb, wcls;
    const float *final_norm = nullptr;
    std::vector<kc::HostLayer> layers;
    int shared = 0;
    /* device side (after kc_model_upload) */
    int uploaded = 0;
    uint8_t *dev_base = nullptr;
    size_t dev_bytes = 0;
    kc::DevMat d_tok_emb;
    const float *d_final_norm = nullptr;
    std::vector<kc::DevLayer> d_layers;   /* norms and per-layer flags (the matrices live in the stream) */
    /* the weight stream: every CTA's rows in the order a step reads them */
    uint8_t *d_stream = nullptr;
    size_t stream_bytes = 0;
    unsigned long long *d_cta_base = nullptr;   /* [stream_G] */
    int stream_G = 0;
    int ffn_unit = 0;   /* rows per ownership unit of the gate|up phase in the stream (32 or 4), set at upload */
    /* the batched prefill's packed weights, built on first use */
    kc::PfModel *pf = nullptr;
    /* tensor parallelism (kc_model_shard): after sharding, cfg holds this rank's
     * dimensions (heads, q/kv widths, hidden) with the full vocab, cfg_full the
     * file's; the classifier rows held here are [cls_row0, cls_row0 + cls_rows) */
    int tp_rank = 0, tp_world = 1;
    kc_config cfg_full{};
    int cls_row0 = 0, cls_rows = 0;
    std::vector<std::vector<uint8_t>> shard_bufs;   /* column slices copied out of the file */
};

/* Classifier rows this model (or rank) holds. */
inline int model_cls_rows(const kc_model *m) { return m->tp_world > 1 ? m->cls_rows : m->cfg.vocab; }

#endif
