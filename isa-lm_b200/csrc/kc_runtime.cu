/* Runtime of libkrafla_cuda: HBM upload of the model, the decode state with
 * its device arena and KV cache, the launches of the persistent step kernel
 * (one cooperative launch for many token steps: token and position live in
 * device memory), and the C ABI of include/krafla_cuda.h. */
#include <cmath>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <cstdlib>
#include <new>
#include <atomic>
#include <functional>
#include <mutex>
#include <thread>
#include <string>
#include <numeric>
#include <vector>
#include <sys/mman.h>

#include "kc_internal.h"
#include "kc_kernels.cuh"
#include "kc_step.cuh"
#include "kc_prefill.h"
#include "kc_sampler.cuh"

namespace kc {
static thread_local std::string g_err;
void set_error(const std::string &msg) { g_err = msg; }
void clear_error() { g_err.clear(); }

static int cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return KC_OK;
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    (void)cudaGetLastError();
    if (e == cudaErrorMemoryAllocation) return KC_E_NOMEM;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver || e == cudaErrorNoKernelImageForDevice)
        return KC_E_ISA;
    return KC_E_IO;
}
}  // namespace kc

#define CK(call)                                                      \
    do {                                                              \
        cudaError_t e_ = (call);                                      \
        if (e_ != cudaSuccess) return kc::cuda_status(e_, #call);     \
    } while (0)

using namespace kc;

static size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

extern "C" const char *kc_last_error(void) { return kc::g_err.c_str(); }

extern "C" const char *kc_status_str(int s) {
    switch (s) {
    case KC_OK: return "ok";
    case KC_E_IO: return "i/o error";
    case KC_E_FORMAT: return "bad file format";
    case KC_E_SHAPE: return "bad tensor shape";
    case KC_E_NOMEM: return "out of memory";
    case KC_E_ISA: return "device lacks required architecture";
    }
    return "unknown";
}

extern "C" int kc_device_check(void) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        (void)cudaGetLastError();
        set_error("no CUDA device");
        return KC_E_ISA;
    }
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, 0));
    if (prop.major != 10 || prop.minor != 0) {
        set_error("device 0 is sm_" + std::to_string(prop.major * 10 + prop.minor) + ", this build runs on sm_100a");
        return KC_E_ISA;
    }
    return KC_OK;
}

/* ------------------------------------------------------------------ model */

extern "C" int kc_model_from_host(kc_model **out, const kc_config *cfg, const kc_tensor *tok_emb,
                                  const kc_tensor *wcls, const float *final_norm, const kc_layer_desc *layers) {
    *out = nullptr;
    kc_model *m = new (std::nothrow) kc_model();
    if (!m) return KC_E_NOMEM;
    m->cfg = *cfg;
    auto conv = [](const kc_tensor &t) {
        HostMat h;
        h.q = t.q; h.d = t.d; h.rows = t.rows; h.cols = t.cols; h.type = t.type; h.d16 = t.d_f16;
        return h;
    };
    m->tok_emb = conv(*tok_emb);
    m->wcls = conv(*wcls);
    m->shared = wcls->q == tok_emb->q;
    m->final_norm = final_norm;
    m->layers.resize((size_t)cfg->n_layers);
    for (int l = 0; l < cfg->n_layers; l++) {
        const kc_layer_desc &s = layers[l];
        HostLayer &L = m->layers[(size_t)l];
        L.attn_norm = s.attn_norm; L.ffn_norm = s.ffn_norm;
        L.wq = conv(s.wq); L.wk = conv(s.wk); L.wv = conv(s.wv); L.wo = conv(s.wo);
        L.w1 = conv(s.w1); L.w2 = conv(s.w2); L.w3 = conv(s.w3);
        L.bq = s.bq; L.bk = s.bk; L.bv = s.bv; L.q_norm = s.q_norm; L.k_norm = s.k_norm;
        L.post_attn_norm = s.post_attn_norm; L.post_ffn_norm = s.post_ffn_norm;
        L.window = s.window; L.local_rope = s.local_rope;
    }
    *out = m;
    return KC_OK;
}

extern "C" const kc_config *kc_model_config(const kc_model *m) { return m->tp_world > 1 ? &m->cfg_full : &m->cfg; }

extern "C" int kc_model_shard_info(const kc_model *m, int *out) {
    const kc_config &c = m->cfg;
    const int v[9] = { m->tp_rank, m->tp_world, c.n_heads, c.n_kv_heads, c.q_dim, c.kv_dim, c.hidden_dim,
                       m->cls_row0, model_cls_rows(m) };
    std::memcpy(out, v, sizeof v);
    return KC_OK;
}

extern "C" int kc_set_device(int device) {
    clear_error();
    CK(cudaSetDevice(device));
    return KC_OK;
}

/* Rows [r0, r0 + n) of a file matrix: a view. */
static HostMat row_view(const HostMat &M, int r0, int n) {
    HostMat v = M;
    const size_t qrow = M.type == KC_Q4_0 ? (size_t)M.cols / 2 : (size_t)M.cols;
    const size_t drow = (size_t)(M.cols / KC_QK) * (M.d16 ? 2 : 4);
    v.q = (const uint8_t *)M.q + (size_t)r0 * qrow;
    v.d = (const uint8_t *)M.d + (size_t)r0 * drow;
    v.rows = n;
    return v;
}

/* Columns [c0, c0 + n) of every row (c0, n multiples of 32): a copy kept by the model. */
static HostMat col_slice(kc_model *m, const HostMat &M, int c0, int n) {
    const size_t nb = (size_t)M.cols / KC_QK, b0 = (size_t)c0 / KC_QK, wb = (size_t)n / KC_QK;
    const size_t bq = M.type == KC_Q4_0 ? KC_QK / 2 : KC_QK, ds = M.d16 ? 2 : 4;
    std::vector<uint8_t> q((size_t)M.rows * wb * bq), d((size_t)M.rows * wb * ds);
    for (size_t r = 0; r < (size_t)M.rows; r++) {
        std::memcpy(q.data() + r * wb * bq, (const uint8_t *)M.q + (r * nb + b0) * bq, wb * bq);
        std::memcpy(d.data() + r * wb * ds, (const uint8_t *)M.d + (r * nb + b0) * ds, wb * ds);
    }
    m->shard_bufs.push_back(std::move(q));
    m->shard_bufs.push_back(std::move(d));
    HostMat v = M;
    v.q = m->shard_bufs[m->shard_bufs.size() - 2].data();
    v.d = m->shard_bufs.back().data();
    v.cols = n;
    return v;
}

extern "C" int kc_model_shard(kc_model *m, int rank, int world) {
    clear_error();
    const kc_config c = m->cfg;
    if (m->uploaded || m->tp_world > 1) {
        set_error("shard a model once, before kc_model_upload");
        return KC_E_SHAPE;
    }
    if (world < 1 || world > KC_TP_MAX || rank < 0 || rank >= world) return KC_E_SHAPE;
    if (world == 1) return KC_OK;
    if (c.post_norms) {
        set_error("post-norm models do not run tensor parallel");
        return KC_E_SHAPE;
    }
    if (c.n_heads % world || c.n_kv_heads % world || (c.q_dim / world) % KC_QK || c.q_dim % world ||
        (c.hidden_dim / world) % KC_QK || c.hidden_dim % world) {
        set_error("heads, q_dim/32 and hidden_dim/32 must divide by the number of ranks");
        return KC_E_SHAPE;
    }
    const int qd = c.q_dim / world, kvd = c.kv_dim / world, hid = c.hidden_dim / world;
    for (HostLayer &H : m->layers) {
        H.wq = row_view(H.wq, rank * qd, qd);
        H.wk = row_view(H.wk, rank * kvd, kvd);
        H.wv = row_view(H.wv, rank * kvd, kvd);
        if (H.bq) { H.bq += (size_t)rank * qd; H.bk += (size_t)rank * kvd; H.bv += (size_t)rank * kvd; }
        H.wo = col_slice(m, H.wo, rank * qd, qd);
        H.w1 = row_view(H.w1, rank * hid, hid);
        H.w3 = row_view(H.w3, rank * hid, hid);
        H.w2 = col_slice(m, H.w2, rank * hid, hid);
    }
    const int v0 = (int)((long long)c.vocab * rank / world), v1 = (int)((long long)c.vocab * (rank + 1) / world);
    m->wcls = row_view(m->shared ? m->tok_emb : m->wcls, v0, v1 - v0);
    m->shared = 0;
    m->cls_row0 = v0;
    m->cls_rows = v1 - v0;
    m->cfg_full = c;
    m->cfg.n_heads = c.n_heads / world;
    m->cfg.n_kv_heads = c.n_kv_heads / world;
    m->cfg.q_dim = qd;
    m->cfg.kv_dim = kvd;
    m->cfg.hidden_dim = hid;
    m->tp_rank = rank;
    m->tp_world = world;
    return KC_OK;
}
extern "C" size_t kc_model_device_bytes(const kc_model *m) { return m->dev_bytes + pf_model_bytes(m->pf); }

extern "C" void kc_model_free(kc_model *m) {
    if (!m) return;
    if (m->dev_base) cudaFree(m->dev_base);
    if (m->d_stream) cudaFree(m->d_stream);
    if (m->d_cta_base) cudaFree(m->d_cta_base);
    pf_free_model(m->pf);
    if (m->map) munmap(m->map, m->map_size);
    delete m;
}

namespace {
/* Upload plan: every host array, its size, and where its device pointer goes. */
struct Item {
    const void *src;
    size_t bytes;
    const void **dst;
};
}  // namespace

/* Types and shapes of the streamed matrices; KC_E_SHAPE when a matrix class
 * changes type between layers or a matrix is not Q8_0/Q4_0. */
/* Ownership of the gate|up phase's rows (kc_debug_ffn_split): -1 by the
 * model, 0 whole blocks, 1 split blocks. */
static int g_ffn_split = -1;

extern "C" int kc_debug_ffn_split(int mode) {
    const int old = g_ffn_split;
    g_ffn_split = mode < 0 ? -1 : (mode ? 1 : 0);
    return old;
}

/* Rows per unit of the gate|up phase for G CTAs: whole 32-row blocks (each CTA
 * quantizes its own blocks), unless whole blocks leave the busiest CTA more
 * than ~2 us of weight bytes (at its share of the HBM rate) above the average,
 * then 4-row units with split blocks (their CTAs exchange one maximum). */
static int ffn_unit(const kc_config &c, const StreamGeom &g, int G) {
    if (g_ffn_split >= 0) return g_ffn_split ? 4 : QK;
    const int nbk = c.hidden_dim / QK, maxb = (nbk + G - 1) / G;
    const double block_bytes = 2.0 * QK * rec_bytes(g.t_up, g.d16_up, c.dim, 0);
    const double gap_us = ((double)maxb - (double)nbk / G) * block_bytes / 44000.0;
    return gap_us > 2.0 ? 4 : QK;
}

static int stream_geom(const kc_model *m, StreamGeom &g) {
    const kc_config &c = m->cfg;
    const HostLayer &L0 = m->layers[0];
    const HostMat &cls = m->shared ? m->tok_emb : m->wcls;
    auto ty = [](const HostMat &h) { return h.type == KC_Q4_0 ? T_Q4 : T_Q8; };
    g = StreamGeom{};
    g.dim = c.dim; g.q_dim = c.q_dim; g.kv_dim = c.kv_dim; g.hidden = c.hidden_dim; g.vocab = model_cls_rows(m);
    g.t_q = ty(L0.wq); g.t_k = ty(L0.wk); g.t_v = ty(L0.wv); g.t_o = ty(L0.wo);
    g.t_up = ty(L0.w1); g.t_down = ty(L0.w2); g.t_cls = ty(cls);
    g.d16_q = L0.wq.d16; g.d16_k = L0.wk.d16; g.d16_v = L0.wv.d16; g.d16_o = L0.wo.d16;
    g.d16_up = L0.w1.d16; g.d16_down = L0.w2.d16; g.d16_cls = cls.d16;
    g.b_q = L0.bq != nullptr; g.b_k = L0.bk != nullptr; g.b_v = L0.bv != nullptr;
    auto same = [](const HostMat &a, const HostMat &b) { return a.type == b.type && a.d16 == b.d16; };
    auto quant = [](const HostMat &h) { return h.type == KC_Q4_0 || h.type == KC_Q8_0; };
    for (const HostLayer &H : m->layers) {
        const bool ok = same(H.wq, L0.wq) && same(H.wk, L0.wk) && same(H.wv, L0.wv) && same(H.wo, L0.wo) &&
                        same(H.w1, L0.w1) && same(H.w3, L0.w1) && same(H.w2, L0.w2) && (H.bq != nullptr) == g.b_q &&
                        (H.bk != nullptr) == g.b_k && (H.bv != nullptr) == g.b_v && quant(H.wq) && quant(H.wk) &&
                        quant(H.wv) && quant(H.wo) && quant(H.w1) && quant(H.w2);
        if (!ok) {
            set_error("weight types differ between layers or are not Q8_0/Q4_0");
            return KC_E_SHAPE;
        }
    }
    if (!quant(cls)) {
        set_error("classifier is not Q8_0/Q4_0");
        return KC_E_SHAPE;
    }
    /* one block-scale type for the whole stream (the step kernel is built per
     * type): f16 when every streamed matrix has f16 scales, else f32 (f16
     * scales widened, exactly) */
    if (!(g.d16_q && g.d16_k && g.d16_v && g.d16_o && g.d16_up && g.d16_down && g.d16_cls))
        g.d16_q = g.d16_k = g.d16_v = g.d16_o = g.d16_up = g.d16_down = g.d16_cls = 0;
    g.d_unit = m->ffn_unit ? m->ffn_unit : QK;   /* set by upload_stream */
    return KC_OK;
}

/* An IEEE half as float (exact: every half is a float). */
static float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, mm = h & 0x3ffu;
    if (e == 0) return (sign ? -1.0f : 1.0f) * (float)mm * (1.0f / 16777216.0f);
    const uint32_t x = sign | (e == 31 ? 0x7f800000u | (mm << 13) : ((e + 112u) << 23) | (mm << 13));
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

/* One row record of the stream: quants, scales (f16 as in the file when the
 * stream's scales are f16 (s16), else f32), bias, zero padding to rec. */
static uint8_t *put_rec(uint8_t *dst, const HostMat &M, int r, const float *bias, int rec, bool s16) {
    const size_t qrow = M.type == KC_Q4_0 ? (size_t)M.cols / 2 : (size_t)M.cols, nb = (size_t)M.cols / KC_QK;
    const size_t dsz = M.d16 ? 2 : 4;
    std::memcpy(dst, (const uint8_t *)M.q + (size_t)r * qrow, qrow);
    const uint8_t *d = (const uint8_t *)M.d + (size_t)r * nb * dsz;
    if (M.d16 && !s16) {
        for (size_t b = 0; b < nb; b++) {
            uint16_t h;
            std::memcpy(&h, d + 2 * b, 2);
            const float f = half_to_float(h);
            std::memcpy(dst + qrow + 4 * b, &f, 4);
        }
    } else {
        std::memcpy(dst + qrow, d, nb * dsz);
    }
    size_t off = qrow + nb * (s16 ? 2 : 4);
    if (bias) {
        std::memcpy(dst + off, bias + r, sizeof(float));
        off += sizeof(float);
    }
    std::memset(dst + off, 0, (size_t)rec - off);
    return dst + rec;
}

/* Part `part` of CTA j's stream: layer `part`'s A, C, D, E phases of
 * make_plan, or (part == n_layers) the classifier. */
static size_t fill_stream_part(const kc_model *m, const PhasePlan *P, int part, uint8_t *dst) {
    const kc_config &c = m->cfg;
    uint8_t *p = dst;
    const HostMat &cls = m->shared ? m->tok_emb : m->wcls;
    if (part < c.n_layers) {
        const HostLayer &H = m->layers[(size_t)part];
        for (int s = 0; s < P[PH_A].nseg; s++) {
            const Seg &S = P[PH_A].seg[s];
            const bool isq = S.row0 < c.q_dim, isk = !isq && S.row0 < c.q_dim + c.kv_dim;
            const HostMat &M = isq ? H.wq : isk ? H.wk : H.wv;
            const float *bias = isq ? H.bq : isk ? H.bk : H.bv;
            const int lo = isq ? 0 : isk ? c.q_dim : c.q_dim + c.kv_dim;
            for (int r = 0; r < S.rows; r++) p = put_rec(p, M, S.row0 + r - lo, bias, S.rec, S.d16);
        }
        const Seg &C = P[PH_C].seg[0];
        for (int r = 0; r < C.rows; r++) p = put_rec(p, H.wo, C.row0 + r, nullptr, C.rec, C.d16);
        const Seg &D = P[PH_D].seg[0];
        for (int r = 0; r < D.rows; r++) {
            p = put_rec(p, H.w1, D.row0 + r, nullptr, D.rec / 2, D.d16);
            p = put_rec(p, H.w3, D.row0 + r, nullptr, D.rec / 2, D.d16);
        }
        const Seg &E = P[PH_E].seg[0];
        for (int r = 0; r < E.rows; r++) p = put_rec(p, H.w2, E.row0 + r, nullptr, E.rec, E.d16);
    } else {
        const Seg &F = P[PH_F].seg[0];
        for (int r = 0; r < F.rows; r++) p = put_rec(p, cls, F.row0 + r, nullptr, F.rec, F.d16);
    }
    return (size_t)(p - dst);
}

static size_t stream_layer_bytes(const PhasePlan *P) {
    return (size_t)(P[PH_A].bytes + P[PH_C].bytes + P[PH_D].bytes + P[PH_E].bytes);
}
static size_t stream_cta_bytes(const kc_model *m, const PhasePlan *P) {
    return (size_t)m->cfg.n_layers * stream_layer_bytes(P) + (size_t)P[PH_F].bytes;
}

/* Host -> device upload through pinned staging (the load path): W worker
 * threads, each with two pinned slots and its own stream; a worker fills one
 * slot on the CPU (a gather from the mapped file) while the copy of its other
 * slot runs, so the gathers of all workers and the copies overlap. A job is
 * `bytes` (<= the slot size) written by fill(slot) and copied to dst. */
struct UploadJob {
    uint8_t *dst;
    size_t bytes;
    std::function<size_t(uint8_t *)> fill;   /* returns the bytes written (checked) */
};

static int upload_jobs(const std::vector<UploadJob> &jobs, size_t slot) {
    if (jobs.empty()) return KC_OK;
    int dev = 0;
    CK(cudaGetDevice(&dev));
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const int W = (int)std::min<size_t>({ (size_t)8, (size_t)hw, jobs.size() });
    std::vector<uint8_t *> buf((size_t)2 * W, nullptr);
    std::vector<cudaStream_t> st((size_t)W, nullptr);
    std::vector<cudaEvent_t> ev((size_t)2 * W, nullptr);
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 2 * W && e == cudaSuccess; i++) {
        e = cudaHostAlloc((void **)&buf[(size_t)i], slot, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev[(size_t)i], cudaEventDisableTiming);
    }
    for (int w = 0; w < W && e == cudaSuccess; w++) e = cudaStreamCreateWithFlags(&st[(size_t)w], cudaStreamNonBlocking);
    std::atomic<size_t> next{ 0 };
    std::atomic<int> status{ e == cudaSuccess ? KC_OK : cuda_status(e, "upload staging") };
    std::mutex mu;
    std::string msg;   /* the first worker's error message (messages are per thread) */
    auto fail = [&](int code) {
        std::lock_guard<std::mutex> lk(mu);
        if (status == KC_OK) {
            msg = g_err;
            status = code;
        }
    };
    auto worker = [&](int w) {
        const cudaError_t de = cudaSetDevice(dev);
        if (de != cudaSuccess) {
            fail(cuda_status(de, "upload worker"));
            return;
        }
        int k = 0;
        for (size_t i; status == KC_OK && (i = next++) < jobs.size(); k ^= 1) {
            const UploadJob &J = jobs[i];
            uint8_t *slot_buf = buf[(size_t)(2 * w + k)];
            cudaEvent_t done = ev[(size_t)(2 * w + k)];
            cudaError_t ce = cudaEventSynchronize(done);   /* this slot's previous copy has left */
            if (ce == cudaSuccess && J.fill(slot_buf) != J.bytes) {
                set_error("upload: gathered size mismatch");
                fail(KC_E_IO);
                return;
            }
            if (ce == cudaSuccess) ce = cudaMemcpyAsync(J.dst, slot_buf, J.bytes, cudaMemcpyHostToDevice, st[(size_t)w]);
            if (ce == cudaSuccess) ce = cudaEventRecord(done, st[(size_t)w]);
            if (ce != cudaSuccess) {
                fail(cuda_status(ce, "upload copy"));
                return;
            }
        }
    };
    if (status == KC_OK) {
        std::vector<std::thread> th;
        for (int w = 0; w < W; w++) th.emplace_back(worker, w);
        for (std::thread &t : th) t.join();
    }
    for (int w = 0; w < W; w++)
        if (st[(size_t)w]) {
            const cudaError_t ce = cudaStreamSynchronize(st[(size_t)w]);
            if (ce != cudaSuccess && status == KC_OK) status = cuda_status(ce, "upload copy");
            cudaStreamDestroy(st[(size_t)w]);
        }
    for (int i = 0; i < 2 * W; i++) {
        if (ev[(size_t)i]) cudaEventDestroy(ev[(size_t)i]);
        if (buf[(size_t)i]) cudaFreeHost(buf[(size_t)i]);
    }
    if (status != KC_OK && !msg.empty()) set_error(msg);
    return status;
}

/* CTAs of the step kernel on a device of `sms` SMs: one per SM, at most one
 * per row of x (every CTA owns rows of x, so that each one's reads of a
 * phase's words lie, in the data flow, before the next write of those words). */
static int step_grid(const kc_config &c, int sms) { return std::min(sms, c.dim); }

/* The batched prefill's GEMM operands (unsharded models), packed on the
 * device from the weight stream just uploaded: a table of where each matrix
 * row's record lies in the stream (the walk of fill_stream_part), then one
 * pack launch per matrix; no weight crosses the host link twice. */
static int pack_prefill(kc_model *m, const StreamGeom &g, int G, const std::vector<unsigned long long> &base) {
    const kc_config &c = m->cfg;
    const size_t L = (size_t)c.n_layers, nq = (size_t)c.q_dim + 2 * (size_t)c.kv_dim, nd = (size_t)c.dim;
    const size_t nh = 2 * (size_t)c.hidden_dim, hid = (size_t)c.hidden_dim;
    const size_t oo = L * nq, o13 = oo + L * nd, o2 = o13 + L * nh, ocls = o2 + L * nd, n = ocls + (size_t)g.vocab;
    std::vector<unsigned long long> t(n, 0);
    for (int j = 0; j < G; j++) {
        PhasePlan P[NPHASE];
        make_plan(g, j, G, P);
        const size_t lb = stream_layer_bytes(P);
        for (size_t l = 0; l < L; l++) {
            unsigned long long off = base[(size_t)j] + l * lb;
            for (int k = 0; k < P[PH_A].nseg; k++) {
                const Seg &S = P[PH_A].seg[k];
                for (int r = 0; r < S.rows; r++, off += (unsigned)S.rec) t[l * nq + (size_t)(S.row0 + r)] = off;
            }
            const Seg &C = P[PH_C].seg[0], &D = P[PH_D].seg[0], &E = P[PH_E].seg[0];
            for (int r = 0; r < C.rows; r++, off += (unsigned)C.rec) t[oo + l * nd + (size_t)(C.row0 + r)] = off;
            for (int r = 0; r < D.rows; r++, off += (unsigned)D.rec) {
                t[o13 + l * nh + (size_t)(D.row0 + r)] = off;                       /* gate */
                t[o13 + l * nh + hid + (size_t)(D.row0 + r)] = off + (unsigned)(D.rec / 2);   /* up */
            }
            for (int r = 0; r < E.rows; r++, off += (unsigned)E.rec) t[o2 + l * nd + (size_t)(E.row0 + r)] = off;
        }
        unsigned long long off = base[(size_t)j] + L * lb;
        const Seg &F = P[PH_F].seg[0];
        for (int r = 0; r < F.rows; r++, off += (unsigned)F.rec) t[ocls + (size_t)(F.row0 + r)] = off;
    }
    unsigned long long *d = nullptr;
    cudaStream_t st = nullptr;
    CK(cudaMalloc(&d, sizeof(unsigned long long) * n));
    cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d, t.data(), sizeof(unsigned long long) * n, cudaMemcpyHostToDevice, st);
    int rc = e == cudaSuccess ? KC_OK : cuda_status(e, "prefill row table");
    if (rc == KC_OK) rc = pf_pack_model(m, m->d_stream, PfRowTable{ d, d + oo, d + o13, d + o2, d + ocls, g.d16_q }, st);
    if (st) cudaStreamDestroy(st);
    cudaFree(d);
    return rc;
}

/* The weight stream for a device of G SMs: every CTA's rows of every matrix,
 * contiguous in the order the step kernel consumes them (one upload job per
 * CTA and layer, and one for its classifier rows: gathered from the mapped
 * file into a pinned slot). */
static int upload_stream(kc_model *m, int G) {
    StreamGeom g;
    int st = stream_geom(m, g);
    if (st != KC_OK) return st;
    m->ffn_unit = ffn_unit(m->cfg, g, G);
    g.d_unit = m->ffn_unit;
    std::vector<unsigned long long> base((size_t)G);
    size_t total = 0, maxc = 0;
    for (int j = 0; j < G; j++) {
        PhasePlan P[NPHASE];
        make_plan(g, j, G, P);
        const size_t b = stream_cta_bytes(m, P);
        base[(size_t)j] = total;
        total += align256(b);
        maxc = std::max(maxc, std::max(stream_layer_bytes(P), (size_t)P[PH_F].bytes));
    }
    CK(cudaMalloc(&m->d_stream, total ? total : 256));
    CK(cudaMalloc(&m->d_cta_base, sizeof(unsigned long long) * (size_t)G));
    CK(cudaMemcpy(m->d_cta_base, base.data(), sizeof(unsigned long long) * (size_t)G, cudaMemcpyHostToDevice));
    std::vector<UploadJob> jobs;
    const int L = m->cfg.n_layers;
    for (int j = 0; j < G; j++) {
        PhasePlan P[NPHASE];
        make_plan(g, j, G, P);
        const size_t lb = stream_layer_bytes(P);
        for (int part = 0; part <= L; part++) {
            const size_t b = part < L ? lb : (size_t)P[PH_F].bytes;
            if (b == 0) continue;
            jobs.push_back({ m->d_stream + base[(size_t)j] + (size_t)part * lb, b, [m, g, j, G, part](uint8_t *dst) {
                                 PhasePlan Q[NPHASE];
                                 make_plan(g, j, G, Q);
                                 return fill_stream_part(m, Q, part, dst);
                             } });
        }
    }
    st = upload_jobs(jobs, std::max<size_t>(maxc, 16));
    if (st != KC_OK) return st;
    m->stream_bytes = total;
    m->stream_G = G;
    if (m->tp_world == 1) return pack_prefill(m, g, G, base);
    return KC_OK;
}

extern "C" int kc_model_upload(kc_model *m) {
    clear_error();
    if (m->uploaded) return KC_OK;
    int st = kc_device_check();
    if (st != KC_OK) return st;
    const kc_config &c = m->cfg;
    std::vector<Item> items;
    m->d_layers.assign((size_t)c.n_layers, DevLayer{});
    auto mat = [&](const HostMat &h, DevMat &d) {
        d.rows = h.rows; d.cols = h.cols; d.type = h.type; d.d16 = h.d16;
        items.push_back({ h.q, h.qbytes(), (const void **)&d.q });
        items.push_back({ h.d, h.dbytes(), &d.d });
    };
    auto vec = [&](const float *src, size_t n, const float *&dst) {
        if (src) items.push_back({ src, n * sizeof(float), (const void **)&dst });
    };
    mat(m->tok_emb, m->d_tok_emb);
    for (int l = 0; l < c.n_layers; l++) {
        const HostLayer &H = m->layers[(size_t)l];
        DevLayer &D = m->d_layers[(size_t)l];
        vec(H.attn_norm, (size_t)c.dim, D.attn_norm);
        vec(H.ffn_norm, (size_t)c.dim, D.ffn_norm);
        vec(H.q_norm, (size_t)c.head_dim, D.q_norm); vec(H.k_norm, (size_t)c.head_dim, D.k_norm);
        vec(H.post_attn_norm, (size_t)c.dim, D.post_attn_norm); vec(H.post_ffn_norm, (size_t)c.dim, D.post_ffn_norm);
        D.window = H.window;
        D.local_rope = H.local_rope;
    }
    vec(m->final_norm, (size_t)c.dim, m->d_final_norm);
    size_t total = 0;
    for (const Item &it : items) total += align256(it.bytes);
    uint8_t *base = nullptr;
    CK(cudaMalloc(&base, total ? total : 256));
    /* the file-layout arrays through the pinned pipeline, in pieces of PIECE bytes */
    constexpr size_t PIECE = (size_t)4 << 20;
    std::vector<UploadJob> jobs;
    size_t off = 0;
    for (const Item &it : items) {
        for (size_t o = 0; o < it.bytes; o += PIECE) {
            const size_t n = std::min(PIECE, it.bytes - o);
            const uint8_t *src = (const uint8_t *)it.src + o;
            jobs.push_back({ base + off + o, n, [src, n](uint8_t *dst) {
                                 memcpy(dst, src, n);
                                 return n;
                             } });
        }
        *it.dst = base + off;
        off += align256(it.bytes);
    }
    st = upload_jobs(jobs, PIECE);
    if (st != KC_OK) {
        cudaFree(base);
        return st;
    }
    m->dev_base = base;
    int dev = 0, sms = 0;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    st = upload_stream(m, step_grid(m->cfg, sms));
    if (st != KC_OK) return st;
    m->dev_bytes = total + m->stream_bytes;
    m->uploaded = 1;
    return KC_OK;
}

/* ------------------------------------------------------------------ state */

struct kc_state {
    kc_model *m = nullptr;
    kc_config c{};
    int kv_type = KC_F32;
    cudaStream_t st = nullptr;
    uint8_t *arena = nullptr;
    /* the step kernel's tagged words (tag << 32 | float bits): x after the O
     * and after the down phase [2][dim], the CTAs' sums of squares [2][grid],
     * post-norm block outputs [2][dim], q|k|v, attention partials, attention
     * output, FFN hidden */
    unsigned long long *xw = nullptr, *sspw = nullptr, *yw = nullptr, *qkvw = nullptr, *partw = nullptr;
    unsigned long long *aow = nullptr, *hbw = nullptr, *amaxw = nullptr;
    unsigned tag_next = 1;   /* tag of the next launch's first output (0: the zeroed buffers' tag) */
    float *logits = nullptr;
    uint8_t *kc = nullptr, *vc = nullptr;   /* [L][max_seq][kv_dim] of the KV type */
    float *kd = nullptr, *vd = nullptr;     /* Q8 cache scales [L][max_seq][n_kv_heads] */
    float *rcos = nullptr, *rsin = nullptr, *lcos = nullptr, *lsin = nullptr;
    float *inv0 = nullptr;   /* [vocab]: 1/rms of each embedding row (layer 0's RMSNorm) */
    unsigned *err = nullptr;
    LoopState *ls = nullptr;
    int *feed = nullptr, *out_tokens = nullptr;
    float *h_logits = nullptr;
    LoopState *h_ls = nullptr;
    unsigned *h_err = nullptr;   /* pinned copy of the device error word */
    int num_sms = 148;
    /* the persistent step kernel */
    LayerPlan *d_plan = nullptr;
    unsigned *bar = nullptr;
    unsigned long long *timeline = nullptr;
    unsigned *timeline_n = nullptr;
    StepArgs sa{};
    int step_smem = 0;
    /* prompt tokens per batched prefill step (ml_state.batch); 1: token by token */
    int batch = KC_BATCH_MAX;
    PfScratch *pfs = nullptr;
    /* tensor parallelism: this rank's exchange buffer (IPC-exported), the
     * other ranks' buffers once connected, steps launched so far */
    uint8_t *tp_box = nullptr;
    cudaIpcMemHandle_t tp_handle{};
    uint8_t *tp_peer[KC_TP_MAX] = {};
    int tp_connected = 0;
    unsigned long long tp_steps = 0;
    /* the logits ring row of the last call's last token (kc_sample); -1: none */
    int last_row = -1;
};

/* RoPE inverse frequency of pair i (model/transformer.c:16-38; the scaling
 * formulas of transformers: linear, yarn, llama3), in double. */
static double rope_inv_freq(const kc_config &c, int i) {
    const double inv = std::pow((double)c.rope_theta, -2.0 * i / c.head_dim);
    if (c.rope_type == KC_ROPE_LINEAR) return inv / c.rope_factor;
    if (c.rope_type == KC_ROPE_YARN) {
        const double hd = c.head_dim, orig = c.rope_orig_max_seq, lb = 2.0 * std::log((double)c.rope_theta);
        const double pi2 = 2.0 * 3.14159265358979323846;
        double lo = std::floor(hd * std::log(orig / ((double)c.rope_low_freq_factor * pi2)) / lb);
        double hi = std::ceil(hd * std::log(orig / ((double)c.rope_high_freq_factor * pi2)) / lb);
        if (lo < 0.0) lo = 0.0;
        if (hi > hd - 1.0) hi = hd - 1.0;
        if (lo == hi) hi += 0.001;
        double ramp = (i - lo) / (hi - lo);
        ramp = ramp < 0.0 ? 0.0 : (ramp > 1.0 ? 1.0 : ramp);
        return inv / c.rope_factor * ramp + inv * (1.0 - ramp);
    }
    if (c.rope_type != KC_ROPE_LLAMA3) return inv;
    const double f = c.rope_factor, lo = c.rope_low_freq_factor, hi = c.rope_high_freq_factor;
    const double orig = c.rope_orig_max_seq, wavelen = 2.0 * 3.14159265358979323846 / inv;
    if (wavelen < orig / hi) return inv;
    if (wavelen > orig / lo) return inv / f;
    const double smooth = (orig / wavelen - lo) / (hi - lo);
    return (1.0 - smooth) * inv / f + smooth * inv;
}

/* Bytes per cache element of a KV type. */
static size_t kv_elem_bytes(int kv_type) { return kv_type == KC_F32 ? 4 : (kv_type == KC_F16 ? 2 : 1); }

static const int KC_MAX_SMEM = 227 * 1024;
constexpr int KC_MAX_DEVICES = 64;

/* The calling thread's current device, checked against the per-device tables. */
static int current_device(int &dev) {
    CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= KC_MAX_DEVICES) {
        set_error("device index " + std::to_string(dev) + " beyond this library's table of " +
                  std::to_string(KC_MAX_DEVICES));
        return KC_E_SHAPE;
    }
    return KC_OK;
}

/* Opt-in to the full shared memory of an sm_100 CTA, once per device (the
 * attribute belongs to the current device; outside any stream capture). */
static int set_smem_attributes() {
    static bool done[KC_MAX_DEVICES];
    int dev = 0;
    const int rc = current_device(dev);
    if (rc != KC_OK) return rc;
    if (done[dev]) return KC_OK;
    const void *fns[] = { (const void *)step_kernel<KC_F32, true>,  (const void *)step_kernel<KC_F16, true>,
                          (const void *)step_kernel<KC_Q8_0, true>, (const void *)step_kernel<KC_F32, false>,
                          (const void *)step_kernel<KC_F16, false>, (const void *)step_kernel<KC_Q8_0, false>,
                          (const void *)matvec_kernel, (const void *)activation_kernel };
    for (const void *f : fns) {
        cudaFuncAttributes fa;
        CK(cudaFuncGetAttributes(&fa, f));
        CK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, KC_MAX_SMEM - (int)fa.sharedSizeBytes));
    }
    done[dev] = true;
    return KC_OK;
}

/* The kernel-level matvec's error word: one per device (a __device__ variable
 * lives in every device's copy of this module), sticky until kc_dev_sync
 * reports it. Its address on each device, looked up on first use. */
static __device__ unsigned g_kl_err;
static unsigned *g_kl_err_ptr[KC_MAX_DEVICES];
/* Polls of the kernel-level consumers' first wait on a chunk (kc_debug_wait_limit). */
static unsigned g_wait_limit = WAIT_POLLS;

static int kl_err_word(int dev, unsigned *&w) {
    if (!g_kl_err_ptr[dev]) {
        void *p = nullptr;
        CK(cudaGetSymbolAddress(&p, g_kl_err));
        g_kl_err_ptr[dev] = (unsigned *)p;
    }
    w = g_kl_err_ptr[dev];
    return KC_OK;
}

/* Ring depth that fits beside the fixed part of a streaming CTA's shared memory. */
/* Words of the grid barrier's arrival counter line; the attention counters follow. */
constexpr int ATT_UNITS_MAX = 64;   /* attention unit counters after the step-end barrier's words */
constexpr size_t BAR_WORDS = 32 + (size_t)ATT_CNT_STRIDE * ATT_UNITS_MAX;

static int ring_stages(int slot, int act_bytes, int static_bytes, int res_bytes = 0, int wbuf_bytes = 0) {
    int nst = 16;
    while (nst >= 2 && smem_fixed_bytes(nst, act_bytes, res_bytes, wbuf_bytes) + nst * slot > KC_MAX_SMEM - static_bytes)
        nst--;
    return nst;
}

/* 1/rms of every embedding row, the first layer's RMSNorm factor, computed as
 * the reference computes it: x = dequant(row) (core/quant_ref.c:4-19) times
 * embed_scale (model/transformer.c:226-230), ss += x*x in order, inv = 1 /
 * sqrtf(ss / n + eps) (kernels/scalar/k_scalar.c:59-64), in float with every
 * operation rounded on its own (this file is compiled without contraction).
 * Embedding rows are quantized: with unit norm weights their normalized values
 * sit on exact quantization ties, which only this order resolves as the
 * reference does. */
static void embed_inv_table(const kc_model *m, std::vector<float> &out) {
    const kc_config &c = m->cfg;
    const HostMat &E = m->tok_emb;
    const int dim = c.dim, nb = dim / QK;
    out.assign((size_t)c.vocab, 0.0f);
    auto scale = [&](size_t i) -> float {
        return E.d16 ? half_to_float(((const uint16_t *)E.d)[i]) : ((const float *)E.d)[i];
    };
    auto work = [&](int t0, int t1) {
        std::vector<float> x((size_t)dim);
        for (int t = t0; t < t1; t++) {
            for (int b = 0; b < nb; b++) {
                const float d = scale((size_t)t * nb + b);
                for (int j = 0; j < QK; j++) {
                    int v;
                    if (E.type == KC_Q8_0) {
                        v = ((const int8_t *)E.q)[(size_t)t * dim + (size_t)b * QK + j];
                    } else {
                        const uint8_t byte = ((const uint8_t *)E.q)[((size_t)t * nb + b) * (QK / 2) + (j & 15)];
                        v = (j < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
                    }
                    volatile float xv = (float)v * d;
                    float xf = xv;
                    if (c.embed_scale != 1.0f) { volatile float t2 = xf * c.embed_scale; xf = t2; }
                    x[(size_t)b * QK + j] = xf;
                }
            }
            float ss = 0.0f;
            for (int i = 0; i < dim; i++) {
                volatile float sq = x[(size_t)i] * x[(size_t)i];
                ss = ss + sq;
            }
            volatile float mean = ss / (float)dim;
            volatile float arg = mean + c.norm_eps;
            volatile float root = std::sqrt((float)arg);
            out[(size_t)t] = 1.0f / root;
        }
    };
    unsigned nt = std::thread::hardware_concurrency();
    if (nt < 1) nt = 1;
    if (nt > 64) nt = 64;
    std::vector<std::thread> th;
    for (unsigned i = 0; i < nt; i++)
        th.emplace_back(work, (int)((long long)c.vocab * i / nt), (int)((long long)c.vocab * (i + 1) / nt));
    for (auto &t : th) t.join();
}

static PMat pmat(const DevMat &m) { return PMat{ m.q, m.d, m.rows, m.type, m.d16 }; }

/* The step kernel's instance for a KV cache type and the stream's scale type. */
typedef void (*StepFn)(StepArgs);
static StepFn step_fn(int kv_type, int d16) {
    if (d16) return kv_type == KC_F16 ? step_kernel<KC_F16, true> : (kv_type == KC_Q8_0 ? step_kernel<KC_Q8_0, true> : step_kernel<KC_F32, true>);
    return kv_type == KC_F16 ? step_kernel<KC_F16, false> : (kv_type == KC_Q8_0 ? step_kernel<KC_Q8_0, false> : step_kernel<KC_F32, false>);
}

/* The persistent step kernel's plan: per-layer pointers in device memory, the
 * ring geometry from the shared-memory budget, the attention split. */
static int setup_step_kernel(kc_state *s) {
    const kc_config &c = s->c;
    kc_model *m = s->m;
    const int G = s->num_sms;
    if (m->stream_G != G) {
        set_error("the model was uploaded for a device with another SM count");
        return KC_E_SHAPE;
    }
    if ((c.dim + G - 1) / G > OWN_MAX) {
        set_error("dim too large for the rows of x a CTA keeps in shared memory");
        return KC_E_SHAPE;
    }
    StreamGeom g;
    int st = stream_geom(m, g);
    if (st != KC_OK) return st;
    std::vector<LayerPlan> plan((size_t)c.n_layers);
    const size_t lkv = (size_t)c.max_seq * c.kv_dim * kv_elem_bytes(s->kv_type);
    const size_t lkd = (size_t)c.max_seq * c.n_kv_heads;
    for (int l = 0; l < c.n_layers; l++) {
        const DevLayer &L = m->d_layers[(size_t)l];
        LayerPlan &P = plan[(size_t)l];
        P.attn_norm = L.attn_norm; P.ffn_norm = L.ffn_norm;
        P.kc = s->kc + (size_t)l * lkv; P.vc = s->vc + (size_t)l * lkv;
        P.kd = s->kd ? s->kd + (size_t)l * lkd : nullptr; P.vd = s->vd ? s->vd + (size_t)l * lkd : nullptr;
        P.rcos = L.local_rope ? s->lcos : s->rcos; P.rsin = L.local_rope ? s->lsin : s->rsin;
        P.window = L.window;
        P.q_norm = L.q_norm; P.k_norm = L.k_norm;
        P.post_attn = L.post_attn_norm; P.post_ffn = L.post_ffn_norm;
    }
    int res = 0;
    for (int j = 0; j < G; j++) {
        PhasePlan P[NPHASE];
        make_plan(g, j, G, P);
        for (int p = 0; p < NPHASE; p++)
            res = std::max(res, plan_rows(P[p]) * (p == PH_D ? 8 : 4 * col_slices(P[p].cols / QK, false)));
    }
    res = (res + 15) & ~15;
    /* the ring slot for bulk copies of up to `chunk` bytes: the largest chunk of any CTA's plan */
    auto plan_slot = [&](int chunk) {
        StreamGeom gc = g;
        gc.chunk = chunk;
        int sl = 0;
        for (int j = 0; j < G; j++) {
            PhasePlan P[NPHASE];
            make_plan(gc, j, G, P);
            sl = std::max(sl, plan_max_chunk(P));
        }
        return (sl + 127) & ~127;
    };
    CK(cudaMalloc(&s->d_plan, sizeof(LayerPlan) * plan.size()));
    CK(cudaMemcpy(s->d_plan, plan.data(), sizeof(LayerPlan) * plan.size(), cudaMemcpyHostToDevice));
    const int group = c.n_heads / c.n_kv_heads;
    const int att_bytes = (int)sizeof(float) * attention_scratch_floats(group, c.head_dim);
    /* attention units: the fewest KV heads whose outputs fill whole 32-value blocks */
    const int att_unit = QK / std::gcd(group * c.head_dim, QK);
    if (c.n_kv_heads % att_unit || c.n_kv_heads / att_unit > ATT_UNITS_MAX ||
        att_unit * group * (MAX_NSPLIT + c.head_dim) > attention_scratch_floats(group, c.head_dim)) {
        set_error("attention head layout outside the step kernel's combine limits");
        return KC_E_SHAPE;
    }
    int act = 0;
    for (int cols : { c.dim, c.q_dim, c.hidden_dim }) act = std::max(act, cols + 8 * (cols / QK));
    act = (std::max(act, att_bytes) + 15) & ~15;
    if (c.dim > 4 * 2048 || c.q_dim > 8 * 2048 || c.hidden_dim > 8 * 2048) {
        set_error("activation wider than the step kernel's prologue (dim 8192, q_dim and hidden 16384)");
        return KC_E_SHAPE;
    }
    cudaFuncAttributes fa;
    CK(cudaFuncGetAttributes(&fa, (const void *)step_fn(s->kv_type, g.d16_q)));
    const int wbuf = 4 * c.dim;
    /* the largest chunk (56 KB down to 32 KB) that leaves three ring slots beside
     * the attention scratch, else the largest that leaves two */
    int slot = 0, nst = 0;
    for (int pass = 0; pass < 2 && nst == 0; pass++)
        for (int kb = CHUNK_BYTES / 1024; kb >= 32; kb -= 4) {
            const int sl = plan_slot(kb * 1024), n = ring_stages(sl, act, (int)fa.sharedSizeBytes, res, wbuf);
            if (n >= (pass == 0 ? 3 : 2)) {
                g.chunk = kb * 1024;
                slot = sl;
                nst = n;
                break;
            }
        }
    if (nst < 2) {
        set_error("layer shapes leave no room for the weight ring in shared memory");
        return KC_E_SHAPE;
    }
    s->step_smem = smem_fixed_bytes(nst, act, res, wbuf) + nst * slot;
    int per_sm = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_fn(s->kv_type, g.d16_q), STEP_THREADS, s->step_smem));
    if (per_sm < 1) {
        set_error("the step kernel does not fit on an SM");
        return KC_E_SHAPE;
    }
    StepArgs &a = s->sa;
    a.layers = s->d_plan;
    a.emb = pmat(m->d_tok_emb);
    a.stream = m->d_stream;
    a.cta_base = m->d_cta_base;
    a.geom = g;
    a.final_norm = m->d_final_norm;
    a.inv0 = s->inv0;
    a.xw = s->xw; a.sspw = s->sspw; a.yw = s->yw; a.qkvw = s->qkvw; a.partw = s->partw; a.aow = s->aow;
    a.hbw = s->hbw; a.logits = s->logits;
    a.bar = s->bar; a.err = s->err; a.ls = s->ls; a.feed = s->feed;
    a.attc = s->bar + 32;
    a.amaxw = s->amaxw;
    a.att_unit = att_unit;
    a.out_tokens = s->out_tokens;
    a.kv_type = s->kv_type;
    a.n_layers = c.n_layers; a.dim = c.dim; a.q_dim = c.q_dim; a.kv_dim = c.kv_dim; a.hidden = c.hidden_dim;
    a.vocab = c.vocab; a.max_seq = c.max_seq; a.n_heads = c.n_heads; a.n_kv_heads = c.n_kv_heads; a.hd = c.head_dim;
    a.eps = c.norm_eps; a.attn_scale = c.attn_scale; a.attn_softcap = c.attn_softcap; a.final_softcap = c.final_softcap;
    a.embed_scale = c.embed_scale; a.act = c.act;
    a.cls_row0 = m->cls_row0;
    a.post_norms = c.post_norms ? 1 : 0;
    a.tp_rank = 0; a.tp_world = 1; a.tp_step0 = 0;
    for (int r = 0; r < KC_TP_MAX; r++) a.tp_box[r] = nullptr;
    a.nsplit = std::min(MAX_NSPLIT, std::max(1, s->num_sms / c.n_kv_heads));
    a.nstage = nst; a.slot_bytes = slot; a.act_bytes = act; a.res_bytes = res; a.wbuf_bytes = wbuf;
    a.timeline = nullptr; a.timeline_n = s->timeline_n; a.timeline_cap = 4096;
    return KC_OK;
}

/* Runs nsteps token steps in one cooperative launch of the step kernel. */
static int launch_steps(kc_state *s, int nsteps, int logits, bool timeline = false) {
    if (s->m->tp_world > 1 && !s->tp_connected) {
        set_error("tensor-parallel state not connected (kc_tp_connect)");
        return KC_E_SHAPE;
    }
    s->last_row = -1;   /* the caller names the row when its last token's logits are kept */
    CK(cudaMemsetAsync(s->bar, 0, sizeof(unsigned) * BAR_WORDS, s->st));
    StepArgs a = s->sa;
    /* this launch's tags: NTAG per layer and step, after the last launch's */
    a.tag0 = s->tag_next;
    s->tag_next += (unsigned)((unsigned long long)nsteps * s->c.n_layers * NTAG);
    a.tp_step0 = s->tp_steps;
    s->tp_steps += (unsigned long long)nsteps;
    a.nsteps = nsteps;
    a.run_cls = logits;
    if (timeline) {
        a.timeline = s->timeline;
        CK(cudaMemsetAsync(s->timeline_n, 0, sizeof(unsigned), s->st));
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)s->num_sms);
    cfg.blockDim = dim3(STEP_THREADS);
    cfg.dynamicSmemBytes = (size_t)s->step_smem;
    cfg.stream = s->st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CK(cudaLaunchKernelEx(&cfg, step_fn(s->kv_type, a.geom.d16_q), a));
    return KC_OK;
}

static int run_steps(kc_state *s, int nsteps, int logits) { return launch_steps(s, nsteps, logits); }

/* A sharded state's exchange buffer (one allocation, exported by CUDA IPC):
 * partial rows y [2][world][dim] as 64-bit words (sequence number | float),
 * best keys [world] and their flags [world], the logits ring
 * [LOGITS_RING][vocab] (every rank's classifier rows land in every rank's
 * ring). Zeroed: sequence numbers start at 1. */
static int tp_alloc(kc_state *s) {
    const kc_config &c = s->c;
    kc_model *m = s->m;
    const size_t W = (size_t)m->tp_world;
    const size_t off_best = align256(sizeof(unsigned long long) * 2 * W * c.dim);
    const size_t off_bflag = off_best + align256(sizeof(unsigned long long) * W);
    const size_t off_logits = off_bflag + align256(sizeof(unsigned) * W);
    const size_t total = off_logits + align256(sizeof(float) * (size_t)LOGITS_RING * c.vocab);
    CK(cudaMalloc(&s->tp_box, total));
    CK(cudaMemset(s->tp_box, 0, total));
    CK(cudaIpcGetMemHandle(&s->tp_handle, s->tp_box));
    s->logits = (float *)(s->tp_box + off_logits);
    StepArgs &a = s->sa;
    a.logits = s->logits;
    a.tp_rank = m->tp_rank;
    a.tp_world = m->tp_world;
    a.tp_off_best = off_best;
    a.tp_off_bflag = off_bflag;
    a.tp_off_logits = off_logits;
    return KC_OK;
}

extern "C" void kc_state_free(kc_state *s) {
    if (!s) return;
    if (s->st) cudaStreamSynchronize(s->st);
    if (s->arena) cudaFree(s->arena);
    if (s->h_logits) cudaFreeHost(s->h_logits);
    if (s->h_ls) cudaFreeHost(s->h_ls);
    if (s->h_err) cudaFreeHost(s->h_err);
    if (s->d_plan) cudaFree(s->d_plan);
    for (int r = 0; r < KC_TP_MAX; r++)
        if (s->tp_peer[r]) cudaIpcCloseMemHandle(s->tp_peer[r]);
    if (s->tp_box) cudaFree(s->tp_box);
    pf_free_scratch(s->pfs);
    if (s->st) cudaStreamDestroy(s->st);
    delete s;
}

extern "C" int kc_state_init(kc_state **out, kc_model *m, int nthreads, int kv_type) {
    (void)nthreads;
    *out = nullptr;
    clear_error();
    if (kv_type != KC_F32 && kv_type != KC_F16 && kv_type != KC_Q8_0) return KC_E_SHAPE;
    const kc_config &c = m->cfg;
    if (c.post_norms && m->tp_world > 1) {
        set_error("post-norm models do not run tensor parallel");
        return KC_E_SHAPE;
    }
    const int group = c.n_heads / c.n_kv_heads;
    const int es = (int)kv_elem_bytes(kv_type);
    if (group * c.head_dim > ATT_MAX_OUT || (c.head_dim * es) % 16 || c.head_dim % 16 ||
        (kv_type != KC_F32 && c.head_dim > 128) || group > NCW) {
        set_error("attention head layout outside this build's kernel limits");
        return KC_E_SHAPE;
    }
    int st = kc_model_upload(m);
    if (st != KC_OK) return st;
    kc_state *s = new (std::nothrow) kc_state();
    if (!s) return KC_E_NOMEM;
    s->m = m;
    s->c = c;
    s->kv_type = kv_type;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&s->num_sms, cudaDevAttrMultiProcessorCount, dev);
    s->num_sms = step_grid(c, s->num_sms);
    auto fail = [&](int code) { kc_state_free(s); return code; };
    cudaError_t e = cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking);
    if (e != cudaSuccess) return fail(cuda_status(e, "stream"));

    const size_t T = (size_t)c.max_seq, h2 = (size_t)c.head_dim / 2;
    const size_t lkv = (size_t)c.n_layers * T * c.kv_dim * kv_elem_bytes(kv_type);
    struct Buf { void **p; size_t bytes; };
    std::vector<Buf> bufs = {
        { (void **)&s->xw, sizeof(unsigned long long) * 2 * c.dim },
        { (void **)&s->yw, sizeof(unsigned long long) * 2 * c.dim },
        { (void **)&s->sspw, sizeof(unsigned long long) * 2 * (size_t)s->num_sms },
        { (void **)&s->qkvw, sizeof(unsigned long long) * (size_t)(c.q_dim + 2 * c.kv_dim) },
        /* quantized vectors: n / 4 quant words, then n / 32 scale words */
        { (void **)&s->aow, sizeof(unsigned long long) * (size_t)(c.q_dim / 4 + c.q_dim / QK) },
        { (void **)&s->hbw, sizeof(unsigned long long) * (size_t)(c.hidden_dim / 4 + c.hidden_dim / QK) },
        /* split FFN blocks: the covering CTAs' partial maxima [hidden / 32][8] */
        { (void **)&s->amaxw, sizeof(unsigned long long) * (size_t)(c.hidden_dim / QK) * 8 },
        { (void **)&s->partw, sizeof(unsigned long long) * (size_t)c.n_heads * MAX_NSPLIT * (c.head_dim + 2) },
        { (void **)&s->logits, sizeof(float) * (size_t)LOGITS_RING * c.vocab },
        { (void **)&s->err, sizeof(unsigned) * 4 },
        /* the step-end barrier's arrival counter, zeroed before each launch */
        { (void **)&s->bar, sizeof(unsigned) * BAR_WORDS },
        { (void **)&s->timeline_n, sizeof(unsigned) * 4 },
        { (void **)&s->timeline, sizeof(unsigned long long) * 4096 },
        { (void **)&s->ls, sizeof(LoopState) },
        { (void **)&s->feed, sizeof(int) * (T + 1) },
        { (void **)&s->out_tokens, sizeof(int) * (T + 1) },
        { (void **)&s->kc, lkv },
        { (void **)&s->vc, lkv },
        { (void **)&s->rcos, sizeof(float) * T * h2 },
        { (void **)&s->inv0, sizeof(float) * (size_t)c.vocab },
        { (void **)&s->rsin, sizeof(float) * T * h2 },
    };
    if (kv_type == KC_Q8_0) {
        bufs.push_back({ (void **)&s->kd, sizeof(float) * (size_t)c.n_layers * T * c.n_kv_heads });
        bufs.push_back({ (void **)&s->vd, sizeof(float) * (size_t)c.n_layers * T * c.n_kv_heads });
    }
    if (c.rope_local_theta > 0.0f) {
        bufs.push_back({ (void **)&s->lcos, sizeof(float) * T * h2 });
        bufs.push_back({ (void **)&s->lsin, sizeof(float) * T * h2 });
    }
    size_t total = 0;
    for (const Buf &b : bufs) total += align256(b.bytes);
    e = cudaMalloc(&s->arena, total);
    if (e != cudaSuccess) return fail(cuda_status(e, "state arena"));
    size_t off = 0;
    for (const Buf &b : bufs) {
        *b.p = s->arena + off;
        off += align256(b.bytes);
    }
    /* zero the arena and wait: the tables below are copied on the legacy
     * stream, which does not order against this non-blocking stream */
    e = cudaMemsetAsync(s->arena, 0, total, s->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->st);
    if (e != cudaSuccess) return fail(cuda_status(e, "memset"));
    e = cudaMallocHost(&s->h_logits, sizeof(float) * c.vocab);
    if (e == cudaSuccess) e = cudaMallocHost(&s->h_ls, sizeof(LoopState));
    if (e == cudaSuccess) e = cudaMallocHost(&s->h_err, sizeof(unsigned));
    if (e != cudaSuccess) return fail(cuda_status(e, "pinned host buffers"));

    /* RoPE tables: double, stored as float (model/transformer.c:146-162) */
    {
        std::vector<float> cs(T * h2), sn(T * h2), lc, ls_;
        const double af = c.rope_type == KC_ROPE_YARN ? c.rope_attn_factor : 1.0;
        if (s->lcos) { lc.resize(T * h2); ls_.resize(T * h2); }
        for (size_t i = 0; i < h2; i++) {
            const double freq = rope_inv_freq(c, (int)i);
            const double lfreq = s->lcos ? std::pow((double)c.rope_local_theta, -2.0 * (double)i / c.head_dim) : 0.0;
            for (size_t p = 0; p < T; p++) {
                const double ang = (double)p * freq;
                cs[p * h2 + i] = (float)(std::cos(ang) * af);
                sn[p * h2 + i] = (float)(std::sin(ang) * af);
                if (s->lcos) {
                    lc[p * h2 + i] = (float)std::cos((double)p * lfreq);
                    ls_[p * h2 + i] = (float)std::sin((double)p * lfreq);
                }
            }
        }
        e = cudaMemcpy(s->rcos, cs.data(), sizeof(float) * T * h2, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(s->rsin, sn.data(), sizeof(float) * T * h2, cudaMemcpyHostToDevice);
        if (e == cudaSuccess && s->lcos) e = cudaMemcpy(s->lcos, lc.data(), sizeof(float) * T * h2, cudaMemcpyHostToDevice);
        if (e == cudaSuccess && s->lsin) e = cudaMemcpy(s->lsin, ls_.data(), sizeof(float) * T * h2, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return fail(cuda_status(e, "rope tables"));
        std::vector<float> inv0;
        embed_inv_table(m, inv0);
        e = cudaMemcpy(s->inv0, inv0.data(), sizeof(float) * c.vocab, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return fail(cuda_status(e, "embedding norms"));
    }
    st = set_smem_attributes();
    if (st != KC_OK) return fail(st);
    st = setup_step_kernel(s);
    if (st != KC_OK) return fail(st);
    if (m->tp_world > 1) {
        st = tp_alloc(s);
        if (st != KC_OK) return fail(st);
    }
    e = cudaStreamSynchronize(s->st);
    if (e != cudaSuccess) return fail(cuda_status(e, "state init"));
    *out = s;
    return KC_OK;
}

extern "C" int kc_tp_handle(kc_state *s, void *out, size_t cap) {
    clear_error();
    if (!s->tp_box || cap < KC_TP_HANDLE_BYTES || sizeof(cudaIpcMemHandle_t) > KC_TP_HANDLE_BYTES) return KC_E_SHAPE;
    std::memset(out, 0, KC_TP_HANDLE_BYTES);
    std::memcpy(out, &s->tp_handle, sizeof(cudaIpcMemHandle_t));
    return KC_OK;
}

extern "C" int kc_tp_connect(kc_state *s, const void *handles) {
    clear_error();
    kc_model *m = s->m;
    if (!s->tp_box || s->tp_connected) return KC_E_SHAPE;
    const uint8_t *h = (const uint8_t *)handles;
    for (int r = 0; r < m->tp_world; r++) {
        if (r == m->tp_rank) {
            s->sa.tp_box[r] = s->tp_box;
            continue;
        }
        cudaIpcMemHandle_t ih;
        std::memcpy(&ih, h + (size_t)r * KC_TP_HANDLE_BYTES, sizeof ih);
        void *p = nullptr;
        CK(cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess));
        s->tp_peer[r] = (uint8_t *)p;
        s->sa.tp_box[r] = (uint8_t *)p;
    }
    s->tp_connected = 1;
    return KC_OK;
}

static int set_loop(kc_state *s, int token, int pos, int feed_mode) {
    LoopState *h = s->h_ls;
    std::memset(h, 0, sizeof *h);
    h->token = token;
    h->pos = pos;
    h->feed_mode = feed_mode;
    CK(cudaMemcpyAsync(s->ls, h, sizeof *h, cudaMemcpyHostToDevice, s->st));
    return KC_OK;
}

static int finish(kc_state *s) {
    /* both words into pinned memory: the copies stay asynchronous, one wait */
    CK(cudaMemcpyAsync(s->h_ls, s->ls, sizeof(LoopState), cudaMemcpyDeviceToHost, s->st));
    CK(cudaMemcpyAsync(s->h_err, s->err, sizeof(unsigned), cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    const unsigned err = *s->h_err;
    if (s->h_ls->err) {
        set_error("a kernel saw a token or position out of range");
        return KC_E_SHAPE;
    }
    if (err) {
        set_error("a device wait gave up (error word " + std::to_string(err) + ")");
        return KC_E_IO;
    }
    return KC_OK;
}

extern "C" float *kc_forward(kc_state *s, int token, int pos) {
    clear_error();
    const kc_config &c = s->c;
    if (pos < 0 || pos >= c.max_seq || token < 0 || token >= c.vocab) return nullptr;
    s->last_row = -1;
    if (set_loop(s, token, pos, 0) != KC_OK) return nullptr;
    if (run_steps(s, 1, 1) != KC_OK) return nullptr;
    s->last_row = 0;
    cudaError_t e = cudaMemcpyAsync(s->h_logits, s->logits, sizeof(float) * c.vocab, cudaMemcpyDeviceToHost, s->st);
    if (e != cudaSuccess) { cuda_status(e, "logits copy"); return nullptr; }
    if (finish(s) != KC_OK) return nullptr;
    return s->h_logits;
}

/* ml_prefill through the step kernel, one token per step: the logits of
 * token-by-token decoding bit for bit (ml_state.batch == 1). */
static int prefill_tokenwise(kc_state *s, const int *tokens, int n, int pos0, float *logits) {
    const kc_config &c = s->c;
    CK(cudaMemcpyAsync(s->feed, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemsetAsync(s->feed + n, 0, sizeof(int), s->st));
    int st = set_loop(s, tokens[0], pos0, 1);
    if (st != KC_OK) return st;
    for (int i0 = 0; i0 < n; i0 += LOGITS_RING) {
        const int k = n - i0 < LOGITS_RING ? n - i0 : LOGITS_RING;
        st = run_steps(s, k, logits ? 1 : 0);
        if (st != KC_OK) return st;
        if (logits)
            CK(cudaMemcpyAsync(logits + (size_t)i0 * c.vocab, s->logits, sizeof(float) * (size_t)k * c.vocab,
                               cudaMemcpyDeviceToHost, s->st));
    }
    if (logits) s->last_row = (n - 1) % LOGITS_RING;
    return finish(s);
}

/* ml_prefill in chunks of up to s->batch tokens through the batched path
 * (tensor-core GEMMs, kc_prefill.cu). */
static int prefill_batched(kc_state *s, const int *tokens, int n, int pos0, float *logits) {
    const kc_config &c = s->c;
    s->last_row = -1;
    kc_model *m = s->m;
    std::vector<PfLayerRun> L((size_t)c.n_layers);
    const size_t lkv = (size_t)c.max_seq * c.kv_dim * kv_elem_bytes(s->kv_type);
    const size_t lkd = (size_t)c.max_seq * c.n_kv_heads;
    for (int l = 0; l < c.n_layers; l++) {
        const DevLayer &D = m->d_layers[(size_t)l];
        PfLayerRun &P = L[(size_t)l];
        P.attn_norm = D.attn_norm;
        P.ffn_norm = D.ffn_norm;
        P.kc = s->kc + (size_t)l * lkv;
        P.vc = s->vc + (size_t)l * lkv;
        P.kd = s->kd ? s->kd + (size_t)l * lkd : nullptr;
        P.vd = s->vd ? s->vd + (size_t)l * lkd : nullptr;
        P.rcos = D.local_rope ? s->lcos : s->rcos;
        P.rsin = D.local_rope ? s->lsin : s->rsin;
        P.window = D.window;
        P.q_norm = D.q_norm;
        P.k_norm = D.k_norm;
        P.post_attn = D.post_attn_norm;
        P.post_ffn = D.post_ffn_norm;
    }
    PfRun r;
    r.m = m;
    r.kv_type = s->kv_type;
    r.layers = L.data();
    r.emb_q = m->d_tok_emb.q;
    r.emb_d = m->d_tok_emb.d;
    r.emb_type = m->d_tok_emb.type;
    r.emb_d16 = m->d_tok_emb.d16;
    r.final_norm = m->d_final_norm;
    r.logits_dev = s->logits;
    r.logits_rows = LOGITS_RING;
    r.err = s->err + 1;
    r.st = s->st;
    r.scratch = &s->pfs;
    r.batch = s->batch;
    return pf_prefill(r, tokens, n, pos0, logits);
}

extern "C" int kc_prefill(kc_state *s, const int *tokens, int n, int pos0, float *logits) {
    clear_error();
    const kc_config &c = s->c;
    if (n < 0 || pos0 < 0 || pos0 + n > c.max_seq) return KC_E_SHAPE;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= c.vocab) return KC_E_SHAPE;
    if (n == 0) return KC_OK;
    if (s->batch > 1 && n > 1 && s->m->tp_world == 1 && pf_fits(c, s->kv_type, pos0 + n - 1))
        return prefill_batched(s, tokens, n, pos0, logits);
    return prefill_tokenwise(s, tokens, n, pos0, logits);
}

extern "C" int kc_set_batch(kc_state *s, int batch) {
    clear_error();
    if (batch < 1 || batch > KC_BATCH_MAX) {
        set_error("batch must be 1.." + std::to_string(KC_BATCH_MAX));
        return KC_E_SHAPE;
    }
    s->batch = batch;
    return KC_OK;
}

extern "C" int kc_generate_greedy(kc_state *s, int token, int pos, int n, int *out_tokens) {
    clear_error();
    const kc_config &c = s->c;
    if (n < 0 || pos < 0 || pos + n > c.max_seq || token < 0 || token >= c.vocab) return KC_E_SHAPE;
    if (n == 0) return KC_OK;
    int st = set_loop(s, token, pos, 0);
    if (st != KC_OK) return st;
    for (int i = 0; i < n; i += 256) {
        st = run_steps(s, n - i < 256 ? n - i : 256, 1);
        if (st != KC_OK) return st;
    }
    s->last_row = (n - 1) % LOGITS_RING;
    CK(cudaMemcpyAsync(out_tokens, s->out_tokens, sizeof(int) * n, cudaMemcpyDeviceToHost, s->st));
    return finish(s);
}

extern "C" int kc_time_decode(kc_state *s, int token, int pos, int warmup, int steps, float *ms) {
    clear_error();
    const kc_config &c = s->c;
    if (pos < 0 || pos + warmup + steps > c.max_seq || token < 0 || token >= c.vocab || steps < 1) return KC_E_SHAPE;
    int st = set_loop(s, token, pos, 0);
    if (st != KC_OK) return st;
    if (warmup > 0) {
        st = run_steps(s, warmup, 1);
        if (st != KC_OK) return st;
    }
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    cudaEventRecord(e0, s->st);
    st = run_steps(s, steps, 1);
    cudaEventRecord(e1, s->st);
    if (st != KC_OK) return st;
    cudaError_t e = cudaEventSynchronize(e1);
    float t = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (e != cudaSuccess) return cuda_status(e, "decode timing");
    *ms = t;
    return finish(s);
}

extern "C" int kc_debug_copy(kc_state *s, int which, void *dst, size_t bytes) {
    const kc_config &c = s->c;
    const void *src = nullptr;
    size_t n = 0;
    const unsigned long long *words = nullptr;   /* tagged words: the floats are their low halves */
    switch (which) {
    case 0: words = s->xw + c.dim; n = (size_t)c.dim; break;
    case 1: words = s->qkvw; n = (size_t)(c.q_dim + 2 * c.kv_dim); break;
    case 2: case 3: {
        /* quantized words: the dequantized values q * d */
        n = (size_t)(which == 2 ? c.q_dim : c.hidden_dim);
        if (bytes < n * sizeof(float)) return KC_E_SHAPE;
        CK(cudaStreamSynchronize(s->st));
        const size_t nw = n / 4 + n / QK;
        std::vector<unsigned long long> h(nw);
        CK(cudaMemcpy(h.data(), which == 2 ? s->aow : s->hbw, nw * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < n; i++) {
            const unsigned qw = (unsigned)h[i / 4], dw = (unsigned)h[n / 4 + i / QK];
            float d;
            std::memcpy(&d, &dw, sizeof d);
            const float v = (float)(int8_t)(qw >> (8 * (i % 4))) * d;
            std::memcpy((char *)dst + i * sizeof(float), &v, sizeof(float));
        }
        return KC_OK;
    }
    case 4: src = s->kc; n = kv_elem_bytes(s->kv_type) * (size_t)c.n_layers * c.max_seq * c.kv_dim; break;
    case 5: src = s->vc; n = kv_elem_bytes(s->kv_type) * (size_t)c.n_layers * c.max_seq * c.kv_dim; break;
    case 6: src = s->kd; n = s->kd ? sizeof(float) * (size_t)c.n_layers * c.max_seq * c.n_kv_heads : 0; break;
    case 7: src = s->vd; n = s->vd ? sizeof(float) * (size_t)c.n_layers * c.max_seq * c.n_kv_heads : 0; break;
    default: return KC_E_SHAPE;
    }
    CK(cudaStreamSynchronize(s->st));
    if (words) {
        if (bytes < n * sizeof(float)) return KC_E_SHAPE;
        std::vector<unsigned long long> h(n);
        CK(cudaMemcpy(h.data(), words, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < n; i++) {
            const unsigned u = (unsigned)h[i];
            std::memcpy((char *)dst + i * sizeof(float), &u, sizeof(float));
        }
        return KC_OK;
    }
    if (bytes < n || !src) return KC_E_SHAPE;
    CK(cudaMemcpy(dst, src, n, cudaMemcpyDeviceToHost));
    return KC_OK;
}

extern "C" int kc_step_timeline(kc_state *s, int token, int pos, unsigned long long *t, int cap, int *n) {
    clear_error();
    const kc_config &c = s->c;
    if (pos < 0 || pos >= c.max_seq || token < 0 || token >= c.vocab) return KC_E_SHAPE;
    int st = set_loop(s, token, pos, 0);
    if (st == KC_OK) st = launch_steps(s, 1, 1, true);
    if (st != KC_OK) return st;
    unsigned cnt = 0;
    CK(cudaMemcpyAsync(&cnt, s->timeline_n, sizeof cnt, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    if (cnt > 4096) cnt = 4096;
    if ((int)cnt > cap) cnt = (unsigned)cap;
    CK(cudaMemcpy(t, s->timeline, sizeof(unsigned long long) * cnt, cudaMemcpyDeviceToHost));
    *n = (int)cnt;
    return finish(s);
}

extern "C" int kc_step_trace(kc_state *s, int token, int pos, unsigned long long *out, size_t cap, int *nphases,
                             int *nctas) {
    clear_error();
    const kc_config &c = s->c;
    if (pos < 0 || pos >= c.max_seq || token < 0 || token >= c.vocab) return KC_E_SHAPE;
    const int P = 5 * c.n_layers + 1, G = s->num_sms;
    const size_t n = (size_t)P * G * 3;
    if (cap < n) return KC_E_SHAPE;
    unsigned long long *d = nullptr;
    CK(cudaMalloc(&d, n * sizeof(unsigned long long)));
    int st = set_loop(s, token, pos, 0);
    if (st == KC_OK) {
        StepArgs save = s->sa;
        s->sa.trace = d;
        s->sa.trace_phases = (unsigned)P;
        st = launch_steps(s, 1, 1, true);
        s->sa = save;
    }
    cudaError_t e = cudaStreamSynchronize(s->st);
    if (e == cudaSuccess) e = cudaMemcpy(out, d, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_status(e, "trace");
    if (st != KC_OK) return st;
    *nphases = P;
    *nctas = G;
    return finish(s);
}

extern "C" int kc_step_events(kc_state *s, int token, int pos, unsigned long long *out, unsigned cap, int *nctas) {
    clear_error();
    const kc_config &c = s->c;
    if (pos < 0 || pos >= c.max_seq || token < 0 || token >= c.vocab || cap == 0) return KC_E_SHAPE;
    const int G = s->num_sms;
    const size_t n = (size_t)G * 2 * cap;
    unsigned long long *d = nullptr;
    CK(cudaMalloc(&d, n * sizeof(unsigned long long)));
    cudaError_t e = cudaMemset(d, 0, n * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_evlog, &d, sizeof(d));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_evcap, &cap, sizeof(cap));
    int st = e == cudaSuccess ? set_loop(s, token, pos, 0) : cuda_status(e, "events");
    if (st == KC_OK) st = launch_steps(s, 1, 1, true);
    e = cudaStreamSynchronize(s->st);
    unsigned long long *null_log = nullptr;
    const cudaError_t e2 = cudaMemcpyToSymbol(g_evlog, &null_log, sizeof(null_log));
    if (e == cudaSuccess) e = e2;
    if (e == cudaSuccess) e = cudaMemcpy(out, d, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_status(e, "events");
    if (st != KC_OK) return st;
    *nctas = G;
    return finish(s);
}

/* ------------------------------------------------------------ kernel-level */

static int activation_smem(int n) { return 128 + n + 8 * (n / QK) + 16; }

extern "C" int kc_quantize_q8_dev(int8_t *q, float *d, const float *x, int k, void *stream) {
    if (k <= 0 || k % QK) return KC_E_SHAPE;
    const int smem = activation_smem(k);
    if (set_smem_attributes() != KC_OK || smem > KC_MAX_SMEM) return KC_E_SHAPE;
    activation_kernel<<<1, NCT, smem, (cudaStream_t)stream>>>(x, nullptr, 0.0f, k, q, d, nullptr);
    CK(cudaGetLastError());
    return KC_OK;
}

extern "C" int kc_rmsnorm_quantize_dev(int8_t *q, float *d, float *xn, const float *x, const float *w, int n, float eps,
                                       void *stream) {
    if (n <= 0 || n % QK || !w) return KC_E_SHAPE;
    const int smem = activation_smem(n);
    if (set_smem_attributes() != KC_OK || smem > KC_MAX_SMEM) return KC_E_SHAPE;
    activation_kernel<<<1, NCT, smem, (cudaStream_t)stream>>>(x, w, eps, n, q, d, xn);
    CK(cudaGetLastError());
    return KC_OK;
}

extern "C" int kc_matvec_dev(float *y, int type, int d_f16, const void *wq, const void *wd, int rows, int cols,
                             const int8_t *xq, const float *xd, void *stream) {
    clear_error();
    if (rows <= 0 || cols <= 0 || cols % QK || (type != KC_Q8_0 && type != KC_Q4_0)) return KC_E_SHAPE;
    int dev = 0, rc = current_device(dev);
    if (rc == KC_OK) rc = set_smem_attributes();
    unsigned *err = nullptr;
    if (rc == KC_OK) rc = kl_err_word(dev, err);
    if (rc != KC_OK) return rc;
    MatvecArgs p{};
    p.m = PMat{ (const uint8_t *)wq, wd, rows, type, d_f16 };
    p.cols = cols; p.xq = xq; p.xd = xd; p.y = y; p.err = err; p.wait_limit = g_wait_limit;
    p.slot_bytes = stage_slot_bytes(type, d_f16, cols, 0);
    p.act_bytes = (cols + 8 * (cols / QK) + 15) & ~15;
    cudaFuncAttributes fa;
    CK(cudaFuncGetAttributes(&fa, matvec_kernel));
    p.nstage = ring_stages(p.slot_bytes, p.act_bytes, (int)fa.sharedSizeBytes);
    if (p.nstage < 2) return KC_E_SHAPE;
    const int smem = smem_fixed_bytes(p.nstage, p.act_bytes) + p.nstage * p.slot_bytes;
    int sms = 148;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int grid = rows < sms ? rows : sms;
    matvec_kernel<<<grid, STEP_THREADS, smem, (cudaStream_t)stream>>>(p);
    CK(cudaGetLastError());
    return KC_OK;
}

/* ------------------------------------------------------------ no-allocation matvec */

/* Device scratch of kc_matvec_f32_noalloc: the quantized activation
 * (KC_NOALLOC_MAX_COLS int8 quants, then their block scales) and the ring's
 * error word. Zero at module load; the quants and scales are rewritten by
 * every call before they are read, and the error word is sticky: a wait that
 * gave up stays flagged until kc_dev_sync reports and clears it. One copy per
 * device, shared by all callers: calls that overlap in time (different
 * streams or threads) race on it. */
constexpr int NOALLOC_XD_OFF = KC_NOALLOC_MAX_COLS;
constexpr int NOALLOC_ERR_OFF = NOALLOC_XD_OFF + (KC_NOALLOC_MAX_COLS / QK) * 4;
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_ERR_OFF + 256];

static unsigned char *g_noalloc_ptr[KC_MAX_DEVICES];   /* the scratch's address on each device, set on first use */

extern "C" int kc_matvec_f32_noalloc(float *y, int type, int d_f16, const void *wq, const void *wd, int rows, int cols,
                                     const float *x, void *stream) {
    clear_error();
    if (rows <= 0 || cols <= 0 || cols % QK || (type != KC_Q8_0 && type != KC_Q4_0)) return KC_E_SHAPE;
    if (cols > KC_NOALLOC_MAX_COLS) {
        set_error("kc_matvec_f32_noalloc: cols " + std::to_string(cols) + " exceeds the scratch limit of " +
                  std::to_string(KC_NOALLOC_MAX_COLS));
        return KC_E_SHAPE;
    }
    int dev = 0;
    const int rc = current_device(dev);
    if (rc != KC_OK) return rc;
    if (!g_noalloc_ptr[dev]) {
        /* once per device, with that device current (the first call should come before any stream capture) */
        void *ptr = nullptr;
        CK(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
        g_noalloc_ptr[dev] = (unsigned char *)ptr;
    }
    if (set_smem_attributes() != KC_OK) return KC_E_IO;
    unsigned char *scr = g_noalloc_ptr[dev];
    int8_t *xq = (int8_t *)scr;
    float *xd = (float *)(scr + NOALLOC_XD_OFF);
    unsigned *err = (unsigned *)(scr + NOALLOC_ERR_OFF);
    const cudaStream_t st = (cudaStream_t)stream;
    const int asmem = 128 + cols + 8 * (cols / QK) + 16;
    activation_kernel<<<1, NCT, asmem, st>>>(x, nullptr, 0.0f, cols, xq, xd, nullptr);
    CK(cudaGetLastError());
    MatvecArgs p{};
    p.m = PMat{ (const uint8_t *)wq, wd, rows, type, d_f16 };
    p.cols = cols; p.xq = xq; p.xd = xd; p.y = y; p.err = err; p.wait_limit = g_wait_limit;
    p.slot_bytes = stage_slot_bytes(type, d_f16, cols, 0);
    p.act_bytes = (cols + 8 * (cols / QK) + 15) & ~15;
    cudaFuncAttributes fa;
    CK(cudaFuncGetAttributes(&fa, matvec_kernel));
    p.nstage = ring_stages(p.slot_bytes, p.act_bytes, (int)fa.sharedSizeBytes);
    if (p.nstage < 2) return KC_E_SHAPE;
    const int smem = smem_fixed_bytes(p.nstage, p.act_bytes) + p.nstage * p.slot_bytes;
    int sms = 148;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int grid = rows < sms ? rows : sms;
    matvec_kernel<<<grid, STEP_THREADS, smem, st>>>(p);
    CK(cudaGetLastError());
    return KC_OK;
}

extern "C" int kc_block_sums_dev(int32_t *s, int type, const void *wq, int rows, int cols, const int8_t *xq,
                                 void *stream) {
    if (rows <= 0 || cols <= 0 || cols % QK || (type != KC_Q8_0 && type != KC_Q4_0)) return KC_E_SHAPE;
    const size_t total = (size_t)rows * (cols / QK);
    int blocks = (int)((total + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    block_sums_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(s, type, (const uint8_t *)wq, rows, cols, xq);
    CK(cudaGetLastError());
    return KC_OK;
}

extern "C" void *kc_dev_alloc(size_t bytes) {
    void *p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    return p;
}
extern "C" void kc_dev_free(void *p) { if (p) cudaFree(p); }
extern "C" int kc_memcpy_htod(void *dst, const void *src, size_t n) { CK(cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice)); return KC_OK; }
extern "C" int kc_memcpy_dtoh(void *dst, const void *src, size_t n) { CK(cudaMemcpy(dst, src, n, cudaMemcpyDeviceToHost)); return KC_OK; }
/* Waits for the current device, then reads (and clears) the sticky error
 * words of the kernel-level matvec entry points on it. */
extern "C" int kc_dev_sync(void) {
    clear_error();
    CK(cudaDeviceSynchronize());
    int dev = 0;
    const int rc = current_device(dev);
    if (rc != KC_OK) return rc;
    unsigned *words[2] = { g_kl_err_ptr[dev], g_noalloc_ptr[dev] ? (unsigned *)(g_noalloc_ptr[dev] + NOALLOC_ERR_OFF) : nullptr };
    const char *names[2] = { "kc_matvec_dev", "kc_matvec_f32_noalloc" };
    std::string msg;
    for (int i = 0; i < 2; i++) {
        if (!words[i]) continue;
        unsigned w = 0;
        CK(cudaMemcpy(&w, words[i], sizeof w, cudaMemcpyDeviceToHost));
        if (!w) continue;
        CK(cudaMemset(words[i], 0, sizeof w));
        msg += std::string(msg.empty() ? "" : "; ") + names[i] + ": a device wait gave up (error word " +
               std::to_string(w) + ")";
    }
    if (msg.empty()) return KC_OK;
    set_error(msg);
    return KC_E_IO;
}

extern "C" int kc_debug_wait_limit(int polls) {
    g_wait_limit = polls < 0 ? WAIT_POLLS : (unsigned)polls;
    return KC_OK;
}

/* ------------------------------------------------------------------ sampler */

struct kc_sampler {
    kc_state *s = nullptr;
    kc_sampler_opts o{};
    uint8_t *arena = nullptr;
    SampleArgs a{};
    SamplerDev host{};        /* mirror of the device state, refreshed after each call */
    std::vector<int> ring;    /* mirror of the device ring */
};

extern "C" void kc_sampler_free(kc_sampler *p) {
    if (!p) return;
    if (p->arena) cudaFree(p->arena);
    delete p;
}

extern "C" int kc_sampler_init(kc_sampler **out, kc_state *s, const kc_sampler_opts *o) {
    clear_error();
    *out = nullptr;
    if (!(o->temperature >= 0.0f) || o->topk < 0) return KC_E_SHAPE;
    kc_sampler *p = new (std::nothrow) kc_sampler();
    if (!p) return KC_E_NOMEM;
    p->s = s;
    p->o = *o;
    if (p->o.repeat_last_n < 0) p->o.repeat_last_n = 0;
    const size_t V = (size_t)s->c.vocab, RL = (size_t)(p->o.repeat_last_n > 0 ? p->o.repeat_last_n : 1);
    /* the spare key buffer also holds the selection's candidates (SM_TOPK_MAX 64-bit words) */
    const size_t KB = std::max(sizeof(unsigned) * V, sizeof(unsigned long long) * SM_TOPK_MAX);
    const size_t sz[] = { sizeof(SamplerDev), sizeof(int) * RL, sizeof(float) * V, sizeof(unsigned) * V,
                          KB, sizeof(int) * V, sizeof(int) * V, sizeof(int) };
    size_t total = 0;
    for (size_t b : sz) total += align256(b);
    cudaError_t e = cudaMalloc(&p->arena, total);
    if (e != cudaSuccess) {
        kc_sampler_free(p);
        return cuda_status(e, "sampler");
    }
    uint8_t *q = p->arena;
    void *ptr[8];
    for (int i = 0; i < 8; i++) {
        ptr[i] = q;
        q += align256(sz[i]);
    }
    SampleArgs &a = p->a;
    a.vocab = s->c.vocab;
    a.temperature = p->o.temperature;
    a.topp = p->o.topp;
    a.topk = p->o.topk;
    a.repeat_penalty = p->o.repeat_penalty;
    a.repeat_last_n = p->o.repeat_last_n;
    a.st = (SamplerDev *)ptr[0];
    a.recent = (int *)ptr[1];
    a.p = (float *)ptr[2];
    a.ka = (unsigned *)ptr[3];
    a.kb = (unsigned *)ptr[4];
    a.va = (int *)ptr[5];
    a.vb = (int *)ptr[6];
    a.token_out = (int *)ptr[7];
    p->host.rng = p->o.seed ? p->o.seed : 0x9E3779B97F4A7C15ull;   /* model/sampler.c:10 */
    p->ring.assign(RL, 0);
    e = cudaMemcpy(a.st, &p->host, sizeof p->host, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(a.recent, p->ring.data(), sizeof(int) * RL, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        kc_sampler_free(p);
        return cuda_status(e, "sampler");
    }
    *out = p;
    return KC_OK;
}

/* The device state and ring back into the host mirror. */
static int sampler_pull(kc_sampler *p) {
    CK(cudaMemcpyAsync(&p->host, p->a.st, sizeof p->host, cudaMemcpyDeviceToHost, p->s->st));
    CK(cudaMemcpyAsync(p->ring.data(), p->a.recent, sizeof(int) * p->ring.size(), cudaMemcpyDeviceToHost, p->s->st));
    CK(cudaStreamSynchronize(p->s->st));
    return KC_OK;
}

extern "C" int kc_sampler_accept(kc_sampler *p, int token) {
    clear_error();
    const int rl = p->o.repeat_last_n;
    if (rl <= 0 || token < 0 || token >= p->s->c.vocab) return KC_OK;
    p->ring[(size_t)p->host.recent_at] = token;
    p->host.recent_at = (p->host.recent_at + 1) % rl;
    if (p->host.n_recent < rl) p->host.n_recent++;
    CK(cudaMemcpyAsync(p->a.st, &p->host, sizeof p->host, cudaMemcpyHostToDevice, p->s->st));
    CK(cudaMemcpyAsync(p->a.recent, p->ring.data(), sizeof(int) * p->ring.size(), cudaMemcpyHostToDevice, p->s->st));
    CK(cudaStreamSynchronize(p->s->st));
    return KC_OK;
}

extern "C" int kc_sampler_rng(kc_sampler *p, uint64_t *rng) {
    *rng = p->host.rng;
    return KC_OK;
}

extern "C" int kc_sample(kc_sampler *p, int *token) {
    clear_error();
    kc_state *s = p->s;
    if (s->last_row < 0) {
        set_error("no logits of a last token on the device: run kc_forward first");
        return KC_E_SHAPE;
    }
    SampleArgs a = p->a;
    a.logits = s->logits + (size_t)s->last_row * s->c.vocab;
    a.ls = nullptr;
    a.out_tokens = nullptr;
    sample_kernel<<<1, SM_THREADS, 0, s->st>>>(a);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(token, a.token_out, sizeof(int), cudaMemcpyDeviceToHost, s->st));
    return sampler_pull(p);
}

extern "C" int kc_generate_sampled(kc_state *s, kc_sampler *p, int token, int pos, int n, int *out_tokens) {
    clear_error();
    const kc_config &c = s->c;
    if (p->s != s || n < 0 || pos < 0 || pos + n > c.max_seq || token < 0 || token >= c.vocab) return KC_E_SHAPE;
    if (n == 0) return KC_OK;
    int st = set_loop(s, token, pos, 0);
    if (st != KC_OK) return st;
    for (int i = 0; i < n; i++) {
        st = run_steps(s, 1, 1);
        if (st != KC_OK) return st;
        SampleArgs a = p->a;
        a.logits = s->logits + (size_t)(i % LOGITS_RING) * c.vocab;
        a.ls = s->ls;
        a.out_tokens = s->out_tokens;
        sample_kernel<<<1, SM_THREADS, 0, s->st>>>(a);
        CK(cudaGetLastError());
    }
    CK(cudaMemcpyAsync(out_tokens, s->out_tokens, sizeof(int) * n, cudaMemcpyDeviceToHost, s->st));
    st = finish(s);
    if (st != KC_OK) return st;
    s->last_row = (n - 1) % LOGITS_RING;
    return sampler_pull(p);
}

