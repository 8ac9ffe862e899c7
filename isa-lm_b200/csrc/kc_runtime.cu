/* Runtime of libkrafla_cuda: HBM upload of the model, the decode state with
 * its device arena and KV cache, one CUDA graph per token step (replayed for
 * every token: token and position live in device memory), and the C ABI of
 * include/krafla_cuda.h. */
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <thread>
#include <string>
#include <vector>
#include <sys/mman.h>

#include "kc_internal.h"
#include "kc_kernels.cuh"

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

extern "C" const kc_config *kc_model_config(const kc_model *m) { return &m->cfg; }
extern "C" size_t kc_model_device_bytes(const kc_model *m) { return m->dev_bytes; }

extern "C" void kc_model_free(kc_model *m) {
    if (!m) return;
    if (m->dev_base) cudaFree(m->dev_base);
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
        mat(H.wq, D.wq); mat(H.wk, D.wk); mat(H.wv, D.wv); mat(H.wo, D.wo);
        mat(H.w1, D.w1); mat(H.w2, D.w2); mat(H.w3, D.w3);
        vec(H.bq, (size_t)c.q_dim, D.bq); vec(H.bk, (size_t)c.kv_dim, D.bk); vec(H.bv, (size_t)c.kv_dim, D.bv);
        vec(H.q_norm, (size_t)c.head_dim, D.q_norm); vec(H.k_norm, (size_t)c.head_dim, D.k_norm);
        vec(H.post_attn_norm, (size_t)c.dim, D.post_attn_norm); vec(H.post_ffn_norm, (size_t)c.dim, D.post_ffn_norm);
        D.window = H.window;
        D.local_rope = H.local_rope;
    }
    vec(m->final_norm, (size_t)c.dim, m->d_final_norm);
    if (!m->shared) mat(m->wcls, m->d_wcls);
    size_t total = 0;
    for (const Item &it : items) total += align256(it.bytes);
    uint8_t *base = nullptr;
    CK(cudaMalloc(&base, total ? total : 256));
    size_t off = 0;
    for (const Item &it : items) {
        cudaError_t e = cudaMemcpy(base + off, it.src, it.bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(base);
            return cuda_status(e, "upload");
        }
        *it.dst = base + off;
        off += align256(it.bytes);
    }
    if (m->shared) m->d_wcls = m->d_tok_emb;
    m->dev_base = base;
    m->dev_bytes = total;
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
    float *x = nullptr, *qkv = nullptr, *ao = nullptr, *hb = nullptr, *logits = nullptr, *part = nullptr;
    float *kc = nullptr, *vc = nullptr, *rcos = nullptr, *rsin = nullptr, *lcos = nullptr, *lsin = nullptr;
    float *flush = nullptr;
    size_t flush_bytes = 0;
    float *inv0 = nullptr;   /* [vocab]: 1/rms of each embedding row (layer 0's RMSNorm) */
    unsigned *counter = nullptr, *err = nullptr;
    LoopState *ls = nullptr;
    int *feed = nullptr, *out_tokens = nullptr;
    float *h_logits = nullptr;
    LoopState *h_ls = nullptr;
    cudaGraphExec_t g_logits = nullptr, g_nologits = nullptr;
    int nsplit = 32;
    int num_sms = 148;
};

/* RoPE inverse frequency of pair i (model/transformer.c:16-38; the scaling
 * formulas of transformers: linear, yarn, llama3), in double. */
static double rope_inv_freq(const kc_config &c, int i) {
    const double inv = std::pow((double)c.rope_theta, -2.0 * i / c.head_dim);
    if (c.rope_type == 2) return inv / c.rope_factor;
    if (c.rope_type == 3) {
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
    if (c.rope_type != 1) return inv;
    const double f = c.rope_factor, lo = c.rope_low_freq_factor, hi = c.rope_high_freq_factor;
    const double orig = c.rope_orig_max_seq, wavelen = 2.0 * 3.14159265358979323846 / inv;
    if (wavelen < orig / hi) return inv;
    if (wavelen > orig / lo) return inv / f;
    const double smooth = (orig / wavelen - lo) / (hi - lo);
    return (1.0 - smooth) * inv / f + smooth * inv;
}

static unsigned *g_err_word = nullptr;
static const int KC_MAX_SMEM = 227 * 1024;

/* Opt-in to the full shared memory of an sm_100 CTA (outside any stream capture). */
static int set_smem_attributes() {
    static bool done = false;
    if (done) return KC_OK;
    const void *fns[] = { (const void *)gemv_kernel, (const void *)attn_kernel, (const void *)quantize_kernel };
    for (const void *f : fns) {
        cudaFuncAttributes a;
        CK(cudaFuncGetAttributes(&a, f));
        CK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, KC_MAX_SMEM - (int)a.sharedSizeBytes));
    }
    done = true;
    return KC_OK;
}   /* device error word of the kernel-level entry points */

/* Launches the GEMV over p's segments. Each segment gets CTAs in proportion
 * to its weight bytes out of the CTAs that fit on the device at once (each
 * CTA then streams a contiguous range of rows). */
static int launch_gemv(kc_state *s, GemvParams &p, cudaStream_t st, unsigned *err) {
    double bytes[MAX_SEGS], total = 0.0;
    for (int i = 0; i < p.nseg; i++) {
        const Seg &g = p.seg[i];
        bytes[i] = (double)g.rows * (g.type == T_Q4 ? p.cols / 2 : p.cols) * (g.epi == EPI_PAIR ? 2 : 1);
        total += bytes[i];
    }
    const int smem = gemv_smem_bytes(p);
    if (smem > KC_MAX_SMEM) return KC_E_SHAPE;
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_kernel, GEMV_THREADS + 32, smem);
    if (per_sm < 1) per_sm = 1;
    const int budget = per_sm * (s ? s->num_sms : 148);
    int ctas = 0;
    for (int i = 0; i < p.nseg; i++) {
        Seg &g = p.seg[i];
        int n = (int)((double)budget * bytes[i] / total + 0.5);
        if (n < 1) n = 1;
        if (n > g.rows) n = g.rows;
        g.cta0 = ctas;
        g.ctas = n;
        ctas += n;
    }
    p.err = err;
    gemv_kernel<<<ctas, GEMV_THREADS + 32, smem, st>>>(p);
    return KC_OK;
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
        if (E.d16) {
            const uint16_t h = ((const uint16_t *)E.d)[i];
            const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, mm = h & 0x3ffu;
            if (e == 0) return (sign ? -1.0f : 1.0f) * (float)mm * (1.0f / 16777216.0f);
            const uint32_t x = sign | (e == 31 ? 0x7f800000u | (mm << 13) : ((e + 112u) << 23) | (mm << 13));
            float f;
            std::memcpy(&f, &x, 4);
            return f;
        }
        return ((const float *)E.d)[i];
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

static int gemv_smem(int cols) { return cols + 8 * (cols / QK) + 128; }

static Seg seg_of(const DevMat &w, int epi, float *out, const float *bias, int nr) {
    Seg g{};
    g.q = w.q; g.d = w.d; g.rows = w.rows; g.type = w.type; g.d16 = w.d16;
    g.epi = epi; g.out = out; g.bias = bias; (void)nr;
    return g;
}

/* The kernels of one decode step, in stream order. kernel_class: when
 * non-null, events are recorded around each class (profiling only). */
static void enqueue_step(kc_state *s, bool logits, cudaEvent_t *ev = nullptr, int *nev = nullptr) {
    kc_model *m = s->m;
    const kc_config &c = s->c;
    cudaStream_t st = s->st;
    auto mark = [&]() {
        if (ev) cudaEventRecord(ev[(*nev)++], st);
    };
    const DevMat &E = m->d_tok_emb;
    mark();
    if (E.d16)
        embed_kernel<true><<<(c.dim + 255) / 256, 256, 0, st>>>(s->x, E.q, E.d, E.type, c.dim, c.vocab, c.max_seq,
                                                                c.embed_scale, s->ls);
    else
        embed_kernel<false><<<(c.dim + 255) / 256, 256, 0, st>>>(s->x, E.q, E.d, E.type, c.dim, c.vocab, c.max_seq,
                                                                 c.embed_scale, s->ls);
    const size_t lkv = (size_t)c.max_seq * c.kv_dim;
    const int group = c.n_heads / c.n_kv_heads;
    const int att_smem = (int)sizeof(float) *
                         (group * c.head_dim + ATT_TILE * (c.head_dim + 1) + ATT_TILE * c.head_dim + group * ATT_TILE + 3 * group);
    for (int l = 0; l < c.n_layers; l++) {
        const DevLayer &L = m->d_layers[(size_t)l];
        /* 1. RMSNorm + quantize + Q/K/V projections (+ biases) */
        GemvParams p{};
        p.cols = c.dim; p.pro = PRO_RMSNORM_QUANT; p.x = s->x; p.norm_w = L.attn_norm; p.eps = c.norm_eps;
        if (l == 0) {
            p.inv_tab = s->inv0;
            p.inv_token = &s->ls->token;
        }
        p.seg[0] = seg_of(L.wq, EPI_STORE, s->qkv, L.bq, 2);
        p.seg[1] = seg_of(L.wk, EPI_STORE, s->qkv + c.q_dim, L.bk, 2);
        p.seg[2] = seg_of(L.wv, EPI_STORE, s->qkv + c.q_dim + c.kv_dim, L.bv, 2);
        p.nseg = 3;
        mark();
        launch_gemv(s, p, st, s->err);
        /* 2. attention (RoPE, KV store, split-K flash decode, combine) */
        AttnParams a{};
        a.qkv = s->qkv; a.kc = s->kc + (size_t)l * lkv; a.vc = s->vc + (size_t)l * lkv;
        a.rcos = L.local_rope ? s->lcos : s->rcos; a.rsin = L.local_rope ? s->lsin : s->rsin;
        a.ao = s->ao; a.part = s->part; a.counter = s->counter; a.ls = s->ls;
        a.n_heads = c.n_heads; a.n_kv_heads = c.n_kv_heads; a.hd = c.head_dim; a.q_dim = c.q_dim; a.kv_dim = c.kv_dim;
        a.max_seq = c.max_seq; a.window = L.window; a.nsplit = s->nsplit; a.scale = c.attn_scale; a.softcap = c.attn_softcap;
        mark();
        attn_kernel<<<dim3(c.n_kv_heads, s->nsplit), ATT_THREADS, att_smem, st>>>(a);
        /* 3. quantize + output projection + residual */
        GemvParams o{};
        o.cols = c.q_dim; o.pro = PRO_QUANT; o.x = s->ao;
        o.seg[0] = seg_of(L.wo, EPI_RESID, s->x, nullptr, 2);
        o.nseg = 1;
        mark();
        launch_gemv(s, o, st, s->err);
        /* 4. RMSNorm + quantize + gate/up + activation */
        GemvParams u{};
        u.cols = c.dim; u.pro = PRO_RMSNORM_QUANT; u.x = s->x; u.norm_w = L.ffn_norm; u.eps = c.norm_eps; u.act = c.act;
        u.seg[0] = seg_of(L.w1, EPI_PAIR, s->hb, nullptr, 1);
        u.seg[0].q2 = L.w3.q;
        u.seg[0].d2 = L.w3.d;
        u.nseg = 1;
        mark();
        launch_gemv(s, u, st, s->err);
        /* 5. quantize + down projection + residual */
        GemvParams dn{};
        dn.cols = c.hidden_dim; dn.pro = PRO_QUANT; dn.x = s->hb;
        dn.seg[0] = seg_of(L.w2, EPI_RESID, s->x, nullptr, 2);
        dn.nseg = 1;
        mark();
        launch_gemv(s, dn, st, s->err);
    }
    mark();
    if (logits) {
        GemvParams h{};
        h.cols = c.dim; h.pro = PRO_RMSNORM_QUANT; h.x = s->x; h.norm_w = m->d_final_norm; h.eps = c.norm_eps;
        h.seg[0] = seg_of(m->d_wcls, EPI_LOGITS, s->logits, nullptr, 2);
        h.nseg = 1;
        h.softcap = c.final_softcap; h.ls = s->ls; h.feed = s->feed; h.out_tokens = s->out_tokens; h.vocab = c.vocab;
        launch_gemv(s, h, st, s->err);
    } else {
        advance_kernel<<<1, 1, 0, st>>>(s->ls, s->feed);
    }
    mark();
}

static int capture(kc_state *s, bool logits, cudaGraphExec_t *out) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    enqueue_step(s, logits);
    cudaError_t e = cudaStreamEndCapture(s->st, &g);
    if (e != cudaSuccess) return cuda_status(e, "graph capture");
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_status(e, "graph instantiate");
    return KC_OK;
}

extern "C" void kc_state_free(kc_state *s) {
    if (!s) return;
    if (s->st) cudaStreamSynchronize(s->st);
    if (s->g_logits) cudaGraphExecDestroy(s->g_logits);
    if (s->g_nologits) cudaGraphExecDestroy(s->g_nologits);
    if (s->arena) cudaFree(s->arena);
    if (s->flush) cudaFree(s->flush);
    if (s->h_logits) cudaFreeHost(s->h_logits);
    if (s->h_ls) cudaFreeHost(s->h_ls);
    if (s->st) cudaStreamDestroy(s->st);
    delete s;
}

extern "C" int kc_state_init(kc_state **out, kc_model *m, int nthreads, int kv_type) {
    (void)nthreads;
    *out = nullptr;
    clear_error();
    if (kv_type != KC_F32 && kv_type != KC_F16 && kv_type != KC_Q8_0) return KC_E_SHAPE;
    const kc_config &c = m->cfg;
    if (kv_type != KC_F32) { set_error("KV cache type not supported by this build yet"); return KC_E_SHAPE; }
    if (c.qk_norm || c.post_norms) { set_error("qk_norm / post_norms not supported by this build yet"); return KC_E_SHAPE; }
    const int group = c.n_heads / c.n_kv_heads;
    if (group * c.head_dim > ATT_THREADS * ATT_MAX_OUT || c.head_dim % 4) {
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
    auto fail = [&](int code) { kc_state_free(s); return code; };
    cudaError_t e = cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking);
    if (e != cudaSuccess) return fail(cuda_status(e, "stream"));

    const size_t T = (size_t)c.max_seq, h2 = (size_t)c.head_dim / 2;
    const size_t lkv = (size_t)c.n_layers * T * c.kv_dim;
    struct Buf { void **p; size_t bytes; };
    std::vector<Buf> bufs = {
        { (void **)&s->x, sizeof(float) * c.dim },
        { (void **)&s->qkv, sizeof(float) * (size_t)(c.q_dim + 2 * c.kv_dim) },
        { (void **)&s->ao, sizeof(float) * c.q_dim },
        { (void **)&s->hb, sizeof(float) * c.hidden_dim },
        { (void **)&s->logits, sizeof(float) * (size_t)LOGITS_RING * c.vocab },
        { (void **)&s->part, sizeof(float) * (size_t)c.n_heads * s->nsplit * (c.head_dim + 2) },
        { (void **)&s->counter, sizeof(unsigned) * c.n_kv_heads },
        { (void **)&s->err, sizeof(unsigned) * 4 },
        { (void **)&s->ls, sizeof(LoopState) },
        { (void **)&s->feed, sizeof(int) * (T + 1) },
        { (void **)&s->out_tokens, sizeof(int) * (T + 1) },
        { (void **)&s->kc, sizeof(float) * lkv },
        { (void **)&s->vc, sizeof(float) * lkv },
        { (void **)&s->rcos, sizeof(float) * T * h2 },
        { (void **)&s->inv0, sizeof(float) * (size_t)c.vocab },
        { (void **)&s->rsin, sizeof(float) * T * h2 },
    };
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
    e = cudaMemsetAsync(s->arena, 0, total, s->st);
    if (e != cudaSuccess) return fail(cuda_status(e, "memset"));
    e = cudaMallocHost(&s->h_logits, sizeof(float) * c.vocab);
    if (e == cudaSuccess) e = cudaMallocHost(&s->h_ls, sizeof(LoopState));
    if (e != cudaSuccess) return fail(cuda_status(e, "pinned host buffers"));

    /* RoPE tables: double, stored as float (model/transformer.c:146-162) */
    {
        std::vector<float> cs(T * h2), sn(T * h2), lc, ls_;
        const double af = c.rope_type == 3 ? c.rope_attn_factor : 1.0;
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
    {
        const int att = (int)sizeof(float) * (group * c.head_dim + ATT_TILE * (c.head_dim + 1) + ATT_TILE * c.head_dim +
                                              group * ATT_TILE + 3 * group);
        GemvParams big{};
        big.nseg = 1;
        big.seg[0].type = T_Q8;
        big.seg[0].d16 = 0;
        big.seg[0].epi = EPI_PAIR;
        const int widest = c.hidden_dim > c.dim ? (c.hidden_dim > c.q_dim ? c.hidden_dim : c.q_dim) : (c.dim > c.q_dim ? c.dim : c.q_dim);
        big.cols = widest;
        if (att > KC_MAX_SMEM || gemv_smem_bytes(big) > KC_MAX_SMEM) {
            set_error("layer shapes exceed this build's shared-memory plan");
            return fail(KC_E_SHAPE);
        }
    }
    e = cudaStreamSynchronize(s->st);
    if (e != cudaSuccess) return fail(cuda_status(e, "state init"));
    st = capture(s, true, &s->g_logits);
    if (st == KC_OK) st = capture(s, false, &s->g_nologits);
    if (st != KC_OK) return fail(st);
    *out = s;
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
    unsigned err = 0;
    CK(cudaMemcpyAsync(s->h_ls, s->ls, sizeof(LoopState), cudaMemcpyDeviceToHost, s->st));
    CK(cudaMemcpyAsync(&err, s->err, sizeof err, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
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
    if (set_loop(s, token, pos, 0) != KC_OK) return nullptr;
    cudaError_t e = cudaGraphLaunch(s->g_logits, s->st);
    if (e != cudaSuccess) { cuda_status(e, "graph launch"); return nullptr; }
    e = cudaMemcpyAsync(s->h_logits, s->logits, sizeof(float) * c.vocab, cudaMemcpyDeviceToHost, s->st);
    if (e != cudaSuccess) { cuda_status(e, "logits copy"); return nullptr; }
    if (finish(s) != KC_OK) return nullptr;
    return s->h_logits;
}

extern "C" int kc_prefill(kc_state *s, const int *tokens, int n, int pos0, float *logits) {
    clear_error();
    const kc_config &c = s->c;
    if (n < 0 || pos0 < 0 || pos0 + n > c.max_seq) return KC_E_SHAPE;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= c.vocab) return KC_E_SHAPE;
    if (n == 0) return KC_OK;
    CK(cudaMemcpyAsync(s->feed, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemsetAsync(s->feed + n, 0, sizeof(int), s->st));
    int st = set_loop(s, tokens[0], pos0, 1);
    if (st != KC_OK) return st;
    for (int i0 = 0; i0 < n; i0 += LOGITS_RING) {
        const int k = n - i0 < LOGITS_RING ? n - i0 : LOGITS_RING;
        for (int i = 0; i < k; i++) CK(cudaGraphLaunch(logits ? s->g_logits : s->g_nologits, s->st));
        if (logits)
            CK(cudaMemcpyAsync(logits + (size_t)i0 * c.vocab, s->logits, sizeof(float) * (size_t)k * c.vocab,
                               cudaMemcpyDeviceToHost, s->st));
    }
    return finish(s);
}

extern "C" int kc_generate_greedy(kc_state *s, int token, int pos, int n, int *out_tokens) {
    clear_error();
    const kc_config &c = s->c;
    if (n < 0 || pos < 0 || pos + n > c.max_seq || token < 0 || token >= c.vocab) return KC_E_SHAPE;
    if (n == 0) return KC_OK;
    int st = set_loop(s, token, pos, 0);
    if (st != KC_OK) return st;
    for (int i = 0; i < n; i++) CK(cudaGraphLaunch(s->g_logits, s->st));
    CK(cudaMemcpyAsync(out_tokens, s->out_tokens, sizeof(int) * n, cudaMemcpyDeviceToHost, s->st));
    return finish(s);
}

extern "C" int kc_time_decode(kc_state *s, int token, int pos, int warmup, int steps, float *ms) {
    clear_error();
    const kc_config &c = s->c;
    if (pos < 0 || pos + warmup + steps > c.max_seq || token < 0 || token >= c.vocab || steps < 1) return KC_E_SHAPE;
    int st = set_loop(s, token, pos, 0);
    if (st != KC_OK) return st;
    for (int i = 0; i < warmup; i++) CK(cudaGraphLaunch(s->g_logits, s->st));
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    cudaEventRecord(e0, s->st);
    for (int i = 0; i < steps; i++) cudaGraphLaunch(s->g_logits, s->st);
    cudaEventRecord(e1, s->st);
    cudaError_t e = cudaEventSynchronize(e1);
    float t = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (e != cudaSuccess) return cuda_status(e, "decode timing");
    *ms = t;
    return finish(s);
}

extern "C" int kc_time_ffn_up(kc_state *s, int layer, int reps, float *ms_per_launch, double *bytes) {
    clear_error();
    const kc_config &c = s->c;
    if (layer < 0 || layer >= c.n_layers || reps < 1) return KC_E_SHAPE;
    const DevLayer &L = s->m->d_layers[(size_t)layer];
    if (!s->flush) {
        s->flush_bytes = (size_t)256 << 20;   /* larger than the 126 MB L2 */
        CK(cudaMalloc(&s->flush, s->flush_bytes));
    }
    GemvParams u{};
    u.cols = c.dim; u.pro = PRO_RMSNORM_QUANT; u.x = s->x; u.norm_w = L.ffn_norm; u.eps = c.norm_eps; u.act = c.act;
    u.seg[0] = seg_of(L.w1, EPI_PAIR, s->hb, nullptr, 1);
    u.seg[0].q2 = L.w3.q;
    u.seg[0].d2 = L.w3.d;
    u.nseg = 1;
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    float total = 0.0f;
    for (int r = 0; r < reps + 1; r++) {
        cudaMemsetAsync(s->flush, r & 0xff, s->flush_bytes, s->st);
        cudaEventRecord(e0, s->st);
        launch_gemv(s, u, s->st, s->err);
        cudaEventRecord(e1, s->st);
        cudaError_t e = cudaEventSynchronize(e1);
        float t = 0.0f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
        if (e != cudaSuccess) {
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
            return cuda_status(e, "ffn-up timing");
        }
        if (r > 0) total += t;   /* the first launch is a warm-up */
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *ms_per_launch = total / reps;
    const HostMat &w1 = s->m->layers[(size_t)layer].w1, &w3 = s->m->layers[(size_t)layer].w3;
    *bytes = (double)(w1.qbytes() + w1.dbytes() + w3.qbytes() + w3.dbytes());
    return KC_OK;
}

extern "C" int kc_profile_step(kc_state *s, int token, int pos, float *ms) {
    clear_error();
    const kc_config &c = s->c;
    if (pos < 0 || pos >= c.max_seq || token < 0 || token >= c.vocab) return KC_E_SHAPE;
    int st = set_loop(s, token, pos, 0);
    if (st != KC_OK) return st;
    const int nev = 2 + 5 * c.n_layers + 1;
    std::vector<cudaEvent_t> ev((size_t)nev);
    for (auto &e : ev) CK(cudaEventCreate(&e));
    int k = 0;
    enqueue_step(s, true, ev.data(), &k);
    CK(cudaStreamSynchronize(s->st));
    for (int i = 0; i < 6; i++) ms[i] = 0.0f;
    /* events: [embed] then per layer qkv, attn, wo, up, down, then [classifier], end */
    float t;
    cudaEventElapsedTime(&t, ev[0], ev[1]);
    ms[5] += t;   /* embedding counted with the classifier ("other") */
    for (int l = 0; l < c.n_layers; l++)
        for (int j = 0; j < 5; j++) {
            cudaEventElapsedTime(&t, ev[1 + 5 * l + j], ev[2 + 5 * l + j]);
            ms[j] += t;
        }
    cudaEventElapsedTime(&t, ev[(size_t)k - 2], ev[(size_t)k - 1]);
    ms[5] += t;
    for (auto &e : ev) cudaEventDestroy(e);
    return finish(s);
}

extern "C" int kc_debug_copy(kc_state *s, int which, void *dst, size_t bytes) {
    const kc_config &c = s->c;
    const void *src = nullptr;
    size_t n = 0;
    switch (which) {
    case 0: src = s->x; n = sizeof(float) * c.dim; break;
    case 1: src = s->qkv; n = sizeof(float) * (size_t)(c.q_dim + 2 * c.kv_dim); break;
    case 2: src = s->ao; n = sizeof(float) * c.q_dim; break;
    case 3: src = s->hb; n = sizeof(float) * c.hidden_dim; break;
    case 4: src = s->kc; n = sizeof(float) * (size_t)c.n_layers * c.max_seq * c.kv_dim; break;
    case 5: src = s->vc; n = sizeof(float) * (size_t)c.n_layers * c.max_seq * c.kv_dim; break;
    default: return KC_E_SHAPE;
    }
    if (bytes < n) return KC_E_SHAPE;
    CK(cudaStreamSynchronize(s->st));
    CK(cudaMemcpy(dst, src, n, cudaMemcpyDeviceToHost));
    return KC_OK;
}

/* ------------------------------------------------------------ kernel-level */

extern "C" int kc_quantize_q8_dev(int8_t *q, float *d, const float *x, int k, void *stream) {
    if (k <= 0 || k % QK) return KC_E_SHAPE;
    GemvParams p{};
    p.cols = k; p.pro = PRO_QUANT; p.x = x;
    const int smem = gemv_smem(k);
    if (set_smem_attributes() != KC_OK || smem > KC_MAX_SMEM) return KC_E_SHAPE;
    quantize_kernel<<<1, GEMV_THREADS, smem, (cudaStream_t)stream>>>(p, q, d, nullptr);
    CK(cudaGetLastError());
    return KC_OK;
}

extern "C" int kc_rmsnorm_quantize_dev(int8_t *q, float *d, float *xn, const float *x, const float *w, int n, float eps,
                                       void *stream) {
    if (n <= 0 || n % QK) return KC_E_SHAPE;
    GemvParams p{};
    p.cols = n; p.pro = PRO_RMSNORM_QUANT; p.x = x; p.norm_w = w; p.eps = eps;
    const int smem = gemv_smem(n);
    if (set_smem_attributes() != KC_OK || smem > KC_MAX_SMEM) return KC_E_SHAPE;
    quantize_kernel<<<1, GEMV_THREADS, smem, (cudaStream_t)stream>>>(p, q, d, xn);
    CK(cudaGetLastError());
    return KC_OK;
}

extern "C" int kc_matvec_dev(float *y, int type, int d_f16, const void *wq, const void *wd, int rows, int cols,
                             const int8_t *xq, const float *xd, void *stream) {
    if (rows <= 0 || cols <= 0 || cols % QK || (type != KC_Q8_0 && type != KC_Q4_0)) return KC_E_SHAPE;
    GemvParams p{};
    p.cols = cols; p.pro = PRO_PREQUANT; p.xq = xq; p.xd = xd;
    DevMat w;
    w.q = (const uint8_t *)wq; w.d = wd; w.rows = rows; w.cols = cols; w.type = type; w.d16 = d_f16;
    p.seg[0] = seg_of(w, EPI_STORE, y, nullptr, 2);
    p.nseg = 1;
    if (set_smem_attributes() != KC_OK) return KC_E_IO;
    if (!g_err_word) {
        CK(cudaMalloc(&g_err_word, sizeof(unsigned)));
        CK(cudaMemset(g_err_word, 0, sizeof(unsigned)));
    }
    const int st = launch_gemv(nullptr, p, (cudaStream_t)stream, g_err_word);
    if (st != KC_OK) return st;
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
extern "C" int kc_dev_sync(void) { CK(cudaDeviceSynchronize()); return KC_OK; }
