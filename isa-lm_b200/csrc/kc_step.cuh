/* The decode token loop as one persistent kernel (sm_100a), and the
 * kernel-level kernels that run the same device code.
 *
 * Weight stream. At upload, every CTA's rows of every matrix are laid out
 * contiguously in HBM in the order a step consumes them — per layer the fused
 * Q|K|V rows, the O rows, the gate|up row pairs, the down rows; then the
 * classifier rows — each row one record: quants, block scales, bias. The
 * producer warp of a CTA streams its own byte range into a ring of
 * shared-memory slots, one bulk copy per chunk of whole rows (<= 56 KB), the
 * slots handed over with full/empty mbarriers, so HBM keeps streaming while
 * the consumers wait on their inputs.
 *
 * The 8 consumer warps run the phases of a step:
 *   A  RMSNorm + quantize x (layer 0: the embedding row, its 1/rms from the
 *      host table) -> Q/K/V rows (+ biases)            model/transformer.c:270-277
 *   B  attention work items (KV head, position range): RoPE, this position's
 *      K/V row into the cache, split flash decode; the last split of a KV
 *      head unit to finish combines the unit's outputs and quantizes them
 *                                                      transformer.c:280-283, ops/ops.c:124-180
 *   C  O rows on the quantized attention output, x += o :284-287
 *   D  RMSNorm + quantize x -> gate/up row pairs -> act(g) * u, quantized by
 *      the CTA that owns the block                     :288-293
 *   E  down rows on the quantized hidden vector, x += y :294-297
 *   F  RMSNorm + quantize x -> classifier rows and the first-index argmax;
 *      the last CTA to arrive advances the token loop  :299-305, model/sampler.c:57-61
 * Between phases the vectors travel as tagged 64-bit words (see "tagged
 * words"): each CTA waits for exactly the words it reads; the one grid
 * barrier of a step is at its end. Several steps run in one launch: the token
 * of step s+1 is the argmax of step s (greedy) or the next prompt token.
 *
 * Each CTA owns the same rows of x in phases C and E; it keeps them in shared
 * memory (the residual add reads no global memory) and publishes them as words.
 *
 * Quantized activations follow the reference's rule bit for bit
 * (kernels/scalar/k_scalar.c:39-57); block dot products are exact int32
 * (dp4a); the float scale-accumulate is (float)s * d_w * d_x per block
 * (k_scalar.c:4-37) summed in lane order, then across the warp in a fixed tree.
 */
#pragma once
#include "kc_kernels.cuh"
#include "krafla_cuda.h"

namespace kc {

struct PMat {
    const uint8_t *q;
    const void *d;
    int rows, type, d16;
};

struct alignas(16) LayerPlan {
    const float *attn_norm, *ffn_norm;
    void *kc, *vc;                  /* this layer's cache [max_seq][kv_dim] of the state's KV type */
    float *kd, *vd;                 /* Q8 cache: scales [max_seq][n_kv_heads] */
    const float *rcos, *rsin;       /* RoPE tables of this layer */
    int window;
    const float *q_norm, *k_norm;   /* per-head RMSNorm of q and k before RoPE (Qwen3), or null */
    const float *post_attn, *post_ffn;   /* RMSNorm of a block's output before the residual add (Gemma 3), or null */
};

/* ------------------------------------------------------------ the weight stream */

/* Types of the streamed matrices (a matrix class has one type in every layer,
 * model/mlb.c:172) and the shapes. */
struct StreamGeom {
    int dim, q_dim, kv_dim, hidden, vocab;
    int t_q, t_k, t_v, t_o, t_up, t_down, t_cls;         /* T_Q8 / T_Q4 */
    int d16_q, d16_k, d16_v, d16_o, d16_up, d16_down, d16_cls;
    int b_q, b_k, b_v;                                     /* rows carry a bias */
    int d_unit;   /* rows of the gate|up phase are shared in units of d_unit: 32 (whole blocks), or 4 when whole
                   * blocks would leave some CTAs with a block more (split blocks agree on their maximum) */
    int chunk;    /* bytes per bulk copy (0: CHUNK_BYTES); the state picks the largest that leaves three ring slots */
};

/* A run of one matrix's rows in a CTA's stream. */
struct Seg {
    int rows;    /* rows of this CTA */
    int row0;    /* first output row */
    int rec;     /* bytes per record (a gate|up pair: both records) */
    int rpc;     /* records per chunk */
    int type, d16, bias;
};

struct PhasePlan {
    Seg seg[3];
    int nseg, cols;
    long long bytes;
};

enum { PH_A = 0, PH_C = 1, PH_D = 2, PH_E = 3, PH_F = 4, NPHASE = 5 };
constexpr int CHUNK_BYTES = 56 * 1024;   /* largest bulk copy (at least one record); a state may use smaller ones */
constexpr int GROUP_ROWS = 4;            /* rows per warp task (two gate|up pairs) */
constexpr int OWN_MAX = 128;             /* rows of x a CTA may own */
static_assert((NCW & (NCW - 1)) == 0, "warp round-robin uses a mask");
constexpr int ATT_CNT_STRIDE = 32;       /* words between attention unit counters (one 128-byte line each) */

/* Record bytes: quants, scales, the bias when present, padded to 16. */
__host__ __device__ inline int rec_bytes(int type, int d16, int cols, int bias) {
    const int q = type == T_Q4 ? cols / 2 : cols, d = (cols / QK) * (d16 ? 2 : 4);
    return (q + d + (bias ? 4 : 0) + 15) & ~15;
}

/* Rows [r0, r1) of a `rows`-row matrix owned by CTA j of G. */
__host__ __device__ inline void share_rows(int rows, int j, int G, int &r0, int &r1) {
    r0 = (int)((long long)rows * j / G);
    r1 = (int)((long long)rows * (j + 1) / G);
}

__host__ __device__ inline Seg make_seg(int rows, int row0, int type, int d16, int cols, int bias, int pair, int chunk) {
    Seg s;
    s.rows = rows;
    s.row0 = row0;
    s.type = type;
    s.d16 = d16;
    s.bias = bias;
    s.rec = rec_bytes(type, d16, cols, bias) * (pair ? 2 : 1);
    const int step = pair ? GROUP_ROWS / 2 : GROUP_ROWS;
    int rpc = s.rec > 0 ? chunk / s.rec : 1;
    if (rpc >= step) rpc -= rpc % step;
    s.rpc = rpc < 1 ? 1 : rpc;
    return s;
}

/* The phases of CTA j's stream for one layer (A, C, D, E) and the classifier (F). */
__host__ __device__ inline void make_plan(const StreamGeom &g, int j, int G, PhasePlan *P) {
    int r0, r1;
    const int ch = g.chunk > 0 ? g.chunk : CHUNK_BYTES;
    for (int p = 0; p < NPHASE; p++) {   /* unused segments read as empty */
        P[p].nseg = 0;
        P[p].cols = 0;
        P[p].bytes = 0;
        for (int k = 0; k < 3; k++) P[p].seg[k] = Seg{ 0, 0, 0, 1, T_Q8, 0, 0 };
    }
    PhasePlan &A = P[PH_A];
    A.nseg = 0;
    A.cols = g.dim;
    const int na = g.q_dim + 2 * g.kv_dim;
    share_rows(na, j, G, r0, r1);
    const int lo[3] = { 0, g.q_dim, g.q_dim + g.kv_dim }, hi[3] = { g.q_dim, g.q_dim + g.kv_dim, na };
    const int ty[3] = { g.t_q, g.t_k, g.t_v }, dd[3] = { g.d16_q, g.d16_k, g.d16_v }, bb[3] = { g.b_q, g.b_k, g.b_v };
    for (int m = 0; m < 3; m++) {
        const int s0 = r0 > lo[m] ? r0 : lo[m], s1 = r1 < hi[m] ? r1 : hi[m];
        if (s1 > s0) A.seg[A.nseg++] = make_seg(s1 - s0, s0, ty[m], dd[m], g.dim, bb[m], 0, ch);
    }
    share_rows(g.dim, j, G, r0, r1);
    P[PH_C].nseg = 1;
    P[PH_C].cols = g.q_dim;
    P[PH_C].seg[0] = make_seg(r1 - r0, r0, g.t_o, g.d16_o, g.q_dim, 0, 0, ch);
    P[PH_E].nseg = 1;
    P[PH_E].cols = g.hidden;
    P[PH_E].seg[0] = make_seg(r1 - r0, r0, g.t_down, g.d16_down, g.hidden, 0, 0, ch);
    share_rows(g.hidden / g.d_unit, j, G, r0, r1);   /* whole blocks, or 4-row units of split blocks */
    r0 *= g.d_unit;
    r1 *= g.d_unit;
    P[PH_D].nseg = 1;
    P[PH_D].cols = g.dim;
    P[PH_D].seg[0] = make_seg(r1 - r0, r0, g.t_up, g.d16_up, g.dim, 0, 1, ch);
    share_rows(g.vocab, j, G, r0, r1);
    P[PH_F].nseg = 1;
    P[PH_F].cols = g.dim;
    P[PH_F].seg[0] = make_seg(r1 - r0, r0, g.t_cls, g.d16_cls, g.dim, 0, 0, ch);
    for (int p = 0; p < NPHASE; p++) {
        long long b = 0;
        for (int s = 0; s < P[p].nseg; s++) b += (long long)P[p].seg[s].rows * P[p].seg[s].rec;
        P[p].bytes = b;
    }
}

/* Rows of a phase (its segments are contiguous in the phase's output). */
__host__ __device__ inline int plan_rows(const PhasePlan &P) {
    int n = 0;
    for (int s = 0; s < P.nseg; s++) n += P.seg[s].rows;
    return n;
}

/* Largest chunk of a plan: the ring's slot size. */
__host__ __device__ inline int plan_max_chunk(const PhasePlan *P) {
    int m = 0;
    for (int p = 0; p < NPHASE; p++)
        for (int s = 0; s < P[p].nseg; s++) {
            const Seg &S = P[p].seg[s];
            const int c = (S.rows < S.rpc ? S.rows : S.rpc) * S.rec;
            m = c > m ? c : m;
        }
    return m;
}

struct StepArgs {
    const LayerPlan *layers;        /* device array [n_layers] */
    PMat emb;
    const uint8_t *stream;          /* the weight stream */
    const unsigned long long *cta_base;   /* [G] byte offset of each CTA's stream */
    StreamGeom geom;
    const float *final_norm, *inv0;
    /* the vectors between phases as tagged words (see "tagged words"): x rows
     * after the O and after the down phase [2][dim], the CTAs' sums of squares
     * of their residual rows [2][G], post-norm models' block outputs [2][dim],
     * q|k|v [q_dim + 2 kv_dim], attention split partials
     * [n_heads][nsplit][hd + 2], attention output [q_dim], FFN hidden [hidden] */
    unsigned long long *xw, *sspw, *yw, *qkvw, *partw, *aow, *hbw;
    unsigned tag0;                  /* tag of the launch's first output (tag_of) */
    /* attention split arrivals: a counter per unit of att_unit KV heads (the
     * fewest whose outputs fill whole 32-value blocks), ATT_CNT_STRIDE words
     * apart, zeroed before each launch */
    unsigned *attc;
    int att_unit;
    /* split FFN blocks (geom.d_unit 4): the covering CTAs' partial maxima,
     * tagged words [hidden / 32][8] */
    unsigned long long *amaxw;
    float *logits;
    unsigned *bar, *err;
    LoopState *ls;
    const int *feed;
    int *out_tokens;
    int n_layers, dim, q_dim, kv_dim, hidden, vocab, max_seq, n_heads, n_kv_heads, hd;
    int kv_type;                    /* KC_F32, KC_F16 or KC_Q8_0 */
    float eps, attn_scale, attn_softcap, final_softcap, embed_scale;
    int act, nsplit, nstage, slot_bytes, act_bytes, res_bytes, wbuf_bytes;
    int nsteps, run_cls;            /* steps in this launch; run the classifier */
    unsigned long long *timeline;   /* optional: globaltimer at start and after each barrier (CTA 0) */
    unsigned *timeline_n;
    unsigned timeline_cap;
    unsigned long long *trace;      /* optional: [phase][G][3] per CTA: prologue done, arrived, released */
    unsigned trace_phases;
    /* tensor parallelism: this rank's classifier rows start at cls_row0; with
     * tp_world > 1, tp_box[r] is rank r's exchange buffer (the own one too):
     * partial rows y [2][world][dim] (64-bit words: sequence number | float)
     * at 0, best logit keys [world] at tp_off_best and their flags at
     * tp_off_bflag, the logits ring at tp_off_logits. tp_step0: the steps of
     * earlier launches (sequence numbers grow by one per exchange). */
    int post_norms;
    int cls_row0;
    int tp_rank, tp_world;
    unsigned long long tp_step0;
    unsigned char *tp_box[KC_TP_MAX];
    unsigned long long tp_off_best, tp_off_bflag, tp_off_logits;
};

/* ------------------------------------------------------------ event log (diagnostics) */

/* kc_step_events: per CTA, consumer thread 0 (who 0) and the producer (who 1)
 * append clock64() << 8 | code to their own g_evcap-entry stream. Null (one
 * uniform branch per event) outside that entry point. */
__device__ unsigned long long *g_evlog;
__device__ unsigned g_evcap;
__shared__ unsigned s_evn[2];
__shared__ unsigned long long *s_evp;   /* g_evlog, read once per launch */

/* Before the first event, ahead of a __syncthreads (every kernel that runs the ring). */
__device__ __forceinline__ void ev_init(bool enabled) {
    if (threadIdx.x == 0) {
        s_evn[0] = s_evn[1] = 0;
        s_evp = enabled ? g_evlog : nullptr;
    }
}

enum { EV_PRO_DONE = 2, EV_STAGE_READY = 3, EV_STAGE_DONE = 4, EV_ARRIVE = 5, EV_RELEASE = 6, EV_EMPTY_WAIT = 7,
       EV_ISSUE = 8, EV_ACT_ENTRY = 9, EV_ACT_LOADED = 10, EV_ACT_INV = 11, EV_ACT_QUANT = 12, EV_ATT_PRE = 13,
       EV_ATT_TILE = 14, EV_ATT_PART = 15, EV_ATT_COMBINE = 16, EV_ATT_DONE = 17,
       /* checkpoints inside an attention item */
       EV_ATT_ENTRY = 20, EV_ATT_ISSUED = 21, EV_ATT_QROPE = 22, EV_ATT_STORED = 23, EV_ATT_SYNCED = 24,
       EV_ATT_SCORES = 25, EV_ATT_SOFTMAX = 26, EV_ATT_PARTIAL = 27, EV_ATT_ARRIVED = 28,
       /* tensor parallelism: a residual exchange's stores issued, every rank's words in */
       EV_TP_SENT = 29, EV_TP_DONE = 30 };

__device__ __forceinline__ void ev(int who, unsigned code) {
    unsigned long long *log = s_evp;
    if (log) {
        const unsigned k = s_evn[who]++;
        if (k < g_evcap) log[((size_t)blockIdx.x * 2 + who) * g_evcap + k] = ((unsigned long long)clock64() << 8) | code;
    }
}

/* ------------------------------------------------------------ consumer barrier */

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

/* Float sum over the consumer threads into red[0]. */
__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    consumer_sync();
    if (lane == 0) red[warp] = v;
    consumer_sync();
    if (warp == 0) {
        float t = lane < NCW ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    consumer_sync();
    return red[0];
}

/* ------------------------------------------------------------ grid barrier */

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

/* Per-CTA trace (debug): mark k (0 prologue done, 1 arrived, 2 released) of
 * phase p, by consumer thread 0. */
__device__ __forceinline__ void trace_mark(const StepArgs &a, unsigned p, int k) {
    if (a.trace && threadIdx.x == 0 && p < a.trace_phases) a.trace[((size_t)p * gridDim.x + blockIdx.x) * 3 + k] = gtimer();
}

__device__ __forceinline__ void timeline_mark(const StepArgs &a) {
    if (a.timeline && blockIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        const unsigned k = atomicAdd(a.timeline_n, 1u);
        if (k < a.timeline_cap) a.timeline[k] = t;
    }
}

/* Bounded wait until the arrival counter reaches `target` (one thread). Gives
 * up after ~1 s, or at once when another CTA has flagged the error word. */
__device__ __forceinline__ void wait_count(const StepArgs &a, unsigned target) {
    unsigned it = 0;
    while (ld_acquire(a.bar) < target) {
        if (++it > (1u << 24)) {
            atomicOr(a.err, 4u);
            return;
        }
        if ((it & 1023) == 0 && ld_acquire(a.err)) return;
    }
    timeline_mark(a);
}

/* The end of a phase as this CTA sees it (diagnostics): its trace marks and,
 * on CTA 0, a timeline entry. No barrier: the next phase's prologue waits on
 * the tagged words it reads. */
__device__ __forceinline__ void phase_end(const StepArgs &a, unsigned &pidx) {
    const unsigned p = pidx++;
    if (threadIdx.x == 0) {
        trace_mark(a, p, 1);
        trace_mark(a, p, 2);
        timeline_mark(a);
        ev(0, EV_ARRIVE);
    }
}

/* ------------------------------------------------------------ tagged words */

/* Within a step, the vectors between phases travel as 64-bit words: a 32-bit
 * tag in the high half (the number of the phase output: launch step, layer and
 * kind, see tag_of) and the float in the low half. An aligned 8-byte store is
 * seen whole or not at all, so each word is its own ready flag: a reader loads
 * the words it needs, then loads again those whose tag is not yet the
 * expected one. No fence, counter or grid barrier sits between the phases of
 * a layer; each CTA waits for exactly the words it reads, the moment they
 * land. Words are compared for equality, so tags may wrap.
 *
 * A word is rewritten only after every reader of its previous value is done:
 * x has one buffer for each of the two phases that write it (after O, after
 * down), and every CTA owns rows of x (the grid has at most one CTA per row).
 * A CTA reads a vector in a prologue and writes its own rows of x later in
 * the same layer; every other vector's next write lies behind, in the data
 * flow, a phase that reads all of x, so behind every CTA's reads. */
typedef unsigned long long word_t;
enum { TAG_QKV = 0, TAG_PART = 1, TAG_AO = 2, TAG_XC = 3, TAG_HB = 4, TAG_XE = 5, NTAG = 6 };
constexpr unsigned POLL_LIMIT = 1u << 22;   /* loads of one word before a reader gives up (seconds) */
constexpr unsigned ERR_POLL = 32u;          /* error bit: a tagged input never came */

__device__ __forceinline__ unsigned tag_of(const StepArgs &a, int step, int l, int kind) {
    return a.tag0 + (unsigned)((step * a.n_layers + l) * NTAG + kind);
}
__device__ __forceinline__ word_t mkword(unsigned tag, float v) {
    return ((word_t)tag << 32) | (word_t)__float_as_uint(v);
}
__device__ __forceinline__ float wval(word_t w) { return __uint_as_float((unsigned)w); }
__device__ __forceinline__ bool wok(word_t w, unsigned tag) { return (unsigned)(w >> 32) == tag; }
__device__ __forceinline__ void st_word(word_t *p, word_t w) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ word_t ld_word(const word_t *p) {
    word_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
/* Two words (16-byte aligned); each element is a single-copy atomic 8 bytes. */
__device__ __forceinline__ void ld_words2(const word_t *p, word_t &a, word_t &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
/* Four words in one 256-bit load (32-byte aligned): half the requests of two
 * v2 loads at the L2 slices that every CTA polls at once. */
__device__ __forceinline__ void ld_words4(const word_t *p, word_t &a, word_t &b, word_t &c, word_t &d) {
    asm volatile("ld.relaxed.gpu.global.v4.u64 {%0, %1, %2, %3}, [%4];"
                 : "=l"(a), "=l"(b), "=l"(c), "=l"(d)
                 : "l"(p)
                 : "memory");
}
/* Loads p again until the word carries tag (bounded; gives up at once when
 * another CTA has flagged the error word). */
__device__ __forceinline__ float wait_word(const word_t *p, unsigned tag, word_t w, unsigned *err) {
    for (unsigned it = 0; !wok(w, tag); it++) {
        if (it >= POLL_LIMIT) {
            atomicOr(err, ERR_POLL);
            break;
        }
        if ((it & 63) == 63 && *(volatile const unsigned *)err) break;
        w = ld_word(p);
    }
    return wval(w);
}
__device__ __forceinline__ void wait_words2(const word_t *p, unsigned tag, word_t &a, word_t &b, unsigned *err) {
    for (unsigned it = 0; !(wok(a, tag) && wok(b, tag)); it++) {
        if (it >= POLL_LIMIT) {
            atomicOr(err, ERR_POLL);
            break;
        }
        if ((it & 63) == 63 && *(volatile const unsigned *)err) break;
        ld_words2(p, a, b);
    }
}
/* Waits for one tagged word and returns its float (one load when it has landed). */
__device__ __forceinline__ float get_word(const word_t *p, unsigned tag, unsigned *err) {
    return wait_word(p, tag, ld_word(p), err);
}

/* Quantized vectors between phases (the attention output, the FFN hidden):
 * n values travel as n / 4 words of four int8 quants (elements 4k..4k+3 in
 * word k, in the low half) and then n / 32 words of block scales, all tagged.
 * The producer owns whole 32-value blocks and quantizes them itself, so the
 * consumers' prologue only copies, and reads 2.25 bytes per value instead
 * of 8. */

/* One block of 32 values, one per lane, quantized by the warp with quant4's
 * rule (the same maximum, d, 127 / amax and rounding, so the same bits as
 * quantizing the floats in the consumer) and published as block b of aw
 * (an n-value vector): lane 4k writes quant word k, lane 0 the scale. */
__device__ __forceinline__ void publish_qblock(word_t *aw, int n, int b, unsigned tag, float v) {
    const int lane = threadIdx.x & 31;
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    unsigned q = 0;
    float d = 0.0f;
    if (!(amax < 1e-30f)) {
        const float id = __fdiv_rn(127.0f, amax);
        d = __fdiv_rn(amax, 127.0f);
        float t = truncf(__fadd_rn(__fmul_rn(v, id), copysignf(0.5f, v)));
        t = fminf(fmaxf(t, -127.0f), 127.0f);
        q = ((unsigned)(int)t & 0xffu) << (8 * (lane & 3));
    }
    q |= __shfl_xor_sync(0xffffffffu, q, 1);
    q |= __shfl_xor_sync(0xffffffffu, q, 2);
    if ((lane & 3) == 0) st_word(aw + (size_t)b * 8 + (lane >> 2), mkword(tag, __uint_as_float(q)));
    if (lane == 0) st_word(aw + n / 4 + b, mkword(tag, d));
}

/* ------------------------------------------------------------ tensor parallelism */

constexpr unsigned TP_ERR = 16u;   /* error bit: a rank's partial rows or best key never came */

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
/* Bounded wait (one thread) until *f >= seq; false after ~1 s or when the
 * error word is set. */
__device__ __forceinline__ bool tp_wait(const unsigned *f, unsigned seq, unsigned *err) {
    for (unsigned it = 0; it < (1u << 22); it++) {
        if (ld_acquire_sys(f) >= seq) return true;
        if ((it & 255) == 255 && ld_acquire(err)) return false;
    }
    atomicOr(err, TP_ERR);
    return false;
}
__device__ __forceinline__ unsigned tp_seq(const StepArgs &a, int step, int l, int ph) {
    return (unsigned)((a.tp_step0 + (unsigned long long)step) * (2ull * a.n_layers) + 2ull * l + ph + 1ull);
}

__device__ __forceinline__ void st_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

/* The residual add after a row-parallel projection (O: ph 0, down: ph 1)
 * across ranks. Each partial row travels as one 64-bit word, sequence number
 * in the high half and the float in the low half: an aligned 8-byte store is
 * seen whole or not at all, so the word is its own flag and no fence or
 * barrier sits between the ranks. The thread of row i stores its partial
 * (the row's column slices summed in order) into slot [ph][rank][row] of every
 * rank's exchange buffer, then waits in its own buffer for every rank's word
 * of that row carrying this exchange's number and adds them in rank order:
 * own[row] += y_0 + y_1 + ... Every rank runs the same grid, so CTA j of every
 * rank owns the same rows of x; a rank can store the next exchange's words
 * into a slot only after this rank has passed the exchange in between. */
__device__ __noinline__ void tp_resid(const StepArgs &a, const float *res, int nrows, int row0, float *own, int ns,
                                      int ph, unsigned seq) {
    const int me = a.tp_rank, W = a.tp_world, D = a.dim;
    for (int i = threadIdx.x; i < nrows; i += NCT) {
        float sum = res[i * ns];
        for (int k = 1; k < ns; k++) sum = __fadd_rn(sum, res[i * ns + k]);
        const unsigned long long word = ((unsigned long long)seq << 32) | __float_as_uint(sum);
        for (int r = 0; r < W; r++)
            st_sys_u64((unsigned long long *)a.tp_box[r] + ((size_t)ph * W + me) * D + row0 + i, word);
    }
    if (threadIdx.x == 0) ev(0, EV_TP_SENT);
    const unsigned long long *y = (const unsigned long long *)a.tp_box[me] + (size_t)ph * W * D;
    for (int i = threadIdx.x; i < nrows; i += NCT) {
        float tot = 0.0f;
        for (int r = 0; r < W; r++) {
            const unsigned long long *p = y + (size_t)r * D + row0 + i;
            unsigned long long w = ld_sys_u64(p);
            for (unsigned it = 0; (unsigned)(w >> 32) != seq; it++) {
                if (it > (1u << 22) || ((it & 255) == 255 && ld_acquire(a.err))) {
                    atomicOr(a.err, TP_ERR);
                    break;
                }
                w = ld_sys_u64(p);
            }
            const float v = __uint_as_float((unsigned)w);
            tot = r == 0 ? v : __fadd_rn(tot, v);
        }
        own[i] = __fadd_rn(own[i], tot);
    }
    if (threadIdx.x == 0) ev(0, EV_TP_DONE);
}

/* The rank's best logit key to every rank, then the maximum over ranks (one
 * thread, the CTA that finishes the step). */
__device__ __noinline__ unsigned long long tp_argmax(const StepArgs &a, unsigned long long b, unsigned seq) {
    const int me = a.tp_rank, W = a.tp_world;
    for (int r = 0; r < W; r++) ((unsigned long long *)(a.tp_box[r] + a.tp_off_best))[me] = b;
    __threadfence_system();
    for (int r = 0; r < W; r++) st_release_sys((unsigned *)(a.tp_box[r] + a.tp_off_bflag) + me, seq);
    unsigned long long best = 0;
    for (int r = 0; r < W; r++) {
        tp_wait((const unsigned *)(a.tp_box[me] + a.tp_off_bflag) + r, seq, a.err);
        __threadfence_system();
        const unsigned long long k = __ldcv((const unsigned long long *)(a.tp_box[me] + a.tp_off_best) + r);
        best = k > best ? k : best;
    }
    return best;
}

/* ------------------------------------------------------------ the ring */

struct Ring {
    uint64_t *full, *empty;
    uint8_t *base;
    int nstage, slot_bytes;
    int slot;         /* the next chunk's slot */
    unsigned round;   /* times the ring has wrapped: the slot's use count */
};

/* The next slot, without divisions. */
__device__ __forceinline__ void ring_next(Ring &rg) {
    if (++rg.slot == rg.nstage) {
        rg.slot = 0;
        rg.round++;
    }
}

/* Consumer: waits until the current slot's chunk has landed. A wait that
 * runs out of its `limit` polls flags error bit 2, then waits once more
 * (bounded) for the copy: no slot is handed back to the producer, and no CTA
 * leaves, while a bulk copy into it may still be in flight. */
__device__ __forceinline__ const uint8_t *ring_wait_full(const Ring &rg, unsigned *err, unsigned limit = WAIT_POLLS) {
    if (!mbar_wait(&rg.full[rg.slot], rg.round & 1u, nullptr, limit)) {
        if ((threadIdx.x & 31) == 0) atomicOr(err, 2u);
        mbar_wait(&rg.full[rg.slot], rg.round & 1u);
    }
    return rg.base + (size_t)rg.slot * rg.slot_bytes;
}

/* Consumer: this warp is done with the current slot. */
__device__ __forceinline__ void ring_release(Ring &rg) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&rg.empty[rg.slot]);
    ring_next(rg);
}

/* Producer: waits for the chunk's slot to be free and issues its bulk copy.
 * The wait does not leave early on another CTA's error: every consumer warp
 * hands back every slot (its own waits drain), so the slot is re-armed only
 * after its last chunk was read. */
__device__ __forceinline__ uint8_t *ring_issue(Ring &rg, unsigned bytes, unsigned *err) {
    ev(1, EV_EMPTY_WAIT);
    if (rg.round > 0 && !mbar_wait(&rg.empty[rg.slot], (rg.round - 1) & 1u)) atomicOr(err, 2u);
    mbar_expect_tx(&rg.full[rg.slot], bytes);
    return rg.base + (size_t)rg.slot * rg.slot_bytes;
}

/* Producer: the chunks of one phase of the stream, from src on. */
__device__ __forceinline__ void produce_phase(Ring &rg, const PhasePlan &P, const uint8_t *&src, unsigned *err) {
    for (int s = 0; s < P.nseg; s++) {
        const Seg &S = P.seg[s];
        for (int r = 0; r < S.rows; r += S.rpc) {
            const int n = min(S.rpc, S.rows - r);
            const unsigned bytes = (unsigned)(n * S.rec);
            uint8_t *dst = ring_issue(rg, bytes, err);
            bulk_g2s(dst, src, bytes, &rg.full[rg.slot]);
            src += bytes;
            ev(1, EV_ISSUE);
            ring_next(rg);
        }
    }
}

/* Producer of the kernel-level matvec: rows [r0, r1) of m in the file's
 * layout, a stage holding the quants of R rows then their scales (copied
 * from the 16-byte boundary below them). */
__device__ __forceinline__ void produce_rows(Ring &rg, const PMat &m, int cols, int r0, int r1, unsigned *err) {
    if (r0 >= r1) return;
    int R, qbytes, dbytes;
    stage_geom(m.type, m.d16, cols, 0, R, qbytes, dbytes);
    const int qrow = m.type == T_Q4 ? cols / 2 : cols, drow = (cols / QK) * (m.d16 ? 2 : 4);
    for (int ra = r0; ra < r1; ra += R) {
        const int nr = min(R, r1 - ra);
        const size_t ds = (size_t)ra * drow, de = (size_t)(ra + nr) * drow;
        const size_t das = ds & ~(size_t)15, dae = (de + 15) & ~(size_t)15;
        const unsigned qb = (unsigned)(nr * qrow), db = (unsigned)(dae - das);
        uint8_t *dst = ring_issue(rg, qb + db, err);
        bulk_g2s(dst, m.q + (size_t)ra * qrow, qb, &rg.full[rg.slot]);
        bulk_g2s(dst + qbytes, (const uint8_t *)m.d + das, db, &rg.full[rg.slot]);
        ring_next(rg);
    }
}

/* ------------------------------------------------------------ consumers */

/* The quantized activation in shared memory: elements 0..15 of block b at
 * xlo[b], 16..31 at xhi[b] (16 bytes each, so a warp's loads of consecutive
 * blocks are conflict-free), the block scales and 8 * the sum of each block's
 * quants (the Q4 offset term). */
struct Act {
    const int4 *xlo, *xhi;
    const float *xd;
    const int *xs;
};

struct ActW {
    int8_t *xlo, *xhi;
    float *xd;
    int *xs;
};

__device__ __forceinline__ ActW act_layout(unsigned char *act, int cols) {
    const int nb = cols / QK;
    ActW w;
    w.xlo = (int8_t *)act;
    w.xhi = (int8_t *)act + nb * 16;
    w.xd = (float *)(act + cols);
    w.xs = (int *)(w.xd + nb);
    return w;
}

__device__ __forceinline__ Act act_view(const ActW &w) {
    return Act{ (const int4 *)w.xlo, (const int4 *)w.xhi, w.xd, w.xs };
}

template <bool D16>
__device__ __forceinline__ float sm_scale(const uint8_t *dr, int b) {
    if constexpr (D16) return __half2float(((const __half *)dr)[b]);
    else return ((const float *)dr)[b];
}

/* Sum over the warp of four values at once: returns, on lanes 8q..8q+7, the
 * total of t[q] (two exchange levels, then three butterfly levels). */
__device__ __forceinline__ float reduce4(const float (&t)[4], int lane) {
    const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0;
    float k0 = h16 ? t[2] : t[0], k1 = h16 ? t[3] : t[1];
    const float s0 = h16 ? t[0] : t[2], s1 = h16 ? t[1] : t[3];
    k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
    k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
    float k = h8 ? k1 : k0;
    const float s = h8 ? k0 : k1;
    k += __shfl_xor_sync(0xffffffffu, s, 8);
    k += __shfl_xor_sync(0xffffffffu, k, 4);
    k += __shfl_xor_sync(0xffffffffu, k, 2);
    k += __shfl_xor_sync(0xffffffffu, k, 1);
    return k;
}

/* Row addressing inside a ring slot: row i's quants at q + i*qs, its scales
 * at d + i*ds; with PAIR the second matrix's record p2 bytes further. */
struct Lay {
    int qs, db, ds, p2;
};

/* Dot products of nr (<= NR) rows against the activation, lane b taking
 * blocks b, b+32, ...; each block's int32 sum is exact (dp4a), scaled as
 * (float)s * d_w * d_x and accumulated in block order per lane. Returns
 * reduce4 of the accumulators: {row0, row1, row2, row3}, or with PAIR
 * {gate0, up0, gate1, up1}. */
template <int TYPE, bool D16, bool PAIR>
__device__ __forceinline__ float dot_group(const uint8_t *q, const uint8_t *d, const Lay &L, int b_lo, int b_hi, int nr,
                                           const Act &x, int lane) {
    constexpr int NR = PAIR ? GROUP_ROWS / 2 : GROUP_ROWS;
    constexpr int NA = PAIR ? 2 : 1;
    float acc[NR][NA];
#pragma unroll
    for (int i = 0; i < NR; i++)
#pragma unroll
        for (int k = 0; k < NA; k++) acc[i][k] = 0.0f;
#pragma unroll 1
    for (int b = b_lo + lane; b < b_hi; b += 32) {
        const int4 xl = x.xlo[b], xh = x.xhi[b];
        const float dx = x.xd[b];
        const int corr = TYPE == T_Q4 ? x.xs[b] : 0;
#pragma unroll
        for (int i = 0; i < NR; i++) {
            if (i < nr) {
#pragma unroll
                for (int k = 0; k < NA; k++) {
                    const uint8_t *qr = q + i * L.qs + k * L.p2, *dr = d + i * L.ds + k * L.p2;
                    int s;
                    if constexpr (TYPE == T_Q4) {
                        s = dot_q4(*(const uint4 *)(qr + 16 * b), xl, xh) - corr;
                    } else {
                        s = dot_q8(*(const uint4 *)(qr + 32 * b), xl) + dot_q8(*(const uint4 *)(qr + 32 * b + 16), xh);
                    }
                    acc[i][k] += __fmul_rn((float)s, sm_scale<D16>(dr, b)) * dx;
                }
            }
        }
    }
    float t[4];
    if constexpr (PAIR) {
        t[0] = acc[0][0];
        t[1] = acc[0][NA - 1];
        t[2] = acc[NR - 1][0];
        t[3] = acc[NR - 1][NA - 1];
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) t[i] = acc[i < NR ? i : NR - 1][0];
    }
    return reduce4(t, lane);
}

/* Column slices of a long row: each slice (a block range) is a task of its
 * own, so that a few long rows still keep every warp busy; the slices' partial
 * sums are added in slice order by the finish pass. 1, 2 or 4. */
__host__ __device__ inline int col_slices(int nb, bool pair) {
    return pair || nb < 128 ? 1 : (nb < 256 ? 2 : 4);
}

/* The rows [0, n) of one ring slot, in tasks of GROUP_ROWS rows (or pairs)
 * times ns column slices, dealt to the warps round-robin by the task's index
 * in the phase (g0 + k), so the warps stay evenly loaded across chunks.
 * Results go to res[(i0 + i) * ns + slice] (the record's bias added by slice
 * 0; pairs: res2[i0 + i] = {gate, up}); with res null, single rows are stored
 * straight to out[i0 + i] (ns 1). */
template <int TYPE, bool D16, bool PAIR>
__device__ __forceinline__ void consume_chunk(const uint8_t *slot, const Lay &L, int n, int nb, int ns, int boff, int g0,
                                              int i0, const Act &x, float *res, float *out, int lane, int warp) {
    constexpr int NR = PAIR ? GROUP_ROWS / 2 : GROUP_ROWS;
    const int ng = (n + NR - 1) / NR, lg = ns == 4 ? 2 : (ns == 2 ? 1 : 0);
    for (int k = (warp - g0) & (NCW - 1); k < (ng << lg); k += NCW) {
        const int sl = k & (ns - 1), r = (k >> lg) * NR, nr = min(NR, n - r);
        const uint8_t *q = slot + r * L.qs, *d = slot + L.db + r * L.ds;
        float v = dot_group<TYPE, D16, PAIR>(q, d, L, (sl * nb) >> lg, ((sl + 1) * nb) >> lg, nr, x, lane);
        if constexpr (PAIR) {
            const float u = __shfl_down_sync(0xffffffffu, v, 8);
            const int i = lane >> 4;
            if ((lane & 15) == 0 && i < nr) ((float2 *)res)[i0 + r + i] = make_float2(v, u);
        } else {
            const int i = lane >> 3;
            if ((lane & 7) == 0 && i < nr) {
                if (boff >= 0 && sl == 0) v = __fadd_rn(v, *(const float *)(q + i * L.qs + boff));
                if (res) res[(i0 + r + i) * ns + sl] = v;
                else out[i0 + r + i] = v;
            }
        }
    }
}

/* Consumer side of one segment of the stream, chunk by chunk from the ring;
 * seg_off: the segment's first row within the phase. */
template <int TYPE, bool D16, bool PAIR>
__device__ __forceinline__ void consume_seg(Ring &rg, Seg S, int seg_off, int cols, const Act &x, float *res,
                                            unsigned *err) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nb = cols / QK;
    const int qrow = TYPE == T_Q4 ? cols / 2 : cols;
    const Lay L{ S.rec, qrow, S.rec, S.rec / 2 };
    const int boff = S.bias ? qrow + nb * (D16 ? 2 : 4) : -1;
    const int ns = col_slices(nb, PAIR);
    constexpr int NR = PAIR ? GROUP_ROWS / 2 : GROUP_ROWS;
    for (int r = 0; r < S.rows; r += S.rpc) {
        const int n = min(S.rpc, S.rows - r);
        const uint8_t *slot = ring_wait_full(rg, err);
        if (threadIdx.x == 0) ev(0, EV_STAGE_READY);
        consume_chunk<TYPE, D16, PAIR>(slot, L, n, nb, ns, boff, ((seg_off + r) / NR) * ns, seg_off + r, x, res,
                                       nullptr, lane, warp);
        if (threadIdx.x == 0) ev(0, EV_STAGE_DONE);
        ring_release(rg);
    }
}

/* All segments of a phase into res (one inlined copy of each consumer loop:
 * Q4/Q8, single rows or gate|up pairs, in the stream's scale type D16), then
 * a consumer barrier. */
template <bool D16>
__device__ __forceinline__ void consume_phase(Ring &rg, const PhasePlan &P, bool pair, const Act &x, float *res,
                                              unsigned *err) {
    int off = 0;
    for (int s = 0; s < P.nseg; s++) {
        const Seg S = P.seg[s];
        switch ((S.type == T_Q4 ? 2 : 0) + (pair ? 1 : 0)) {
        case 3: consume_seg<T_Q4, D16, true>(rg, S, off, P.cols, x, res, err); break;
        case 2: consume_seg<T_Q4, D16, false>(rg, S, off, P.cols, x, res, err); break;
        case 1: consume_seg<T_Q8, D16, true>(rg, S, off, P.cols, x, res, err); break;
        default: consume_seg<T_Q8, D16, false>(rg, S, off, P.cols, x, res, err); break;
        }
        off += S.rows;
    }
    consumer_sync();
}

enum { FIN_STORE = 0, FIN_RESID = 1, FIN_LOGITS = 3 };

/* The rows of a phase after its dot products (res, in row order from row0):
 * store or residual add (on the CTA's rows of x in `own`), each result as a
 * tagged word into wout, or logits into out with the first-index argmax key
 * of the CTA's rows (returned on thread 0; 0 otherwise). */
__device__ __forceinline__ unsigned long long finish_phase(int kind, const float *res, int nrows, int row0, float *out,
                                                        word_t *wout, unsigned tag, float *own, int act, float softcap,
                                                        unsigned long long *cta_best, int ns) {
    unsigned long long best = 0;
    for (int i = threadIdx.x; i < nrows; i += NCT) {
        const int row = row0 + i;
        float sum = res[i * ns];
        for (int k = 1; k < ns; k++) sum = __fadd_rn(sum, res[i * ns + k]);
        if (kind == FIN_STORE) {
            st_word(wout + row, mkword(tag, sum));
        } else if (kind == FIN_RESID) {
            const float v = __fadd_rn(own[i], sum);
            own[i] = v;
            st_word(wout + row, mkword(tag, v));
        } else {
            float v = sum;
            if (softcap > 0.0f) v = __fmul_rn(softcap, tanhf(__fdiv_rn(v, softcap)));
            out[row] = v;
            const unsigned long long k = argmax_key(v, row);
            best = k > best ? k : best;
        }
    }
    if (kind == FIN_LOGITS) {
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if ((threadIdx.x & 31) == 0) cta_best[threadIdx.x >> 5] = best;
        consumer_sync();
        best = 0;
        if (threadIdx.x == 0)
            for (int w = 0; w < NCW; w++) best = cta_best[w] > best ? cta_best[w] : best;
    }
    return best;
}

/* The gate|up phase's finish: h = act(g) * u on the CTA's rows (whole blocks
 * from row0), a block per warp quantized and published into hw (an n-value
 * vector, publish_qblock). */
__device__ __forceinline__ void finish_pair_q(const float *res, int nrows, int row0, word_t *hw, int n, unsigned tag,
                                              int act) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int b = warp; b < nrows / QK; b += NCW) {
        const float2 gu = ((const float2 *)res)[b * QK + lane];
        publish_qblock(hw, n, row0 / QK + b, tag, act_mul(act, gu.x, gu.y));
    }
}

/* Owner of unit u of U units shared by G CTAs (share_rows' inverse). */
__device__ __forceinline__ int unit_owner(int u, int U, int G) { return (int)(((long long)(u + 1) * G - 1) / U); }

/* The gate|up phase's finish when its rows are shared in 4-row units (U of
 * them) and blocks of the hidden vector are split between CTAs: every covering
 * CTA publishes its rows' |max| of each split block (slot: its first unit's
 * offset in the block), then, with every partial it owns published, waits for
 * the other covering CTAs' and quantizes its own rows with the block's maximum
 * (the max of the partials is exact, so the quants and scale are those of the
 * whole block); the block's first CTA writes the scale. Whole blocks as
 * finish_pair_q. Out of line: inlined, its code slowed the models that never
 * take it (cfg1 2.5%). */
__device__ __noinline__ void finish_pair_split(const float *res, int nrows, int row0, word_t *hw, int n, unsigned tag,
                                               int act, word_t *amaxw, int U, unsigned *err) {
    if (nrows <= 0) return;
    constexpr int UPB = QK / 4;   /* units per block */
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, G = gridDim.x, j = blockIdx.x;
    const int b0 = row0 / QK, b1 = (row0 + nrows - 1) / QK;
    auto value = [&](int bi) {
        const int row = bi * QK + lane;
        if (row < row0 || row >= row0 + nrows) return 0.0f;
        const float2 gu = ((const float2 *)res)[row - row0];
        return act_mul(act, gu.x, gu.y);
    };
    auto wmax = [&](float m) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        return m;
    };
    const int my_slot_first = (row0 / 4) % UPB;   /* my first unit's offset in block b0 */
    /* first every partial of a split block */
    for (int bi = b0 + warp; bi <= b1; bi += NCW) {
        const bool whole = unit_owner(bi * UPB, U, G) == j && unit_owner(bi * UPB + UPB - 1, U, G) == j;
        const float m = wmax(fabsf(value(bi)));
        if (!whole && lane == 0) st_word(amaxw + (size_t)bi * UPB + (bi == b0 ? my_slot_first : 0), mkword(tag, m));
    }
    for (int bi = b0 + warp; bi <= b1; bi += NCW) {
        const float v = value(bi);
        float amax = wmax(fabsf(v));
        const int o0 = unit_owner(bi * UPB, U, G);
        if (!(o0 == j && unit_owner(bi * UPB + UPB - 1, U, G) == j)) {
            /* lane k < 8: the CTA whose first unit in the block is unit k, when it is another CTA */
            float other = 0.0f;
            if (lane < UPB) {
                const int ok = unit_owner(bi * UPB + lane, U, G);
                const bool start = lane == 0 || unit_owner(bi * UPB + lane - 1, U, G) != ok;
                if (start && ok != j) other = get_word(amaxw + (size_t)bi * UPB + lane, tag, err);
            }
            amax = fmaxf(amax, wmax(other));
        }
        unsigned q = 0;
        float d = 0.0f;
        if (!(amax < 1e-30f)) {
            const float id = __fdiv_rn(127.0f, amax);
            d = __fdiv_rn(amax, 127.0f);
            float t = truncf(__fadd_rn(__fmul_rn(v, id), copysignf(0.5f, v)));
            t = fminf(fmaxf(t, -127.0f), 127.0f);
            q = ((unsigned)(int)t & 0xffu) << (8 * (lane & 3));
        }
        q |= __shfl_xor_sync(0xffffffffu, q, 1);
        q |= __shfl_xor_sync(0xffffffffu, q, 2);
        const int row = bi * QK + lane;
        if ((lane & 3) == 0 && row >= row0 && row < row0 + nrows)
            st_word(hw + (size_t)bi * 8 + (lane >> 2), mkword(tag, __uint_as_float(q)));
        if (lane == 0 && o0 == j) st_word(hw + n / 4 + bi, mkword(tag, d));
    }
}

/* This CTA's rows of x (own, from row0) as tagged words (after a residual
 * phase that wrote own without them: tensor parallelism, post-norms). */
__device__ __forceinline__ void publish_rows(word_t *w, unsigned tag, const float *own, int nrows, int row0) {
    for (int i = threadIdx.x; i < nrows; i += NCT) st_word(w + row0 + i, mkword(tag, own[i]));
}

/* After a residual phase, the CTA's sum of squares of its n rows (of x, or of
 * a post-norm model's block output) into its tagged word: every CTA
 * publishes one, rows or none (the next RMSNorm adds all G of them). */
__device__ __forceinline__ void publish_ssp(word_t *sspw, unsigned tag, const float *rows, int n) {
    consumer_sync();
    if (threadIdx.x < 32) {
        float t = 0.0f;
        for (int i = threadIdx.x; i < n; i += 32) t += rows[i] * rows[i];
        t = warp_sum(t);
        if (threadIdx.x == 0) st_word(sspw + blockIdx.x, mkword(tag, t));
    }
}

/* The residual add of a phase whose CTA rows fit one warp (n <= 32): lane i
 * sums row i's column slices in order, adds it to own[i] and publishes the
 * row, with no CTA barrier in between. */
__device__ __forceinline__ void finish_resid_warp(const float *res, int n, int row0, word_t *xw, unsigned tag,
                                                  float *own, int ns) {
    const int i = threadIdx.x;
    if (i < n) {
        float sum = res[i * ns];
        for (int k = 1; k < ns; k++) sum = __fadd_rn(sum, res[i * ns + k]);
        const float v = __fadd_rn(own[i], sum);
        own[i] = v;
        st_word(xw + row0 + i, mkword(tag, v));
    }
}

/* Consumer of the kernel-level matvec (rows [r0, r1) as produce_rows staged them). */
template <int TYPE, bool D16>
__device__ void consume_rows(Ring &rg, int cols, int r0, int r1, float *y, const Act &x, unsigned *err,
                             unsigned limit) {
    if (r0 >= r1) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nb = cols / QK;
    const int qrow = TYPE == T_Q4 ? cols / 2 : cols, drow = nb * (D16 ? 2 : 4);
    int R, qbytes, dbytes;
    stage_geom(TYPE, D16, cols, 0, R, qbytes, dbytes);
    for (int ra = r0; ra < r1; ra += R) {
        const int nr = min(R, r1 - ra);
        const uint8_t *slot = ring_wait_full(rg, err, limit);
        const Lay L{ qrow, qbytes + (int)(((size_t)ra * drow) & 15), drow, 0 };
        consume_chunk<TYPE, D16, false>(slot, L, nr, nb, 1, -1, (ra - r0) / GROUP_ROWS, ra, x, nullptr, y, lane, warp);
        ring_release(rg);
    }
}

/* ------------------------------------------------------------ activations */

/* Value i..i+3 of the embedding row of tok, dequantized (core/quant_ref.c:4-19)
 * and times embed_scale (model/transformer.c:226-230). */
__device__ __forceinline__ float4 embed4(const PMat &emb, float embed_scale, int tok, int cols, int i) {
    const int nb = cols / QK, b = i / QK, j = i % QK;
    const float sc = emb.d16 ? __half2float(((const __half *)emb.d)[(size_t)tok * nb + b])
                               : ((const float *)emb.d)[(size_t)tok * nb + b];
    float v[4];
    if (emb.type == T_Q8) {
        const char4 q4 = *(const char4 *)((const int8_t *)emb.q + (size_t)tok * cols + i);
        v[0] = __fmul_rn((float)q4.x, sc); v[1] = __fmul_rn((float)q4.y, sc);
        v[2] = __fmul_rn((float)q4.z, sc); v[3] = __fmul_rn((float)q4.w, sc);
    } else {
        const uchar4 p = *(const uchar4 *)(emb.q + ((size_t)tok * nb + b) * (QK / 2) + (j & 15));
        const bool hi = j >= 16;
        v[0] = __fmul_rn((float)((hi ? p.x >> 4 : p.x & 15) - 8), sc);
        v[1] = __fmul_rn((float)((hi ? p.y >> 4 : p.y & 15) - 8), sc);
        v[2] = __fmul_rn((float)((hi ? p.z >> 4 : p.z & 15) - 8), sc);
        v[3] = __fmul_rn((float)((hi ? p.w >> 4 : p.w & 15) - 8), sc);
    }
    if (embed_scale != 1.0f)
        for (int k = 0; k < 4; k++) v[k] = __fmul_rn(v[k], embed_scale);
    return make_float4(v[0], v[1], v[2], v[3]);
}

/* Value i of the embedding row of tok (any i). */
__device__ __forceinline__ float embed1(const StepArgs &a, int tok, int cols, int i) {
    const int nb = cols / QK, b = i / QK, j = i % QK;
    const float sc = a.emb.d16 ? __half2float(((const __half *)a.emb.d)[(size_t)tok * nb + b])
                               : ((const float *)a.emb.d)[(size_t)tok * nb + b];
    int v;
    if (a.emb.type == T_Q8) {
        v = ((const int8_t *)a.emb.q)[(size_t)tok * cols + i];
    } else {
        const uint8_t byte = a.emb.q[((size_t)tok * nb + b) * (QK / 2) + (j & 15)];
        v = (j < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
    }
    float o = __fmul_rn((float)v, sc);
    if (a.embed_scale != 1.0f) o = __fmul_rn(o, a.embed_scale);
    return o;
}

/* The activation of a phase into shared memory: quantize_q8 of v, with
 * v = RMSNorm(x) * w (k_scalar.c:59-64: o = (x * inv) * w, inv =
 * 1 / sqrt(ss / n + eps)) when norm_w is set. Source: a float vector in global
 * memory written by other CTAs (read through L2) or the embedding row of tok.
 * 1/rms: inv_given when > 0, else from ss = the sum of the G per-CTA partial
 * sums ssp, else reduced here. Every thread issues all its loads before it
 * uses any, so a prologue costs one round trip to L2. */
constexpr int ACT_PASSES = 4;   /* float4 loads a thread holds in registers: 4096 columns at most */

/* Starts copying the norm weights that this thread's act_float slots read
 * into wbuf (asynchronous, no wait): issued before a grid barrier, the copy
 * overlaps the wait instead of adding a round trip after it. */
__device__ __forceinline__ void prefetch_norm(float *wbuf, const float *nw, int cols) {
    const int nb = cols / QK, tid = threadIdx.x, j0 = (tid & 3) * 8;
    if (!nw) return;
#pragma unroll
    for (int p = 0; p < ACT_PASSES / 2; p++) {
        const int b = p * (NCT / 4) + (tid >> 2);
        if (b < nb) {
            cp_async16(wbuf + b * QK + j0, nw + b * QK + j0);
            cp_async16(wbuf + b * QK + j0 + 4, nw + b * QK + j0 + 4);
        }
    }
    cp_async_commit();
}

/* Quantizes the 4 values of block b held by this lane (elements j0..j0+3)
 * with the other 7 lanes of its group and stores them in the split layout. */
__device__ __forceinline__ void put_quant(const ActW &o, int b, int nb, int j0, float u[4]) {
    float d;
    int sum;
    const unsigned word = quant4(u, &d, &sum);
    if (b < nb) {
        *(unsigned *)((j0 < 16 ? o.xlo : o.xhi) + b * 16 + (j0 & 15)) = word;
        if ((threadIdx.x & 7) == 0) {
            o.xd[b] = d;
            o.xs[b] = 8 * sum;
        }
    }
}

/* The activation of a phase into shared memory: quantize_q8 of v, with
 * v = RMSNorm(x) * w (k_scalar.c:59-64: o = (x * inv) * w, inv =
 * 1 / sqrt(ss / n + eps)) when norm_w is set; x arrives as tagged words from
 * the CTAs that wrote it (tag: the phase output read), and every CTA reduces
 * ss from the whole vector it loads, in the same order. Every thread issues
 * all its loads (up to 2 passes of 64 blocks, 4 lanes per block, 8 values per
 * lane) before it waits on any, so the prologue costs one round trip to L2
 * once its input has landed. */
__device__ __forceinline__ void act_float(float eps, const word_t *xw, unsigned tag, const float *norm_w, int cols,
                                       ActW o, float *red, const float *wstaged, unsigned *err) {
    /* 4 lanes per block, 8 values per lane (four word pairs), passes of NCT / 4 blocks */
    const int nb = cols / QK, tid = threadIdx.x, j0 = (tid & 3) * 8;
    const int passes = (nb + NCT / 4 - 1) / (NCT / 4);
    const bool norm = norm_w != nullptr;
    if (tid == 0) ev(0, EV_ACT_ENTRY);
    constexpr int NP = ACT_PASSES / 2;   /* passes of NCT / 4 blocks */
    bool live[NP];
    const word_t *src[NP];
#pragma unroll
    for (int p = 0; p < NP; p++) {
        const int b = p * (NCT / 4) + (tid >> 2);
        live[p] = p < passes && b < nb;
        src[p] = xw + b * QK + j0;
    }
    /* every word this thread reads, requested together; then, in one loop,
     * the stale ones again until all carry the tag */
    word_t v[NP][8];
    bool fresh = false;
    for (unsigned it = 0;; it++) {
#pragma unroll
        for (int p = 0; p < NP; p++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                word_t *q = &v[p][4 * h];
                if (!live[p]) {
                    q[0] = q[1] = q[2] = q[3] = mkword(tag, 0.0f);
                } else if (it == 0 || !(wok(q[0], tag) && wok(q[1], tag) && wok(q[2], tag) && wok(q[3], tag))) {
                    ld_words4(src[p] + 4 * h, q[0], q[1], q[2], q[3]);
                }
            }
        fresh = true;
#pragma unroll
        for (int p = 0; p < NP; p++)
#pragma unroll
            for (int k = 0; k < 8; k++) fresh = fresh && wok(v[p][k], tag);
        if (fresh) break;
        if (it >= POLL_LIMIT) {
            atomicOr(err, ERR_POLL);
            break;
        }
        if ((it & 63) == 63 && *(volatile const unsigned *)err) break;
    }
    if (tid == 0) ev(0, EV_ACT_LOADED);
    /* the norm weights: staged in shared memory by prefetch_norm (this
     * thread's own copies), read where they are used */
    if (norm && wstaged) cp_async_wait_all();
    const float *wsrc = wstaged ? wstaged : norm_w;
    float inv = 1.0f;
    if (norm) {
        float t = 0.0f;
#pragma unroll
        for (int p = 0; p < NP; p++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const float a0 = wval(v[p][4 * h]), a1 = wval(v[p][4 * h + 1]), a2 = wval(v[p][4 * h + 2]),
                            a3 = wval(v[p][4 * h + 3]);
                t += a0 * a0 + a1 * a1 + a2 * a2 + a3 * a3;
            }
        const float ss = block_sum(t, red);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), eps)));
    }
    if (tid == 0) ev(0, EV_ACT_INV);
    /* the passes in one copy of the code: the second pass's values move into
     * the first's registers at the end of each round */
    int b = tid >> 2;
#pragma unroll 1
    for (int p = 0; p < passes; p++, b += NCT / 4) {
        float u[8];
#pragma unroll
        for (int k = 0; k < 8; k++) u[k] = wval(v[0][k]);
        if (norm && b < nb) {
            const float4 w0 = *(const float4 *)(wsrc + b * QK + j0), w1 = *(const float4 *)(wsrc + b * QK + j0 + 4);
            const float wv[8] = { w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w };
#pragma unroll
            for (int i = 0; i < 8; i++) u[i] = __fmul_rn(__fmul_rn(u[i], inv), wv[i]);
        }
        float d;
        int sum;
        const uint2 word = quant8(u, &d, &sum);
        if (b < nb) {
            *(uint2 *)((j0 < 16 ? o.xlo : o.xhi) + b * 16 + (j0 & 15)) = word;
            if ((tid & 3) == 0) {
                o.xd[b] = d;
                o.xs[b] = 8 * sum;
            }
        }
#pragma unroll
        for (int q = 0; q + 1 < NP; q++)
#pragma unroll
            for (int k = 0; k < 8; k++) v[q][k] = v[q + 1][k];
    }
    if (tid == 0) ev(0, EV_ACT_QUANT);
    consumer_sync();
}

/* Layer 0's activation: the embedding row of tok, its 1/rms from the host
 * table (inv), times the norm weights. Out of line: it runs once a step, and
 * inlined its code slowed every layer (cfg1 2.3%). */
__device__ __noinline__ void act_embed(PMat emb, float embed_scale, int tok, const float *norm_w, float inv, int cols,
                                       ActW o) {
    const int nb = cols / QK, tid = threadIdx.x, j0 = (tid & 7) * 4;
#pragma unroll 1
    for (int b0 = 0; b0 < nb; b0 += NCT / 8) {
        const int b = b0 + (tid >> 3);
        float u[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
        if (b < nb) {
            const float4 e4 = embed4(emb, embed_scale, tok, cols, b * QK + j0);
            const float4 w4 = *(const float4 *)(norm_w + b * QK + j0);
            u[0] = __fmul_rn(__fmul_rn(e4.x, inv), w4.x);
            u[1] = __fmul_rn(__fmul_rn(e4.y, inv), w4.y);
            u[2] = __fmul_rn(__fmul_rn(e4.z, inv), w4.z);
            u[3] = __fmul_rn(__fmul_rn(e4.w, inv), w4.w);
        }
        put_quant(o, b, nb, j0, u);
    }
    consumer_sync();
}

/* The same activation for any width, pass by pass (kernel-level entry points). */
__device__ __noinline__ void act_loop(float eps, const float *x, const float *norm_w, int cols, ActW o, float *red) {
    const int nb = cols / QK, tid = threadIdx.x, j0 = (tid & 7) * 4;
    float inv = 1.0f;
    if (norm_w) {
        float t = 0.0f;
        for (int i = tid * 4; i < cols; i += NCT * 4) {
            const float4 v = __ldcg((const float4 *)(x + i));
            t += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        const float ss = block_sum(t, red);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), eps)));
    }
    for (int b0 = 0; b0 < nb; b0 += NCT / 8) {
        const int b = b0 + (tid >> 3);
        float u[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
        if (b < nb) {
            const float4 v = __ldcg((const float4 *)(x + b * QK + j0));
            u[0] = v.x; u[1] = v.y; u[2] = v.z; u[3] = v.w;
            if (norm_w) {
                const float4 w = *(const float4 *)(norm_w + b * QK + j0);
                u[0] = __fmul_rn(__fmul_rn(u[0], inv), w.x);
                u[1] = __fmul_rn(__fmul_rn(u[1], inv), w.y);
                u[2] = __fmul_rn(__fmul_rn(u[2], inv), w.z);
                u[3] = __fmul_rn(__fmul_rn(u[3], inv), w.w);
            }
        }
        put_quant(o, b, nb, j0, u);
    }
    consumer_sync();
}

/* act_loop over tagged words: wider vectors in the step kernel, pass by pass. */
__device__ __forceinline__ void act_loop_w(float eps, const word_t *xw, unsigned tag, const float *norm_w, int cols,
                                        ActW o, float *red, unsigned *err) {
    const int nb = cols / QK, tid = threadIdx.x, j0 = (tid & 7) * 4;
    float inv = 1.0f;
    if (norm_w) {
        /* the sum of squares from x itself (a first pass over the words) */
        float t = 0.0f;
        for (int i = tid; i < cols; i += NCT) {
            const float v = get_word(xw + i, tag, err);
            t += v * v;
        }
        const float ss = block_sum(t, red);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), eps)));
    }
    for (int b0 = 0; b0 < nb; b0 += NCT / 8) {
        const int b = b0 + (tid >> 3);
        float u[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
        if (b < nb) {
            word_t w0, w1, w2, w3;
            const word_t *p = xw + b * QK + j0;
            ld_words2(p, w0, w1);
            ld_words2(p + 2, w2, w3);
            wait_words2(p, tag, w0, w1, err);
            wait_words2(p + 2, tag, w2, w3, err);
            u[0] = wval(w0); u[1] = wval(w1); u[2] = wval(w2); u[3] = wval(w3);
            if (norm_w) {
                const float4 w = *(const float4 *)(norm_w + b * QK + j0);
                u[0] = __fmul_rn(__fmul_rn(u[0], inv), w.x);
                u[1] = __fmul_rn(__fmul_rn(u[1], inv), w.y);
                u[2] = __fmul_rn(__fmul_rn(u[2], inv), w.z);
                u[3] = __fmul_rn(__fmul_rn(u[3], inv), w.w);
            }
        }
        put_quant(o, b, nb, j0, u);
    }
    consumer_sync();
}

/* Post-norm models (model/transformer.c:238-243): the residual stream after a
 * block is x + RMSNorm(y) * pw, y the block's output (its sum of squares from
 * the G per-CTA partials ssw), all three tagged words of the block's phase.
 * Every CTA recomputes it for all cols, adds up its squares and quantizes
 * RMSNorm(x_new) * nw into the activation; the CTA's own rows of x_new go to
 * own (and out as words one phase later, with the next block's output). */
__device__ __noinline__ void act_postnorm(const StepArgs &a, const word_t *x, const word_t *y, const word_t *ssw,
                                          unsigned tag, const float *pw, const float *nw, int cols, ActW o, float *red,
                                          float *own, int own0, int own1) {
    const int nb = cols / QK, tid = threadIdx.x, j0 = (tid & 7) * 4;
    float t = 0.0f;
    for (int g = tid; g < (int)gridDim.x; g += NCT) t += get_word(ssw + g, tag, a.err);
    const float ssy = block_sum(t, red);
    const float invy = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssy, (float)cols), a.eps)));
    auto xn = [&](int i) {
        return __fadd_rn(get_word(x + i, tag, a.err), __fmul_rn(__fmul_rn(get_word(y + i, tag, a.err), invy), pw[i]));
    };
    float s2 = 0.0f;
    for (int i = tid; i < cols; i += NCT) {
        const float v = xn(i);
        s2 += v * v;
    }
    const float ssx = block_sum(s2, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssx, (float)cols), a.eps)));
    for (int r = own0 + tid; r < own1; r += NCT) own[r - own0] = xn(r);
    for (int b0 = 0; b0 < nb; b0 += NCT / 8) {
        const int b = b0 + (tid >> 3);
        float u[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
        if (b < nb)
            for (int k = 0; k < 4; k++) {
                const int i = b * QK + j0 + k;
                u[k] = __fmul_rn(__fmul_rn(xn(i), inv), nw[i]);
            }
        put_quant(o, b, nb, j0, u);
    }
    consumer_sync();
}

/* The finish of a post-norm model's O or down projection: the block output
 * rows (column slices summed in order) into yown and out as words (yw), and
 * the CTA's rows of the residual stream the last prologue computed (own) as
 * words (xw), with the same tag. */
__device__ __noinline__ void finish_post(const float *res, int nrows, int row0, int ns, word_t *xw, word_t *yw,
                                         unsigned tag, const float *own, float *yown) {
    for (int i = threadIdx.x; i < nrows; i += NCT) {
        float sum = res[i * ns];
        for (int k = 1; k < ns; k++) sum = __fadd_rn(sum, res[i * ns + k]);
        yown[i] = sum;
        st_word(yw + row0 + i, mkword(tag, sum));
        st_word(xw + row0 + i, mkword(tag, own[i]));
    }
}

/* act_float for up to 2 * 2048 columns; wider vectors pass by pass. x: the
 * phase output's tagged words; wstaged: norm_w already copied into shared
 * memory by prefetch_norm. */
__device__ __forceinline__ void load_activation(const StepArgs &a, const word_t *x, unsigned tag, const float *norm_w,
                                                int cols, const ActW &o, float *red, const float *wstaged = nullptr) {
    if (cols <= ACT_PASSES * NCT / 8 * QK) act_float(a.eps, x, tag, norm_w, cols, o, red, wstaged, a.err);
    else act_loop_w(a.eps, x, tag, norm_w, cols, o, red, a.err);
}

/* The activation of a phase whose input arrives quantized (publish_qblock
 * words of a cols-value vector): quants and scales into the split layout and
 * 8 * each block's quant sum (the Q4 offset term). Thread t takes blocks t,
 * t + NCT, ...: a block's nine words are requested together, then the stale
 * ones again until all carry the tag. */
__device__ __forceinline__ void act_qwords(const word_t *aw, unsigned tag, int cols, const ActW &o, unsigned *err) {
    const int nb = cols / QK, tid = threadIdx.x;
    if (tid == 0) ev(0, EV_ACT_ENTRY);
#pragma unroll 1
    for (int b = tid; b < nb; b += NCT) {
        word_t w[9];
        const word_t *q = aw + (size_t)b * 8;
        for (unsigned it = 0;; it++) {
#pragma unroll
            for (int h = 0; h < 2; h++)
                if (it == 0 || !(wok(w[4 * h], tag) && wok(w[4 * h + 1], tag) && wok(w[4 * h + 2], tag) &&
                                 wok(w[4 * h + 3], tag)))
                    ld_words4(q + 4 * h, w[4 * h], w[4 * h + 1], w[4 * h + 2], w[4 * h + 3]);
            if (it == 0 || !wok(w[8], tag)) w[8] = ld_word(aw + cols / 4 + b);
            bool fresh = true;
#pragma unroll
            for (int i = 0; i < 9; i++) fresh = fresh && wok(w[i], tag);
            if (fresh) break;
            if (it >= POLL_LIMIT) {
                atomicOr(err, ERR_POLL);
                break;
            }
            if ((it & 63) == 63 && *(volatile const unsigned *)err) break;
        }
        int sum = 0;
        unsigned u[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            u[i] = (unsigned)w[i];
            sum = __dp4a((int)u[i], 0x01010101, sum);
        }
        *(uint4 *)(o.xlo + b * 16) = make_uint4(u[0], u[1], u[2], u[3]);
        *(uint4 *)(o.xhi + b * 16) = make_uint4(u[4], u[5], u[6], u[7]);
        o.xd[b] = wval(w[8]);
        o.xs[b] = 8 * sum;
    }
    if (tid == 0) ev(0, EV_ACT_QUANT);
    consumer_sync();
}

/* An already quantized activation (kernel-level matvec) into the same layout. */
__device__ void act_prequant(const int8_t *pq, const float *pd, int cols, const ActW &o) {
    const int nb = cols / QK;
    for (int i = threadIdx.x; i < cols / 16; i += NCT)
        ((int4 *)((i & 1) ? o.xhi : o.xlo))[i >> 1] = __ldcg((const int4 *)pq + i);
    for (int b = threadIdx.x; b < nb; b += NCT) o.xd[b] = __ldcg(pd + b);
    consumer_sync();
    for (int b = threadIdx.x; b < nb; b += NCT) {
        int sum = 0;
        const int4 lo = ((const int4 *)o.xlo)[b], hi = ((const int4 *)o.xhi)[b];
        for (const int4 &w : { lo, hi }) {
            sum = __dp4a(w.x, 0x01010101, sum);
            sum = __dp4a(w.y, 0x01010101, sum);
            sum = __dp4a(w.z, 0x01010101, sum);
            sum = __dp4a(w.w, 0x01010101, sum);
        }
        o.xs[b] = 8 * sum;
    }
    consumer_sync();
}

/* ------------------------------------------------------------ attention */

constexpr int KVU_MAX = 8;   /* 16-byte units of K (and of V) a thread loads per tile */
/* 16-byte units of a K (or V) tile per consumer thread for head_dim hd at es bytes per element. */
__host__ __device__ constexpr int att_units(int es, int hd) { return (ATT_TILE * (hd * es / 16) + NCT - 1) / NCT; }

/* Shared scratch of an attention item, in floats (layout in att_smem; every
 * region starts on a 16-byte boundary). */
__host__ __device__ inline int att_pad4(int n) { return (n + 3) & ~3; }
__host__ __device__ inline int attention_scratch_floats(int group, int hd) {
    return att_pad4(group * hd) + att_pad4((group * hd + 3) / 4) + att_pad4(group)   /* q, int8 q, its scales */
           + ATT_TILE * (hd + 4) + ATT_TILE                                         /* K tile, K scales */
           + ATT_TILE * hd + ATT_TILE                                               /* V tile, V scales */
           + att_pad4(group * ATT_TILE) + 3 * att_pad4(group)                       /* p, m, l, alpha */
           + att_pad4(hd) * 2 + 4                                                   /* this position's K, V, scales */
           + att_pad4(group * hd);                                                  /* the outputs' running sums */
}

struct AttSmem {
    float *sq, *sqd, *sk, *skd, *sv, *svd, *sp, *sm, *sl, *sa, *knew, *vnew, *knd, *acc;
    int8_t *sqq;
};

__device__ __forceinline__ AttSmem att_smem(float *f, int group, int hd) {
    AttSmem s;
    s.sq = f; f += att_pad4(group * hd);
    s.sqq = (int8_t *)f; f += att_pad4((group * hd + 3) / 4);
    s.sqd = f; f += att_pad4(group);
    s.sk = f; f += ATT_TILE * (hd + 4);   /* float K rows hd + 4 apart: 16-byte aligned, float4 reads conflict-free */
    s.skd = f; f += ATT_TILE;
    s.sv = f; f += ATT_TILE * hd;
    s.svd = f; f += ATT_TILE;
    s.sp = f; f += att_pad4(group * ATT_TILE);
    s.sm = f; f += att_pad4(group);
    s.sl = f; f += att_pad4(group);
    s.sa = f; f += att_pad4(group);
    s.knew = f; f += att_pad4(hd);
    s.vnew = f; f += att_pad4(hd);
    s.knd = f; f += 4;
    s.acc = f;
    return s;
}

/* The splits of a KV head's positions at pos: first = the first position in
 * the window, C = positions per split (a multiple of ATT_TILE); returns how
 * many splits hold positions (the rest of the nsplit items are idle). */
__device__ __forceinline__ int att_splits(const StepArgs &a, const LayerPlan &L, int pos, int &first, int &C) {
    first = L.window && pos >= L.window ? pos + 1 - L.window : 0;
    const int n = pos + 1 - first;
    C = (n + a.nsplit - 1) / a.nsplit;
    C = C < ATT_TILE ? ATT_TILE : (C + ATT_TILE - 1) / ATT_TILE * ATT_TILE;
    return (n + C - 1) / C;
}

__device__ __forceinline__ void attention_combine(const StepArgs &a, int U, int active, float *fsm, unsigned t_part,
                                                  unsigned t_ao);

/* Attention work item (KV head g, split y) of layer L at position pos, on the
 * consumer threads; fsm: shared scratch. ops/ops.c:124-180 with the cache
 * types of model/transformer.c:188-205 (KV: KC_F32, KC_F16 or KC_Q8_0):
 * RoPE on adjacent pairs (k_scalar.c:79-94); the split holding pos stores
 * that position's K (after RoPE) and V in the cache's type (f16 rounding, or
 * the single-scale row quantization per KV head) and uses the stored values;
 * scores q.k * scale (Q8: the query quantized per head, int32 dot,
 * (float)s * (qd * scale) * kd), soft-capped when set; online softmax over
 * 64-position tiles loaded one tile ahead; the weighted V sum (Q8: (p * vd)
 * * v). With one split (and a head group of whole blocks) the item
 * publishes the group's outputs, quantized (t_ao); else the splits publish
 * their partials as tagged words (t_part) and count themselves on their
 * unit's counter, and the one whose arrival brings it to `last` combines the
 * unit (attention_combine). q, k and v arrive as tagged words (t_qkv). */
template <int KV>
__device__ __forceinline__ void attention_item_t(const StepArgs &a, const LayerPlan &L, int g, int y, int pos, float *fsm,
                                                 unsigned t_qkv, unsigned t_part, unsigned t_ao, unsigned last) {
    constexpr int ES = KV == KC_F32 ? 4 : (KV == KC_F16 ? 2 : 1);
    /* F16 and Q8 tiles pass through registers (converted on their way into
     * shared memory), up to head_dim 128; F32 tiles are copied by cp.async */
    constexpr int UNITS = KV == KC_F32 ? 1 : att_units(ES, 128);
    const int hd = a.hd, group = a.n_heads / a.n_kv_heads, h2 = hd / 2, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    int first, C;
    const int active = att_splits(a, L, pos, first, C);
    if (y >= active) return;
    const int t_begin = first + y * C, t_end = min(t_begin + C, pos + 1);
    const AttSmem S = att_smem(fsm, group, hd);
    const int upr = hd * ES / 16;                      /* 16-byte units per cache row */
    const size_t rowb = (size_t)a.kv_dim * ES;
    const uint8_t *kb = (const uint8_t *)L.kc + (size_t)g * hd * ES, *vb = (const uint8_t *)L.vc + (size_t)g * hd * ES;
    /* the first tile's K and V are requested before anything else, so their
     * latency overlaps the query's; each later tile is loaded while the one
     * before is computed; the split's own position comes from knew/vnew */
    uint4 rk[UNITS], rv[UNITS];
    float rkd = 0.0f, rvd = 0.0f;
    auto load_tile = [&](int t0) {
        const int nt = min(ATT_TILE, t_end - t0);
#pragma unroll
        for (int e = 0; e < UNITS; e++) {
            const int idx = tid + e * NCT, t = idx / upr, u = idx - t * upr;
            if (idx < nt * upr && t0 + t != pos) {
                rk[e] = __ldcg((const uint4 *)(kb + (size_t)(t0 + t) * rowb + 16 * u));
                rv[e] = __ldcg((const uint4 *)(vb + (size_t)(t0 + t) * rowb + 16 * u));
            }
        }
        if (KV == KC_Q8_0 && tid < nt && t0 + tid != pos) {
            rkd = __ldcg(L.kd + (size_t)(t0 + tid) * a.n_kv_heads + g);
            rvd = __ldcg(L.vd + (size_t)(t0 + tid) * a.n_kv_heads + g);
        }
    };
    /* F32: K (or V) rows of a tile straight into their shared-memory layout,
     * one cp.async group (the own position's row is not in the cache yet) */
    auto copy_rows = [&](int t0, const uint8_t *src, float *dst, int ld) {
        const int nt = min(ATT_TILE, t_end - t0);
        for (int idx = tid; idx < nt * upr; idx += NCT) {
            const int t = idx / upr, u = idx - t * upr;
            if (t0 + t != pos) cp_async16(dst + t * ld + 4 * u, src + (size_t)(t0 + t) * rowb + 16 * u);
        }
        cp_async_commit();
    };
    if (tid == 0) ev(0, EV_ATT_ENTRY);
    /* this thread's first query pair and its RoPE angle, loaded before the tile
     * so that both round trips overlap */
    const float *cs = L.rcos + (size_t)pos * h2, *sn = L.rsin + (size_t)pos * h2;
    const int nq = group * h2;
    word_t q0a = mkword(t_qkv, 0.0f), q0b = q0a;
    float c0 = 0.0f, s0 = 0.0f;
    if (tid < nq) {
        const int h = tid / h2, i = tid - h * h2;
        ld_words2(a.qkvw + (size_t)(g * group + h) * hd + 2 * i, q0a, q0b);
        c0 = cs[i];
        s0 = sn[i];
    }
    if constexpr (KV == KC_F32) {
        copy_rows(t_begin, kb, S.sk, hd + 4);
        copy_rows(t_begin, vb, S.sv, hd);
    } else {
        load_tile(t_begin);
    }
    if (tid < nq) {
        const int h = tid / h2, i = tid - h * h2;
        wait_words2(a.qkvw + (size_t)(g * group + h) * hd + 2 * i, t_qkv, q0a, q0b, a.err);
    }
    if (tid == 0) ev(0, EV_ATT_ISSUED);
    /* qk_norm (model/transformer.c:244-248): 1/rms of each query head first */
    __shared__ float qinv[NCW];
    if (L.q_norm) {
        if (warp < group) {
            const word_t *qh = a.qkvw + (size_t)(g * group + warp) * hd;
            float t = 0.0f;
            for (int i = lane; i < hd; i += 32) {
                const float v = get_word(qh + i, t_qkv, a.err);
                t += v * v;
            }
            t = warp_sum(t);
            if (lane == 0) qinv[warp] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)hd), a.eps)));
        }
        consumer_sync();
    }
    for (int idx = tid; idx < nq; idx += NCT) {
        const int h = idx / h2, i = idx % h2;
        const word_t *qh = a.qkvw + (size_t)(g * group + h) * hd;
        const bool first_pair = idx == tid;
        float qa = first_pair ? wval(q0a) : get_word(qh + 2 * i, t_qkv, a.err);
        float qb = first_pair ? wval(q0b) : get_word(qh + 2 * i + 1, t_qkv, a.err);
        const float c = first_pair ? c0 : cs[i], s = first_pair ? s0 : sn[i];
        if (L.q_norm) {
            qa = __fmul_rn(__fmul_rn(qa, qinv[h]), L.q_norm[2 * i]);
            qb = __fmul_rn(__fmul_rn(qb, qinv[h]), L.q_norm[2 * i + 1]);
        }
        S.sq[h * hd + 2 * i] = __fsub_rn(__fmul_rn(qa, c), __fmul_rn(qb, s));
        S.sq[h * hd + 2 * i + 1] = __fadd_rn(__fmul_rn(qa, s), __fmul_rn(qb, c));
    }
    if (tid == 0) ev(0, EV_ATT_QROPE);
    /* the split holding pos stores that position's K (after RoPE) and V */
    if (t_end == pos + 1 && warp < 2) {
        const word_t *src = a.qkvw + a.q_dim + (warp ? a.kv_dim : 0) + (size_t)g * hd;
        float *row = warp ? S.vnew : S.knew;
        float kinv = 1.0f;
        if (warp == 0 && L.k_norm) {
            float t = 0.0f;
            for (int i = lane; i < hd; i += 32) {
                const float v = get_word(src + i, t_qkv, a.err);
                t += v * v;
            }
            t = warp_sum(t);
            kinv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)hd), a.eps)));
        }
        for (int i = lane; i < h2; i += 32) {
            word_t wa, wb;
            ld_words2(src + 2 * i, wa, wb);
            wait_words2(src + 2 * i, t_qkv, wa, wb, a.err);
            float xa = wval(wa), xb = wval(wb);
            if (warp == 0 && L.k_norm) {
                xa = __fmul_rn(__fmul_rn(xa, kinv), L.k_norm[2 * i]);
                xb = __fmul_rn(__fmul_rn(xb, kinv), L.k_norm[2 * i + 1]);
            }
            if (warp == 0) {
                row[2 * i] = __fsub_rn(__fmul_rn(xa, cs[i]), __fmul_rn(xb, sn[i]));
                row[2 * i + 1] = __fadd_rn(__fmul_rn(xa, sn[i]), __fmul_rn(xb, cs[i]));
            } else {
                row[2 * i] = xa;
                row[2 * i + 1] = xb;
            }
        }
        __syncwarp();
        uint8_t *dst = (uint8_t *)(warp ? L.vc : L.kc) + ((size_t)pos * a.kv_dim + (size_t)g * hd) * ES;
        if constexpr (KV == KC_F32) {
            for (int i = lane; i < hd; i += 32) ((float *)dst)[i] = row[i];
        } else if constexpr (KV == KC_F16) {
            for (int i = lane; i < hd; i += 32) {
                const __half hv = __float2half_rn(row[i]);
                ((__half *)dst)[i] = hv;
                row[i] = __half2float(hv);
            }
        } else {
            const float d = warp_quantize_row(row, hd, (int8_t *)dst, row, lane);
            if (lane == 0) {
                (warp ? L.vd : L.kd)[(size_t)pos * a.n_kv_heads + g] = d;
                S.knd[warp] = d;
            }
        }
    }
    if (tid < group) {
        S.sm[tid] = -INFINITY;
        S.sl[tid] = 0.0f;
    }
    const int nout = group * hd;
    /* one thread per score (a dot over hd) and per output (a sum over the
     * tile), each summed in the order of the reference's loops; the outputs'
     * running sums in shared memory (acc) */
    constexpr int tpd = 1;
    for (int o = tid; o < nout; o += NCT) S.acc[o] = 0.0f;
    consumer_sync();
    if (KV == KC_Q8_0 && warp < group)
        S.sqd[warp] = warp_quantize_row(S.sq + warp * hd, hd, S.sqq + warp * hd, nullptr, lane);
    if (tid == 0) ev(0, EV_ATT_PRE);
    for (int t0 = t_begin; t0 < t_end; t0 += ATT_TILE) {
        const int nt = min(ATT_TILE, t_end - t0);
        if constexpr (KV == KC_F32) {
            /* the tile came by cp.async, all but the own position's row */
            if (pos >= t0 && pos < t0 + nt)
                for (int i = tid; i < hd; i += NCT) {
                    S.sk[(pos - t0) * (hd + 4) + i] = S.knew[i];
                    S.sv[(pos - t0) * hd + i] = S.vnew[i];
                }
        }
#pragma unroll
        for (int e = 0; e < (KV == KC_F32 ? 0 : UNITS); e++) {
            const int idx = tid + e * NCT, t = idx / upr, u = idx - t * upr;
            if (idx < nt * upr) {
                const bool own = t0 + t == pos;
                if constexpr (KV == KC_Q8_0) {
                    if (own) {
#pragma unroll
                        for (int k = 0; k < 16; k++) {
                            ((int8_t *)S.sk)[t * hd + 16 * u + k] = (int8_t)S.knew[16 * u + k];
                            S.sv[t * hd + 16 * u + k] = S.vnew[16 * u + k];
                        }
                    } else {
                        *(uint4 *)((int8_t *)S.sk + t * hd + 16 * u) = rk[e];
                        const int8_t *vq = (const int8_t *)&rv[e];
#pragma unroll
                        for (int k = 0; k < 16; k++) S.sv[t * hd + 16 * u + k] = (float)vq[k];
                    }
                } else {
                    constexpr int PER = 16 / ES;   /* elements per unit */
                    float kf[PER], vf[PER];
                    if (own) {
#pragma unroll
                        for (int k = 0; k < PER; k++) {
                            kf[k] = S.knew[PER * u + k];
                            vf[k] = S.vnew[PER * u + k];
                        }
                    } else if constexpr (KV == KC_F32) {
                        continue;   /* not reached: F32 tiles come by cp.async */
                    } else {
                        const __half *ka = (const __half *)&rk[e], *va = (const __half *)&rv[e];
#pragma unroll
                        for (int k = 0; k < PER; k++) { kf[k] = __half2float(ka[k]); vf[k] = __half2float(va[k]); }
                    }
#pragma unroll
                    for (int k = 0; k < PER; k++) {
                        S.sk[t * (hd + 4) + PER * u + k] = kf[k];
                        S.sv[t * hd + PER * u + k] = vf[k];
                    }
                }
            }
        }
        if (KV == KC_Q8_0 && tid < nt) {
            const bool own = t0 + tid == pos;
            S.skd[tid] = own ? S.knd[0] : rkd;
            S.svd[tid] = own ? S.knd[1] : rvd;
        }
        if (tid == 0) ev(0, EV_ATT_STORED);
        if constexpr (KV == KC_F32) {
            cp_async_wait_all();   /* this thread's copies of the tile's K and V */
        } else {
            if (t0 + ATT_TILE < t_end) load_tile(t0 + ATT_TILE);
        }
        consumer_sync();
        if (tid == 0) ev(0, EV_ATT_SYNCED);
        /* scores: tpd threads per (head, position); every lane takes part in
         * the shuffles, those past the tile with zero */
        for (int pi = tid / tpd; pi < group * ATT_TILE; pi += NCT / tpd) {
            const int h = pi / ATT_TILE, t = pi % ATT_TILE, part = tid % tpd, span = hd / tpd;
            float s = -INFINITY;
            if constexpr (KV == KC_Q8_0) {
                int sum = 0;
                if (t < nt) {
                    const int *qw = (const int *)(S.sqq + h * hd + part * span);
                    const int *kw = (const int *)((const int8_t *)S.sk + t * hd + part * span);
                    for (int i = 0; i < span / 4; i++) sum = __dp4a(qw[i], kw[i], sum);
                }
                for (int o = tpd / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                if (t < nt) s = __fmul_rn(__fmul_rn((float)sum, __fmul_rn(S.sqd[h], a.attn_scale)), S.skd[t]);
            } else {
                float dot = 0.0f;
                if (t < nt) {
                    /* float4 reads of q (broadcast) and of the K row, the sum in order */
                    const float4 *q4 = (const float4 *)(S.sq + h * hd + part * span),
                                 *k4 = (const float4 *)(S.sk + t * (hd + 4) + part * span);
#pragma unroll 4
                    for (int i = 0; i < span / 4; i++) {
                        const float4 qv = q4[i], kv = k4[i];
                        dot = fmaf(qv.x, kv.x, dot);
                        dot = fmaf(qv.y, kv.y, dot);
                        dot = fmaf(qv.z, kv.z, dot);
                        dot = fmaf(qv.w, kv.w, dot);
                    }
                }
                for (int o = tpd / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
                if (t < nt) s = __fmul_rn(dot, a.attn_scale);
            }
            if (t < nt && a.attn_softcap > 0.0f) s = __fmul_rn(a.attn_softcap, tanhf(__fdiv_rn(s, a.attn_softcap)));
            if (part == 0) S.sp[h * ATT_TILE + t] = s;
        }
        consumer_sync();
        /* F32: K is read; the next tile's K lands during the softmax and the V sum */
        if (KV == KC_F32 && t0 + ATT_TILE < t_end) copy_rows(t0 + ATT_TILE, kb, S.sk, hd + 4);
        if (tid == 0) ev(0, EV_ATT_SCORES);
        for (int h = warp; h < group; h += NCW) {
            const float s0 = S.sp[h * ATT_TILE + lane], s1 = S.sp[h * ATT_TILE + 32 + lane];
            const float m_old = S.sm[h], m_new = fmaxf(m_old, warp_max(fmaxf(s0, s1)));
            const float p0 = lane < nt ? expf(s0 - m_new) : 0.0f, p1 = lane + 32 < nt ? expf(s1 - m_new) : 0.0f;
            const float sum = warp_sum(p0 + p1);
            const float alpha = expf(m_old - m_new);
            S.sp[h * ATT_TILE + lane] = p0;
            S.sp[h * ATT_TILE + 32 + lane] = p1;
            if (lane == 0) {
                S.sm[h] = m_new;
                S.sl[h] = S.sl[h] * alpha + sum;
                S.sa[h] = alpha;
            }
        }
        consumer_sync();
        if (tid == 0) ev(0, EV_ATT_SOFTMAX);
        /* outputs: a thread per (head, dimension), positions in order */
        for (int o = tid; o < nout; o += NCT) {
            const int h = o / hd, i = o % hd;
            float v = S.acc[o] * S.sa[h];
            const float *ph = S.sp + h * ATT_TILE;
            int t = 0;
            /* the weights four at a time (broadcast float4 reads) */
#pragma unroll 4
            for (; t + 4 <= nt; t += 4) {
                float4 w4 = *(const float4 *)(ph + t);
                if constexpr (KV == KC_Q8_0) {
                    const float4 d4 = *(const float4 *)(S.svd + t);
                    w4 = make_float4(__fmul_rn(w4.x, d4.x), __fmul_rn(w4.y, d4.y), __fmul_rn(w4.z, d4.z),
                                     __fmul_rn(w4.w, d4.w));
                }
                const float *vc = S.sv + t * hd + i;
                v = fmaf(w4.x, vc[0], v);
                v = fmaf(w4.y, vc[hd], v);
                v = fmaf(w4.z, vc[2 * hd], v);
                v = fmaf(w4.w, vc[3 * hd], v);
            }
            for (; t < nt; t++) {
                const float w = KV == KC_Q8_0 ? __fmul_rn(ph[t], S.svd[t]) : ph[t];
                v = fmaf(w, S.sv[t * hd + i], v);
            }
            S.acc[o] = v;
        }
        consumer_sync();
        /* F32: V is read; the next tile's V lands during the next scores */
        if (KV == KC_F32 && t0 + ATT_TILE < t_end) copy_rows(t0 + ATT_TILE, vb, S.sv, hd);
        if (tid == 0) ev(0, EV_ATT_TILE);
    }
    if (active == 1 && a.att_unit == 1) {
        /* one split: its outputs are the head group's (the combine with one
         * weight, 1 / l, gives the same bits), quantized a block per warp */
        for (int b = warp; b < nout / QK; b += NCW) {
            const int o = b * QK + lane;
            publish_qblock(a.aow, a.q_dim, g * (nout / QK) + b, t_ao,
                           __fmul_rn(S.acc[o], __fdiv_rn(1.0f, S.sl[o / hd])));
        }
        if (tid == 0) ev(0, EV_ATT_DONE);
        return;
    }
    /* this split's partial as tagged words: unnormalized outputs, running max
     * and sum (no fence, no counter: the combine waits on the words) */
    const int stride = hd + 2;
    for (int o = tid; o < nout; o += NCT) {
        const int h = o / hd, i = o % hd;
        st_word(a.partw + ((size_t)(g * group + h) * a.nsplit + y) * stride + i, mkword(t_part, S.acc[o]));
    }
    if (tid < group) {
        word_t *ph = a.partw + ((size_t)(g * group + tid) * a.nsplit + y) * stride;
        st_word(ph + hd, mkword(t_part, S.sm[tid]));
        st_word(ph + hd + 1, mkword(t_part, S.sl[tid]));
    }
    if (tid == 0) ev(0, EV_ATT_PARTIAL);
    /* arrival on the unit's counter (released after every thread's partial
     * words); the split that brings it to `last` has every partial visible
     * (acquired) and combines the unit at once */
    __shared__ int s_last;
    consumer_sync();
    if (tid == 0) {
        unsigned prev;
        asm volatile("atom.release.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "l"(a.attc + (size_t)(g / a.att_unit) * ATT_CNT_STRIDE)
                     : "memory");
        s_last = prev == last;
        if (prev == last) asm volatile("fence.acq_rel.gpu;" ::: "memory");
    }
    consumer_sync();
    if (s_last) attention_combine(a, g / a.att_unit, active, fsm, t_part, t_ao);
}

/* The combine of attention unit U (a.att_unit KV heads whose outputs are
 * whole 32-value blocks: outputs [U * n, U * n + n), n = att_unit * group *
 * hd) by the split that arrived last, once every split's partial is visible:
 * first a warp per query head, a lane per split: the splits' running maxima
 * and sums, M = max m_s, e_s = exp(m_s - M), weight w_s = e_s / sum_s l_s e_s
 * into shared memory; then a thread per output sums the splits' partials in
 * split order with those weights; then a warp per block quantizes and
 * publishes the unit's blocks of the attention output (t_ao). */
/* One output of the combine: the sum over the active splits of partial x
 * weight, in split order, the splits' words requested CB at a time (one
 * round trip per batch). */
template <int CB>
__device__ __forceinline__ float combine_sum(const word_t *ps, int stride, const float *wh, int active, unsigned t_part,
                                             bool &ok) {
    float num = 0.0f;
#pragma unroll 1
    for (int s0 = 0; s0 < active; s0 += CB) {
        float pv[CB];
#pragma unroll
        for (int k = 0; k < CB; k++) {
            pv[k] = 0.0f;
            if (s0 + k < active) {
                const word_t wv = ld_word(ps + (size_t)(s0 + k) * stride);
                ok = ok && wok(wv, t_part);
                pv[k] = wval(wv);
            }
        }
#pragma unroll
        for (int k = 0; k < CB; k++)
            if (s0 + k < active) num = fmaf(pv[k], wh[s0 + k], num);
    }
    return num;
}

__device__ __forceinline__ void attention_combine(const StepArgs &a, int U, int active, float *fsm, unsigned t_part,
                                                  unsigned t_ao) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, hd = a.hd, stride = hd + 2;
    const int heads = a.att_unit * (a.n_heads / a.n_kv_heads), h0 = U * heads, n = heads * hd;
    float *sw = fsm, *out = fsm + heads * MAX_NSPLIT;   /* [heads][MAX_NSPLIT] weights, [n] outputs */
    if (tid == 0) ev(0, EV_ATT_COMBINE);
    for (int w = warp; w < heads; w += NCW) {
        const word_t *ps = a.partw + ((size_t)(h0 + w) * a.nsplit + lane) * stride;
        float m = -INFINITY, lsum = 0.0f;
        if (lane < active) {
            word_t wm, wl;
            ld_words2(ps + hd, wm, wl);
            if (!wok(wm, t_part) || !wok(wl, t_part)) atomicOr(a.err, ERR_POLL);
            m = wval(wm);
            lsum = wval(wl);
        }
        const float M = warp_max(m);
        const float e = lane < active ? expf(m - M) : 0.0f;
        sw[w * MAX_NSPLIT + lane] = e / warp_sum(lsum * e);
    }
    consumer_sync();
#pragma unroll 1
    for (int o = tid; o < n; o += NCT) {
        const int h = o / hd, i = o - h * hd;
        const word_t *ps = a.partw + (size_t)(h0 + h) * a.nsplit * stride + i;
        const float *wh = sw + h * MAX_NSPLIT;
        bool ok = true;
        /* short contexts (a few splits) take the short batch: fewer predicated slots */
        const float num = active <= 8 ? combine_sum<8>(ps, stride, wh, active, t_part, ok)
                                      : combine_sum<MAX_NSPLIT>(ps, stride, wh, active, t_part, ok);
        if (!ok) atomicOr(a.err, ERR_POLL);
        out[o] = num;
    }
    consumer_sync();
    for (int b = warp; b < n / QK; b += NCW) publish_qblock(a.aow, a.q_dim, U * (n / QK) + b, t_ao, out[b * QK + lane]);
    if (tid == 0) ev(0, EV_ATT_DONE);
}

/* ------------------------------------------------------------ shared layout */

/* Dynamic shared memory of a streaming CTA: mbarriers [2][nstage], per-warp
 * argmax [NCW], flag, reduction scratch [32], the owned rows of x [OWN_MAX],
 * activation (or attention scratch) of act_bytes, then the ring (128 B
 * aligned). */
struct Smem {
    uint64_t *full, *empty;
    unsigned long long *cta_best;
    int *flag;
    float *red;
    float *own;
    float *yown;   /* post-norm models: the CTA's rows of the last block output */
    float *res;
    float *wbuf;   /* the next norm phase's weights, copied in ahead of its barrier */
    unsigned char *act;
    uint8_t *ring;
};

/* res_bytes: a phase's row results (16-byte multiple). */
__host__ __device__ inline int smem_fixed_bytes(int nstage, int act_bytes, int res_bytes = 0, int wbuf_bytes = 0) {
    return 16 * nstage + 8 * NCW + 16 + 4 * 32 + 8 * OWN_MAX + res_bytes + wbuf_bytes + act_bytes +
           128;
}

__device__ __forceinline__ Smem carve(unsigned char *smem, int nstage, int act_bytes, int res_bytes = 0,
                                      int wbuf_bytes = 0) {
    Smem s;
    s.full = (uint64_t *)smem;
    s.empty = s.full + nstage;
    s.cta_best = (unsigned long long *)(s.empty + nstage);
    s.flag = (int *)(s.cta_best + NCW);
    s.red = (float *)(s.flag + 4);
    s.own = s.red + 32;
    s.yown = s.own + OWN_MAX;
    s.res = s.yown + OWN_MAX;
    s.wbuf = (float *)((unsigned char *)s.res + res_bytes);
    s.act = (unsigned char *)s.wbuf + wbuf_bytes;
    s.ring = (uint8_t *)(((uintptr_t)(s.act + act_bytes) + 127) & ~(uintptr_t)127);
    return s;
}

__device__ __forceinline__ void init_ring(const Smem &s, int nstage) {
    if (threadIdx.x == 0) {
        for (int i = 0; i < nstage; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], NCW);
        }
        fence_barrier_init();
    }
    __syncthreads();
}

/* ------------------------------------------------------------ the step kernel */

__shared__ PhasePlan s_plan[NPHASE];

/* The layer plans in shared memory, double-buffered by the running layer
 * index gl: layer gl + 1's plan is copied (cp.async, LP_UNITS threads) while
 * layer gl runs, so no phase waits on a global load of its layer's pointers. */
__shared__ LayerPlan s_lp[2];
constexpr int LP_UNITS = sizeof(LayerPlan) / 16;
static_assert(sizeof(LayerPlan) % 16 == 0, "LayerPlan copies in 16-byte units");
__device__ __forceinline__ void fetch_plan(const LayerPlan *src, LayerPlan *dst) {
    if (threadIdx.x < LP_UNITS) cp_async16((char *)dst + 16 * threadIdx.x, (const char *)src + 16 * threadIdx.x);
}

/* Producer: this CTA's stream once per step (the classifier only when the
 * step computes logits). */
__device__ __forceinline__ void producer(const StepArgs &a, Ring rg) {
    const uint8_t *base = a.stream + a.cta_base[blockIdx.x];
    for (int s = 0; s < a.nsteps; s++) {
        const uint8_t *src = base;
        for (int l = 0; l < a.n_layers; l++)
            for (int p = PH_A; p <= PH_E; p++) produce_phase(rg, s_plan[p], src, a.err);
        if (a.run_cls) produce_phase(rg, s_plan[PH_F], src, a.err);
    }
}

/* One instance per KV cache type (KV: KC_F32, KC_F16, KC_Q8_0) and block
 * scale type of the weight stream (D16: f16, else f32); the host launches the
 * state's. Each carries only its own attention and consumer code, and the
 * post-norm and tensor-parallel steps are out of line, so the instructions a
 * layer runs through stay fewer and closer together. */
template <int KV, bool D16>
__global__ void __launch_bounds__(STEP_THREADS, 1) step_kernel(const __grid_constant__ StepArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const Smem sh = carve(smem, a.nstage, a.act_bytes, a.res_bytes, a.wbuf_bytes);
    ev_init(true);
    if (threadIdx.x == 0) make_plan(a.geom, blockIdx.x, gridDim.x, s_plan);
    init_ring(sh, a.nstage);
    Ring rg{ sh.full, sh.empty, sh.ring, a.nstage, a.slot_bytes, 0, 0u };
    if ((threadIdx.x >> 5) == NCW) {
        if ((threadIdx.x & 31) == 0) producer(a, rg);
        return;
    }
    const int j = blockIdx.x, G = gridDim.x;
    int own0, own1;
    share_rows(a.dim, j, G, own0, own1);
    const int nown = own1 - own0;
    unsigned expect = 0, pidx = 0;   /* step-end barrier arrivals due so far, trace index */
    unsigned att_seen = 0;           /* arrivals on each attention unit counter so far in this launch */
    /* x words, sums of squares, post-norm block outputs: one buffer for the O
     * phase (C) and one for the down phase (E) */
    word_t *const xw_c = a.xw, *const xw_e = a.xw + a.dim;
    word_t *const ss_c = a.sspw, *const ss_e = a.sspw + G;
    word_t *const yw_c = a.yw, *const yw_e = a.yw + a.dim;
    if (threadIdx.x == 0) timeline_mark(a);
    fetch_plan(a.layers, &s_lp[0]);
    cp_async_wait_all();
    consumer_sync();
    unsigned gl = 0;   /* running layer index over the launch's steps */
    for (int step = 0; step < a.nsteps; step++) {
        /* the loop state, read by one thread and shared (every thread of every
         * CTA on the same line would queue at its L2 slice) */
        __shared__ int s_ls[4];
        __shared__ float s_inv0;
        if (threadIdx.x == 0) {
            const int tok = __ldcg(&a.ls->token), pos = __ldcg(&a.ls->pos);
            const bool ok = tok >= 0 && tok < a.vocab && pos >= 0 && pos < a.max_seq;
            if (!ok) atomicOr(&a.ls->err, 1u);
            s_ls[0] = ok ? tok : 0;
            s_ls[1] = ok ? pos : 0;
            s_ls[2] = (__ldcg(&a.ls->step) % LOGITS_RING) * a.vocab;
            s_inv0 = a.inv0[s_ls[0]];
        }
        consumer_sync();
        const int tk = s_ls[0], ps = s_ls[1], logit_row0 = s_ls[2];
        const float inv0 = s_inv0;
        /* the step as one loop over its stages: per layer A (Q/K/V), B
         * (attention), C (O + residual), D (gate/up), E (down + residual),
         * then F (classifier). Every matrix phase runs through the same code
         * (one copy of the prologue call, of the consumer loops and of the
         * finish): the instructions a layer executes stay few enough to be
         * cached instead of fetched again from L2 in every phase. */
        const int nstages = 5 * a.n_layers + (a.run_cls ? 1 : 0);
        for (int sg = 0; sg < nstages; sg++) {
            const int l = sg / 5, k = sg - 5 * l;
            const bool cls = l == a.n_layers;   /* F */
            const LayerPlan &L = s_lp[gl & 1];
            if (k == 1) {
                /* B: attention; the next layer's plan is fetched meanwhile (the
                 * buffer's last reader, the previous layer's A prologue, is done) */
                fetch_plan(a.layers + (l + 1 < a.n_layers ? l + 1 : 0), &s_lp[(gl + 1) & 1]);
                trace_mark(a, pidx, 0);
                if (threadIdx.x == 0) ev(0, EV_PRO_DONE);
                const unsigned t_qkv = tag_of(a, step, l, TAG_QKV);
                /* arrivals on each unit counter before this layer's: every CTA
                 * keeps the count (the counters only grow within a launch) */
                int first, span;
                const int active = att_splits(a, L, ps, first, span);
                const bool direct = active == 1 && a.att_unit == 1;
                const unsigned last = att_seen + (unsigned)(a.att_unit * active) - 1u;
                for (int it = j; it < a.n_kv_heads * a.nsplit; it += G)
                    attention_item_t<KV>(a, L, it / a.nsplit, it % a.nsplit, ps, (float *)sh.act, t_qkv, t_qkv + 1,
                                         t_qkv + 2, last);
                if (!direct) att_seen += (unsigned)(a.att_unit * active);
                consumer_sync();   /* the attention scratch is the next activation's space */
                phase_end(a, pidx);
                continue;
            }
            /* the stage's matrix phase: its plan, input words and their tag, norm */
            const int ph = cls ? PH_F : (k == 0 ? PH_A : (k == 2 ? PH_C : (k == 3 ? PH_D : PH_E)));
            const int cols = ph == PH_C ? a.q_dim : (ph == PH_E ? a.hidden : a.dim);
            const ActW w = act_layout(sh.act, cols);
            const unsigned tg = tag_of(a, step, cls ? a.n_layers - 1 : l, 0);   /* the layer's first tag */
            if (ph == PH_A && l == 0) {
                act_embed(a.emb, a.embed_scale, tk, L.attn_norm, inv0, a.dim, w);
                /* the residual stream starts as the embedding row: this CTA's rows of x */
                for (int r = own0 + (int)threadIdx.x; r < own1; r += NCT) sh.own[r - own0] = embed1(a, tk, a.dim, r);
            } else {
                if (ph == PH_C || ph == PH_E) {   /* attention output, FFN hidden: quantized words */
                    act_qwords(ph == PH_C ? a.aow : a.hbw, tg + (ph == PH_C ? TAG_AO : TAG_HB), cols, w, a.err);
                } else {
                    /* x after the previous layer's down phase (A, F) or this layer's O phase (D) */
                    const bool e = ph != PH_D;
                    const unsigned tin = ph == PH_D ? tg + TAG_XC : (ph == PH_F ? tg + TAG_XE : tg - NTAG + TAG_XE);
                    const float *nw = ph == PH_D ? L.ffn_norm : (ph == PH_F ? a.final_norm : L.attn_norm);
                    if (a.post_norms)
                        act_postnorm(a, e ? xw_e : xw_c, e ? yw_e : yw_c, e ? ss_e : ss_c, tin,
                                     e ? s_lp[(gl - 1) & 1].post_ffn : L.post_attn, nw, a.dim, w, sh.red, sh.own, own0,
                                     own1);
                    else
                        load_activation(a, e ? xw_e : xw_c, tin, nw, cols, w, sh.red, nw ? sh.wbuf : nullptr);
                }
            }
            trace_mark(a, pidx, 0);
            if (threadIdx.x == 0) ev(0, EV_PRO_DONE);
            const PhasePlan &P = s_plan[ph];
            consume_phase<D16>(rg, P, ph == PH_D, act_view(w), sh.res, a.err);
            const int ns = col_slices(cols / QK, false);
            if (ph == PH_A) {
                finish_phase(FIN_STORE, sh.res, plan_rows(P), P.nseg ? P.seg[0].row0 : 0, nullptr, a.qkvw,
                             tg + TAG_QKV, nullptr, 0, 0.0f, sh.cta_best, ns);
            } else if (ph == PH_D) {
                if (a.geom.d_unit == QK)
                    finish_pair_q(sh.res, P.seg[0].rows, P.seg[0].row0, a.hbw, a.hidden, tg + TAG_HB, a.act);
                else
                    finish_pair_split(sh.res, P.seg[0].rows, P.seg[0].row0, a.hbw, a.hidden, tg + TAG_HB, a.act,
                                      a.amaxw, a.hidden / a.geom.d_unit, a.err);
            } else if (ph == PH_F) {
                const Seg &F = P.seg[0];
                const unsigned long long b =
                    finish_phase(FIN_LOGITS, sh.res, F.rows, a.cls_row0 + F.row0, a.logits + logit_row0, nullptr, 0,
                                 nullptr, 0, a.final_softcap, sh.cta_best, ns);
                if (threadIdx.x == 0 && b) atomicMax(&a.ls->best, b);
                if (a.tp_world > 1) {
                    /* this rank's logits rows into every other rank's ring (each thread
                     * re-reads the rows it wrote itself) */
                    for (int i = threadIdx.x; i < F.rows; i += NCT) {
                        const size_t o = (size_t)logit_row0 + a.cls_row0 + F.row0 + i;
                        const float v = a.logits[o];
                        for (int r = 0; r < a.tp_world; r++)
                            if (r != a.tp_rank) ((float *)(a.tp_box[r] + a.tp_off_logits))[o] = v;
                    }
                    __threadfence_system();
                }
                break;   /* F is the step's last stage */
            } else {
                /* C and E: the residual add on the CTA's rows of x */
                const bool c = ph == PH_C;
                const unsigned tx = tg + (c ? TAG_XC : TAG_XE);
                word_t *const xo = c ? xw_c : xw_e, *const so = c ? ss_c : ss_e;
                if (a.post_norms) {
                    finish_post(sh.res, nown, own0, ns, xo, c ? yw_c : yw_e, tx, sh.own, sh.yown);
                    publish_ssp(so, tx, sh.yown, nown);
                } else if (a.tp_world > 1) {
                    tp_resid(a, sh.res, nown, own0, sh.own, ns, c ? 0 : 1, tp_seq(a, step, l, c ? 0 : 1));
                    publish_rows(xo, tx, sh.own, nown, own0);
                } else if (nown <= 32) {
                    finish_resid_warp(sh.res, nown, own0, xo, tx, sh.own, ns);
                } else {
                    finish_phase(FIN_RESID, sh.res, nown, own0, nullptr, xo, tx, sh.own, 0, 0.0f, sh.cta_best, ns);
                }
                if (c) {
                    prefetch_norm(sh.wbuf, L.ffn_norm, a.dim);
                } else {
                    /* the next layer's plan (landed long ago) to every thread, then its
                     * norm weights on their way while the next prologue waits */
                    if (threadIdx.x < LP_UNITS) cp_async_wait_all();
                    consumer_sync();
                    prefetch_norm(sh.wbuf,
                                  l + 1 < a.n_layers ? s_lp[(gl + 1) & 1].attn_norm : (a.run_cls ? a.final_norm : nullptr),
                                  a.dim);
                    gl++;
                }
            }
            phase_end(a, pidx);
        }
        /* every CTA arrives; the last one advances the loop state, then
         * releases the others with one more arrival (the one grid barrier of a
         * step: it also orders this step's KV rows before the next step's reads) */
        consumer_sync();
        const unsigned pfin = pidx++;
        expect += gridDim.x;
        if (threadIdx.x == 0) {
            trace_mark(a, pfin, 1);
            __threadfence();
            const unsigned prev = atomicAdd(a.bar, 1u);
            if (prev == expect - 1) {
                LoopState *ls = a.ls;
                const int st = ls->step;
                if (a.run_cls) {
                    unsigned long long b = atomicAdd(&ls->best, 0ull);
                    if (a.tp_world > 1) b = tp_argmax(a, b, (unsigned)(a.tp_step0 + (unsigned long long)step + 1ull));
                    const int next = (int)(0xffffffffu - (unsigned)(b & 0xffffffffull));
                    a.out_tokens[st] = next;
                    ls->token = ls->feed_mode ? a.feed[st + 1] : next;
                } else {
                    ls->token = a.feed[st + 1];
                }
                ls->step = st + 1;
                ls->pos = ls->pos + 1;
                ls->best = 0ull;
                __threadfence();
                atomicAdd(a.bar, 1u);
            }
            wait_count(a, expect + 1);
            trace_mark(a, pfin, 2);
        }
        expect += 1;
        consumer_sync();
    }
}

/* ------------------------------------------------------------ kernel-level kernels */

/* One matrix against one quantized activation (kc_matvec_dev): the step
 * kernel's ring and consumers over rows [0, rows), CTA j of G owning its
 * share, the matrix in the file's layout. */
struct MatvecArgs {
    PMat m;
    int cols;
    const int8_t *xq;
    const float *xd;
    float *y;
    unsigned *err;                 /* sticky device error word of the entry point */
    unsigned wait_limit;           /* polls of the consumers' first wait on a chunk */
    int nstage, slot_bytes, act_bytes;
};

__global__ void __launch_bounds__(STEP_THREADS, 1) matvec_kernel(const __grid_constant__ MatvecArgs p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const Smem sh = carve(smem, p.nstage, p.act_bytes);
    ev_init(false);
    init_ring(sh, p.nstage);
    Ring rg{ sh.full, sh.empty, sh.ring, p.nstage, p.slot_bytes, 0, 0u };
    int r0, r1;
    share_rows(p.m.rows, blockIdx.x, gridDim.x, r0, r1);
    if ((threadIdx.x >> 5) == NCW) {
        if ((threadIdx.x & 31) == 0) produce_rows(rg, p.m, p.cols, r0, r1, p.err);
        return;
    }
    const ActW w = act_layout(sh.act, p.cols);
    act_prequant(p.xq, p.xd, p.cols, w);
    if (p.m.type == T_Q4) {
        if (p.m.d16) consume_rows<T_Q4, true>(rg, p.cols, r0, r1, p.y, act_view(w), p.err, p.wait_limit);
        else consume_rows<T_Q4, false>(rg, p.cols, r0, r1, p.y, act_view(w), p.err, p.wait_limit);
    } else {
        if (p.m.d16) consume_rows<T_Q8, true>(rg, p.cols, r0, r1, p.y, act_view(w), p.err, p.wait_limit);
        else consume_rows<T_Q8, false>(rg, p.cols, r0, r1, p.y, act_view(w), p.err, p.wait_limit);
    }
}

/* The activation prologue alone (kc_quantize_q8_dev, kc_rmsnorm_quantize_dev):
 * one CTA of consumer threads writes its shared arrays out. */
__global__ void __launch_bounds__(NCT, 1) activation_kernel(const float *x, const float *w, float eps, int n, int8_t *q,
                                                           float *d, float *xn) {
    extern __shared__ __align__(128) unsigned char smem[];
    float *red = (float *)smem;
    const ActW o = act_layout(smem + 128, n);
    act_loop(eps, x, w, n, o, red);
    for (int i = threadIdx.x; i < n; i += NCT) {
        const int b = i / QK, j = i % QK;
        q[i] = j < 16 ? o.xlo[b * 16 + j] : o.xhi[b * 16 + j - 16];
    }
    for (int b = threadIdx.x; b < n / QK; b += NCT) d[b] = o.xd[b];
    if (xn && w) {
        float ss = 0.0f;
        for (int i = threadIdx.x * 4; i < n; i += NCT * 4) {
            const float4 v = *(const float4 *)(x + i);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        ss = block_sum(ss, red);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
        for (int i = threadIdx.x; i < n; i += NCT) xn[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
    }
}

/* int32 block sums through dot_q4 / dot_q8 (the streaming kernels' integer path). */
__global__ void block_sums_kernel(int32_t *out, int type, const uint8_t *wq, int rows, int cols, const int8_t *xq) {
    const int nb = cols / QK;
    const size_t total = (size_t)rows * nb;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / nb), b = (int)(i % nb);
        const int4 *x4 = (const int4 *)(xq + (size_t)b * QK);
        int s;
        if (type == T_Q4) {
            const uint4 w = *(const uint4 *)(wq + ((size_t)r * nb + b) * 16);
            int xsum = 0;
            for (int j = 0; j < QK; j++) xsum += xq[(size_t)b * QK + j];
            s = dot_q4(w, x4[0], x4[1]) - 8 * xsum;
        } else {
            const uint4 *w = (const uint4 *)(wq + (size_t)r * cols + (size_t)b * QK);
            s = dot_q8(w[0], x4[0]) + dot_q8(w[1], x4[1]);
        }
        out[i] = s;
    }
}

}  // namespace kc
