/* The decode token loop as one persistent kernel (sm_100a), and the
 * kernel-level kernels that run the same device code.
 *
 * Streaming CTA: NCW consumer warps + 1 producer warp, one CTA per SM. Each
 * CTA owns a fixed 1/G share of the rows of every weight matrix. The producer
 * streams those rows (quants and block scales, contiguous in HBM) through a
 * shared-memory ring with bulk copies in the order the step uses them (per
 * layer: Q/K/V, O, gate+up, down; then the classifier), waiting only for free
 * ring slots, so HBM keeps streaming while the consumers wait at phase
 * boundaries.
 *
 * The consumers run the phases of a step, separated by grid barriers (an
 * arrival counter in global memory; every wait is bounded):
 *   A  RMSNorm + quantize x (layer 0: the embedding row, its 1/rms from the
 *      host table) -> Q/K/V rows (+ biases)            model/transformer.c:270-277
 *   B  attention work items (KV head, position range): RoPE, this position's
 *      K/V row into the cache, split flash decode; the last CTA per KV head
 *      combines the splits                             transformer.c:280-283, ops/ops.c:124-180
 *   C  quantize the attention output -> O rows, x += o  transformer.c:284-287
 *   D  RMSNorm + quantize x -> gate/up row pairs -> act(g) * u   :288-293
 *   E  quantize h -> down rows, x += y                 :294-297
 *   F  RMSNorm + quantize x -> classifier rows and the first-index argmax;
 *      the last CTA to arrive advances the token loop  :299-305, model/sampler.c:57-61
 * Several steps run in one launch: the token of step s+1 is the argmax of
 * step s (greedy) or the next prompt token (prefill).
 *
 * Quantized activations follow the reference's rule bit for bit
 * (kernels/scalar/k_scalar.c:39-57); block dot products are exact int32
 * (dp4a); the float scale-accumulate is (float)s * d_w * d_x per block
 * (k_scalar.c:4-37) summed in lane and warp-tree order.
 */
#pragma once
#include "kc_kernels.cuh"

namespace kc {

struct PMat {
    const uint8_t *q;
    const void *d;
    int rows, type, d16;
};

struct LayerPlan {
    PMat wq, wk, wv, wo, w1, w3, w2;
    const float *attn_norm, *ffn_norm, *bq, *bk, *bv;
    float *kc, *vc;                 /* this layer's F32 cache [max_seq][kv_dim] */
    const float *rcos, *rsin;       /* RoPE tables of this layer */
    int window;
};

struct StepArgs {
    const LayerPlan *layers;        /* device array [n_layers] */
    PMat emb, cls;
    const float *final_norm, *inv0;
    float *x, *qkv, *ao, *hb, *logits, *part;
    float *ssp;                     /* [G] per-CTA sum of squares of the x rows it last wrote */
    unsigned *att_counter, *bar, *err;
    LoopState *ls;
    const int *feed;
    int *out_tokens;
    int n_layers, dim, q_dim, kv_dim, hidden, vocab, max_seq, n_heads, n_kv_heads, hd;
    float eps, attn_scale, attn_softcap, final_softcap, embed_scale;
    int act, nsplit, nstage, slot_bytes, act_bytes;
    int nsteps, run_cls;            /* steps in this launch; run the classifier */
    unsigned long long *timeline;   /* optional: globaltimer at start and after each barrier (CTA 0) */
    unsigned *timeline_n;
    unsigned timeline_cap;
    unsigned long long *trace;      /* optional: [phase][G][3] per CTA: prologue done, arrived, released */
    unsigned trace_phases;
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
       EV_ISSUE = 8 };

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

/* Grid barrier: every CTA arrives once; `expect` (the same in every CTA)
 * counts the arrivals due so far in this launch (the host zeroes the counter
 * before each launch). */
__device__ __forceinline__ void grid_barrier(const StepArgs &a, unsigned &expect) {
    consumer_sync();
    const unsigned p = expect / gridDim.x;
    expect += gridDim.x;
    if (threadIdx.x == 0) {
        trace_mark(a, p, 1);
        ev(0, EV_ARRIVE);
        __threadfence();
        atomicAdd(a.bar, 1u);
        wait_count(a, expect);
        trace_mark(a, p, 2);
        ev(0, EV_RELEASE);
    }
    consumer_sync();
}

/* ------------------------------------------------------------ the ring */

struct Ring {
    uint64_t *full, *empty;
    uint8_t *base;
    int nstage, slot_bytes;
    unsigned idx;   /* tiles issued (producer) or consumed (consumer) so far */
};

/* Rows [r0, r1) of a `rows`-row matrix owned by CTA j of G. */
__device__ __forceinline__ void share_rows(int rows, int j, int G, int &r0, int &r1) {
    r0 = (int)((long long)rows * j / G);
    r1 = (int)((long long)rows * (j + 1) / G);
}

/* Producer: issue the tiles of rows [r0, r1) of m (and of m2 when pair). */
__device__ __forceinline__ void produce_rows(Ring &rg, const PMat &m, const PMat *m2, int cols, int r0, int r1,
                                             unsigned *err) {
    if (r0 >= r1) return;
    const int pair = m2 != nullptr;
    int R, qbytes, dbytes;
    stage_geom(m.type, m.d16, cols, pair, R, qbytes, dbytes);
    const int qrow = m.type == T_Q4 ? cols / 2 : cols, drow = (cols / QK) * (m.d16 ? 2 : 4);
    for (int ra = r0; ra < r1; ra += R) {
        const int slot = (int)(rg.idx % (unsigned)rg.nstage);
        ev(1, EV_EMPTY_WAIT);
        if (rg.idx >= (unsigned)rg.nstage && !mbar_wait(&rg.empty[slot], (rg.idx / rg.nstage - 1) & 1u, err))
            atomicOr(err, 2u);
        const int nr = min(R, r1 - ra);
        const size_t ds = (size_t)ra * drow, de = (size_t)(ra + nr) * drow;
        const size_t das = ds & ~(size_t)15, dae = (de + 15) & ~(size_t)15;
        const unsigned qb = (unsigned)(nr * qrow), db = (unsigned)(dae - das);
        uint8_t *dst = rg.base + (size_t)slot * rg.slot_bytes;
        mbar_expect_tx(&rg.full[slot], (qb + db) * (pair ? 2u : 1u));
        bulk_g2s(dst, m.q + (size_t)ra * qrow, qb, &rg.full[slot]);
        bulk_g2s(dst + qbytes, (const uint8_t *)m.d + das, db, &rg.full[slot]);
        if (pair) {
            bulk_g2s(dst + qbytes + dbytes, m2->q + (size_t)ra * qrow, qb, &rg.full[slot]);
            bulk_g2s(dst + 2 * qbytes + dbytes, (const uint8_t *)m2->d + das, db, &rg.full[slot]);
        }
        ev(1, EV_ISSUE);
        rg.idx++;
    }
}

/* ------------------------------------------------------------ consumers */

struct Act {
    const int8_t *xq;   /* [cols] quantized activation */
    const float *xd;    /* [cols/32] its scales */
    const int *xs;      /* [cols/32] 8 * sum of each block's quants */
};

struct Epi {
    int kind;           /* EPI_STORE / EPI_RESID / EPI_PAIR / EPI_LOGITS */
    float *out;
    const float *bias;
    int act;            /* EPI_PAIR: 0 SiLU, 1 GELU */
    float softcap;      /* EPI_LOGITS: final soft-cap, 0 = none */
    int logit_row0;     /* EPI_LOGITS: offset of this step's logits row */
};

__device__ __forceinline__ void epilogue(const Epi &e, int row, float acc, float acc2, unsigned long long &best) {
    switch (e.kind) {
    case EPI_STORE: e.out[row] = e.bias ? __fadd_rn(acc, e.bias[row]) : acc; break;
    case EPI_RESID: e.out[row] = __fadd_rn(e.out[row], acc); break;
    case EPI_PAIR: e.out[row] = act_mul(e.act, acc, acc2); break;
    case EPI_LOGITS: {
        float v = acc;
        if (e.softcap > 0.0f) v = __fmul_rn(e.softcap, tanhf(__fdiv_rn(v, e.softcap)));
        e.out[e.logit_row0 + row] = v;
        const unsigned long long k = argmax_key(v, row);
        best = k > best ? k : best;
        break;
    }
    }
}

template <bool D16>
__device__ __forceinline__ float sm_scale(const uint8_t *dr, int b) {
    if constexpr (D16) return __half2float(((const __half *)dr)[b]);
    else return ((const float *)dr)[b];
}

/* Dot products of nr (<= NR) weight rows held in shared memory (quants of row
 * r at q + r*qrow, scales at d + r*drow; with PAIR the second matrix at q2, d2)
 * against the activation, over the 32-chunk slices s0, s0 + sstep, ... of the
 * rows. Chunks are 16 bytes: a Q4 block or half a Q8 block. The activation of
 * a chunk is loaded once for all rows. Warp-reduced into acc[r][0..1]. */
template <int TYPE, bool D16, bool PAIR, int NR>
__device__ __forceinline__ void dot_rows(const uint8_t *q, const uint8_t *d, const uint8_t *q2, const uint8_t *d2,
                                         int qrow, int drow, int nr, int s0, int sstep, int nch, const Act &x, int lane,
                                         float (&acc)[NR][2]) {
    constexpr int CPB = TYPE == T_Q4 ? 1 : 2;
    const int4 *x4 = (const int4 *)x.xq;
#pragma unroll
    for (int r = 0; r < NR; r++) acc[r][0] = acc[r][1] = 0.0f;
    for (int s = s0; s * 32 < nch; s += sstep) {
        const int c = s * 32 + lane;
        const bool ok = c < nch;
        const int b = c / CPB;
        if constexpr (TYPE == T_Q4) {
            if (ok) {
                const int4 xlo = x4[2 * b], xhi = x4[2 * b + 1];
                const float dx = x.xd[b];
                const int corr = x.xs[b];
#pragma unroll
                for (int r = 0; r < NR; r++) {
                    if (r < nr) {
                        const uint4 w = *(const uint4 *)(q + r * qrow + 16 * c);
                        acc[r][0] += __fmul_rn((float)(dot_q4(w, xlo, xhi) - corr), sm_scale<D16>(d + r * drow, b)) * dx;
                        if constexpr (PAIR) {
                            const uint4 w2 = *(const uint4 *)(q2 + r * qrow + 16 * c);
                            acc[r][1] += __fmul_rn((float)(dot_q4(w2, xlo, xhi) - corr), sm_scale<D16>(d2 + r * drow, b)) * dx;
                        }
                    }
                }
            }
        } else {
            const int4 xv = ok ? x4[c] : make_int4(0, 0, 0, 0);
            const float dx = ok ? x.xd[b] : 0.0f;
#pragma unroll
            for (int r = 0; r < NR; r++) {
                if (r < nr) {
                    int t0 = ok ? dot_q8(*(const uint4 *)(q + r * qrow + 16 * c), xv) : 0;
                    t0 += __shfl_xor_sync(0xffffffffu, t0, 1);   /* both halves of the block */
                    if (ok && !(lane & 1)) acc[r][0] += __fmul_rn((float)t0, sm_scale<D16>(d + r * drow, b)) * dx;
                    if constexpr (PAIR) {
                        int t1 = ok ? dot_q8(*(const uint4 *)(q2 + r * qrow + 16 * c), xv) : 0;
                        t1 += __shfl_xor_sync(0xffffffffu, t1, 1);
                        if (ok && !(lane & 1)) acc[r][1] += __fmul_rn((float)t1, sm_scale<D16>(d2 + r * drow, b)) * dx;
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < NR; r++) {
        if (r < nr) {
            acc[r][0] = warp_sum(acc[r][0]);
            if constexpr (PAIR) acc[r][1] = warp_sum(acc[r][1]);
        }
    }
}

/* Consumer side of rows [r0, r1) of m (and m2), tile by tile from the ring.
 * A tile of at least NCW rows is split by whole rows (NR rows per warp at a
 * time, epilogue by the warp); a smaller tile (long rows) splits each row over
 * NCW / R warps, whose partial sums meet in psum in a fixed order. */
template <int TYPE, bool D16, bool PAIR>
__device__ void consume_rows(Ring &rg, int cols, int r0, int r1, const Epi &e, const Act &x, float *psum,
                             unsigned *err, unsigned long long &best) {
    if (r0 >= r1) return;
    const int nb = cols / QK, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int CPB = TYPE == T_Q4 ? 1 : 2;
    const int nch = nb * CPB;
    const int qrow = TYPE == T_Q4 ? cols / 2 : cols, drow = nb * (D16 ? 2 : 4);
    int R, qbytes, dbytes;
    stage_geom(TYPE, D16, cols, PAIR, R, qbytes, dbytes);
    for (int ra = r0; ra < r1; ra += R) {
        const int slot = (int)(rg.idx % (unsigned)rg.nstage);
        if (!mbar_wait(&rg.full[slot], (rg.idx / rg.nstage) & 1u, err) && lane == 0) atomicOr(err, 2u);
        if (threadIdx.x == 0) ev(0, EV_STAGE_READY);
        const int nr = min(R, r1 - ra);
        const int doff = (int)(((size_t)ra * drow) & 15);
        const uint8_t *sq = rg.base + (size_t)slot * rg.slot_bytes;
        const uint8_t *sd = sq + qbytes + doff;
        const uint8_t *sq2 = sq + qbytes + dbytes, *sd2 = sq2 + qbytes + doff;
        if (R >= 2 * NCW) {
            for (int g = 2 * warp; g < nr; g += 2 * NCW) {
                float acc[2][2];
                dot_rows<TYPE, D16, PAIR, 2>(sq + (size_t)g * qrow, sd + g * drow, sq2 + (size_t)g * qrow,
                                             sd2 + g * drow, qrow, drow, min(2, nr - g), 0, 1, nch, x, lane, acc);
                if (lane == 0) {
                    epilogue(e, ra + g, acc[0][0], acc[0][1], best);
                    if (g + 1 < nr) epilogue(e, ra + g + 1, acc[1][0], acc[1][1], best);
                }
            }
            __syncwarp();
            if (threadIdx.x == 0) ev(0, EV_STAGE_DONE);
            if (lane == 0) mbar_arrive(&rg.empty[slot]);
        } else if (R >= NCW) {
            for (int g = warp; g < nr; g += NCW) {
                float acc[1][2];
                dot_rows<TYPE, D16, PAIR, 1>(sq + (size_t)g * qrow, sd + g * drow, sq2 + (size_t)g * qrow,
                                             sd2 + g * drow, qrow, drow, 1, 0, 1, nch, x, lane, acc);
                if (lane == 0) epilogue(e, ra + g, acc[0][0], acc[0][1], best);
            }
            __syncwarp();
            if (threadIdx.x == 0) ev(0, EV_STAGE_DONE);
            if (lane == 0) mbar_arrive(&rg.empty[slot]);
        } else {
            const int G = NCW / R, r = warp / G, gg = warp % G;
            float *ps = psum + (rg.idx & 1) * 128;
            if (r < nr) {
                float acc[1][2];
                dot_rows<TYPE, D16, PAIR, 1>(sq + (size_t)r * qrow, sd + r * drow, sq2 + (size_t)r * qrow,
                                             sd2 + r * drow, qrow, drow, 1, gg, G, nch, x, lane, acc);
                if (lane == 0) {
                    ps[r * G + gg] = acc[0][0];
                    ps[64 + r * G + gg] = acc[0][1];
                }
            }
            __syncwarp();
            if (threadIdx.x == 0) ev(0, EV_STAGE_DONE);
            if (lane == 0) mbar_arrive(&rg.empty[slot]);
            consumer_sync();
            const int t = threadIdx.x;
            if (t < nr) {
                float acc = 0.0f, acc2 = 0.0f;
                for (int k = 0; k < G; k++) {   /* a fixed order: the result does not depend on timing */
                    acc += ps[t * G + k];
                    acc2 += ps[64 + t * G + k];
                }
                epilogue(e, ra + t, acc, acc2, best);
            }
        }
        rg.idx++;
    }
}

__device__ __forceinline__ void consume(Ring &rg, const PMat &m, const PMat *m2, int cols, int r0, int r1,
                                        const Epi &e, const Act &x, float *psum, unsigned *err,
                                        unsigned long long &best) {
    if (m.type == T_Q4) {
        if (m2) {
            if (m.d16) consume_rows<T_Q4, true, true>(rg, cols, r0, r1, e, x, psum, err, best);
            else consume_rows<T_Q4, false, true>(rg, cols, r0, r1, e, x, psum, err, best);
        } else {
            if (m.d16) consume_rows<T_Q4, true, false>(rg, cols, r0, r1, e, x, psum, err, best);
            else consume_rows<T_Q4, false, false>(rg, cols, r0, r1, e, x, psum, err, best);
        }
    } else {
        if (m2) {
            if (m.d16) consume_rows<T_Q8, true, true>(rg, cols, r0, r1, e, x, psum, err, best);
            else consume_rows<T_Q8, false, true>(rg, cols, r0, r1, e, x, psum, err, best);
        } else {
            if (m.d16) consume_rows<T_Q8, true, false>(rg, cols, r0, r1, e, x, psum, err, best);
            else consume_rows<T_Q8, false, false>(rg, cols, r0, r1, e, x, psum, err, best);
        }
    }
}

/* ------------------------------------------------------------ activations */

enum { SRC_GLOBAL = 0, SRC_EMBED = 1, SRC_PREQUANT = 2 };

constexpr int ACT_MAXP = 4;   /* passes of 64 blocks a thread keeps in registers (cols <= 8192) */

/* The activation of a phase into shared memory (xq, xd, xs): quantize_q8 of
 * v, with v = RMSNorm(x) * w (k_scalar.c:59-64: o = (x * inv) * w, inv =
 * 1 / sqrt(ss / n + eps)) when norm_w is set. The source: a float vector in
 * global memory written by other CTAs (read through L2), the embedding row of
 * token tok (dequantized, times embed_scale), or an already quantized vector
 * (pq, pd). 1/rms: inv_given when > 0, else from ss = the sum of the G
 * per-CTA partial sums ssp (the residual epilogues' x^2, added in CTA order),
 * else reduced here. Each thread loads all its values before using any. */
__device__ __noinline__ void load_activation(const StepArgs &a, int src, const float *x, int tok, const float *norm_w, float inv_given,
                                const float *ssp, int cols, const int8_t *pq, const float *pd, int8_t *xq, float *xd,
                                int *xs, float *red) {
    const int nb = cols / QK, tid = threadIdx.x;
    if (src == SRC_PREQUANT) {
        for (int i = tid; i < cols / 16; i += NCT) ((int4 *)xq)[i] = __ldcg((const int4 *)pq + i);
        for (int b = tid; b < nb; b += NCT) xd[b] = __ldcg(pd + b);
        consumer_sync();
        for (int b = tid; b < nb; b += NCT) {
            const int4 *q4 = (const int4 *)(xq + b * QK);
            int sum = 0;
            for (int k = 0; k < 2; k++) {
                const int4 w = q4[k];
                sum = __dp4a(w.x, 0x01010101, sum);
                sum = __dp4a(w.y, 0x01010101, sum);
                sum = __dp4a(w.z, 0x01010101, sum);
                sum = __dp4a(w.w, 0x01010101, sum);
            }
            xs[b] = 8 * sum;
        }
        consumer_sync();
        return;
    }
    auto load4 = [&](int i, float v[4]) {
        if (src == SRC_GLOBAL) {
            const float4 t = __ldcg((const float4 *)(x + i));
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
            const int b = i / QK, j = i % QK;
            const float sc = a.emb.d16 ? __half2float(((const __half *)a.emb.d)[(size_t)tok * nb + b])
                                       : ((const float *)a.emb.d)[(size_t)tok * nb + b];
            if (a.emb.type == T_Q8) {
                const char4 q4 = *(const char4 *)((const int8_t *)a.emb.q + (size_t)tok * cols + i);
                v[0] = __fmul_rn((float)q4.x, sc); v[1] = __fmul_rn((float)q4.y, sc);
                v[2] = __fmul_rn((float)q4.z, sc); v[3] = __fmul_rn((float)q4.w, sc);
            } else {
                const uchar4 p = *(const uchar4 *)(a.emb.q + ((size_t)tok * nb + b) * (QK / 2) + (j & 15));
                const bool hi = j >= 16;
                v[0] = __fmul_rn((float)((hi ? p.x >> 4 : p.x & 15) - 8), sc);
                v[1] = __fmul_rn((float)((hi ? p.y >> 4 : p.y & 15) - 8), sc);
                v[2] = __fmul_rn((float)((hi ? p.z >> 4 : p.z & 15) - 8), sc);
                v[3] = __fmul_rn((float)((hi ? p.w >> 4 : p.w & 15) - 8), sc);
            }
            if (a.embed_scale != 1.0f)
                for (int k = 0; k < 4; k++) v[k] = __fmul_rn(v[k], a.embed_scale);
        }
    };
    constexpr int per_pass = NCT / 8;   /* blocks per pass: 8 lanes x 4 values each */
    const int passes = (nb + per_pass - 1) / per_pass;
    const int j0 = (tid & 7) * 4;
    float v[ACT_MAXP][4];
    float4 wv[ACT_MAXP];
    const bool cached = passes <= ACT_MAXP;
    if (cached) {
#pragma unroll
        for (int p = 0; p < ACT_MAXP; p++) {
            const int b = p * per_pass + tid / 8;
            if (p < passes && b < nb) {
                load4(b * QK + j0, v[p]);
                if (norm_w) wv[p] = *(const float4 *)(norm_w + b * QK + j0);
            } else {
                v[p][0] = v[p][1] = v[p][2] = v[p][3] = 0.0f;
            }
        }
    }
    float inv = inv_given;
    if (norm_w && !(inv_given > 0.0f)) {
        if (ssp) {
            if (tid < 32) {
                float t = 0.0f;
                for (int k = tid; k < gridDim.x; k += 32) t += __ldcg(ssp + k);
                t = warp_sum(t);
                if (tid == 0) red[0] = t;
            }
            consumer_sync();
        } else {
            float ss = 0.0f;
            if (cached) {
#pragma unroll
                for (int p = 0; p < ACT_MAXP; p++)
                    ss += v[p][0] * v[p][0] + v[p][1] * v[p][1] + v[p][2] * v[p][2] + v[p][3] * v[p][3];
            } else {
                for (int i = tid * 4; i < cols; i += NCT * 4) {
                    float t[4];
                    load4(i, t);
                    ss += t[0] * t[0] + t[1] * t[1] + t[2] * t[2] + t[3] * t[3];
                }
            }
            block_sum(ss, red);
        }
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], (float)cols), a.eps)));
    }
    for (int p = 0; p < passes; p++) {
        const int b = p * per_pass + tid / 8;
        float u[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
        float4 w4 = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        if (b < nb) {
            if (cached) {
#pragma unroll
                for (int pp = 0; pp < ACT_MAXP; pp++)
                    if (pp == p) { u[0] = v[pp][0]; u[1] = v[pp][1]; u[2] = v[pp][2]; u[3] = v[pp][3]; if (norm_w) w4 = wv[pp]; }
            } else {
                load4(b * QK + j0, u);
                if (norm_w) w4 = *(const float4 *)(norm_w + b * QK + j0);
            }
            if (norm_w) {
                u[0] = __fmul_rn(__fmul_rn(u[0], inv), w4.x);
                u[1] = __fmul_rn(__fmul_rn(u[1], inv), w4.y);
                u[2] = __fmul_rn(__fmul_rn(u[2], inv), w4.z);
                u[3] = __fmul_rn(__fmul_rn(u[3], inv), w4.w);
            }
        }
        float d;
        int sum;
        const unsigned word = quant4(u, &d, &sum);
        if (b < nb) {
            ((unsigned *)xq)[(b * QK + j0) / 4] = word;
            if ((tid & 7) == 0) {
                xd[b] = d;
                xs[b] = 8 * sum;
            }
        }
    }
    consumer_sync();
}

/* The sum of squares of the rows [r0, r1) of x this CTA has just written
 * into ssp[blockIdx.x]: the next RMSNorm adds the G partial sums instead of
 * reading all of x before it can scale any of it. */
__device__ __forceinline__ void publish_ssq(const StepArgs &a, int r0, int r1, float *red) {
    consumer_sync();
    float t = 0.0f;
    for (int r = r0 + (int)threadIdx.x; r < r1; r += NCT) {
        const float v = __ldcg(a.x + r);
        t += v * v;
    }
    t = block_sum(t, red);
    if (threadIdx.x == 0) a.ssp[blockIdx.x] = t;
}

/* ------------------------------------------------------------ attention */

/* Shared scratch of an attention item, in floats. */
__host__ __device__ inline int attention_scratch_floats(int group, int hd) {
    return group * hd + ATT_TILE * (hd + 1) + ATT_TILE * hd + group * ATT_TILE + 3 * group;
}

/* Attention work item (KV head g, split y) of layer L at position pos (F32
 * cache), on the consumer threads; fsm: shared scratch. RoPE on adjacent pairs
 * (k_scalar.c:79-94); the split holding pos first writes that position's K
 * (after RoPE) and V into the cache; scores q.k * scale (soft-capped when
 * set), online softmax and the weighted V sum over the split's positions; the
 * last CTA of the KV head to finish combines the splits into a.ao. */
__device__ void attention_item(const StepArgs &a, const LayerPlan &L, int g, int y, int pos, float *fsm, int *flag) {
    const int hd = a.hd, group = a.n_heads / a.n_kv_heads, h2 = hd / 2, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int first = L.window && pos >= L.window ? pos + 1 - L.window : 0;
    const int n = pos + 1 - first;
    int C = (n + a.nsplit - 1) / a.nsplit;
    C = C < ATT_TILE ? ATT_TILE : (C + ATT_TILE - 1) / ATT_TILE * ATT_TILE;
    const int active = (n + C - 1) / C;
    if (y >= active) return;
    const int t_begin = first + y * C, t_end = min(t_begin + C, pos + 1);
    float *sq = fsm, *sk = sq + group * hd, *sv = sk + ATT_TILE * (hd + 1), *sp = sv + ATT_TILE * hd;
    float *sm = sp + group * ATT_TILE, *sl = sm + group, *sa = sl + group;
    const float *cs = L.rcos + (size_t)pos * h2, *sn = L.rsin + (size_t)pos * h2;
    for (int idx = tid; idx < group * h2; idx += NCT) {
        const int h = idx / h2, i = idx % h2;
        const float *qh = a.qkv + (size_t)(g * group + h) * hd;
        const float qa = __ldcg(qh + 2 * i), qb = __ldcg(qh + 2 * i + 1), c = cs[i], s = sn[i];
        sq[h * hd + 2 * i] = __fsub_rn(__fmul_rn(qa, c), __fmul_rn(qb, s));
        sq[h * hd + 2 * i + 1] = __fadd_rn(__fmul_rn(qa, s), __fmul_rn(qb, c));
    }
    if (t_end == pos + 1) {
        const float *kn = a.qkv + a.q_dim + (size_t)g * hd, *vn = a.qkv + a.q_dim + a.kv_dim + (size_t)g * hd;
        float *kr = L.kc + (size_t)pos * a.kv_dim + (size_t)g * hd, *vr = L.vc + (size_t)pos * a.kv_dim + (size_t)g * hd;
        for (int i = tid; i < h2; i += NCT) {
            const float ka = __ldcg(kn + 2 * i), kb = __ldcg(kn + 2 * i + 1), c = cs[i], s = sn[i];
            kr[2 * i] = __fsub_rn(__fmul_rn(ka, c), __fmul_rn(kb, s));
            kr[2 * i + 1] = __fadd_rn(__fmul_rn(ka, s), __fmul_rn(kb, c));
        }
        for (int i = tid; i < hd; i += NCT) vr[i] = __ldcg(vn + i);
    }
    if (tid < group) {
        sm[tid] = -INFINITY;
        sl[tid] = 0.0f;
    }
    const int nout = group * hd;
    constexpr int MAXO = (ATT_MAX_OUT + NCT - 1) / NCT;
    float acc[MAXO];
#pragma unroll
    for (int k = 0; k < MAXO; k++) acc[k] = 0.0f;
    consumer_sync();
    for (int t0 = t_begin; t0 < t_end; t0 += ATT_TILE) {
        const int nt = min(ATT_TILE, t_end - t0), h4 = hd / 4;
        for (int idx = tid; idx < nt * h4; idx += NCT) {
            const int t = idx / h4, c4 = idx % h4;
            const size_t off = (size_t)(t0 + t) * a.kv_dim + (size_t)g * hd + 4 * c4;
            const float4 kv = __ldcg((const float4 *)(L.kc + off));
            const float4 vv = __ldcg((const float4 *)(L.vc + off));
            float *kd = sk + t * (hd + 1) + 4 * c4;
            kd[0] = kv.x; kd[1] = kv.y; kd[2] = kv.z; kd[3] = kv.w;
            *(float4 *)(sv + t * hd + 4 * c4) = vv;
        }
        consumer_sync();
        for (int idx = tid; idx < group * ATT_TILE; idx += NCT) {
            const int h = idx / ATT_TILE, t = idx % ATT_TILE;
            float s = -INFINITY;
            if (t < nt) {
                const float *qh = sq + h * hd, *kt = sk + t * (hd + 1);
                float dot = 0.0f;
                for (int i = 0; i < hd; i++) dot = fmaf(qh[i], kt[i], dot);
                s = __fmul_rn(dot, a.attn_scale);
                if (a.attn_softcap > 0.0f) s = __fmul_rn(a.attn_softcap, tanhf(__fdiv_rn(s, a.attn_softcap)));
            }
            sp[h * ATT_TILE + t] = s;
        }
        consumer_sync();
        for (int h = warp; h < group; h += NCW) {
            const float s = sp[h * ATT_TILE + lane];
            const float m_old = sm[h], m_new = fmaxf(m_old, warp_max(s));
            const float pr = lane < nt ? expf(s - m_new) : 0.0f;
            const float sum = warp_sum(pr);
            const float alpha = expf(m_old - m_new);
            sp[h * ATT_TILE + lane] = pr;
            if (lane == 0) {
                sm[h] = m_new;
                sl[h] = sl[h] * alpha + sum;
                sa[h] = alpha;
            }
        }
        consumer_sync();
#pragma unroll
        for (int k = 0; k < MAXO; k++) {
            const int o = tid + k * NCT;
            if (o < nout) {
                const int h = o / hd, i = o % hd;
                float v = acc[k] * sa[h];
                const float *ph = sp + h * ATT_TILE;
                for (int t = 0; t < nt; t++) v = fmaf(ph[t], sv[t * hd + i], v);
                acc[k] = v;
            }
        }
        consumer_sync();
    }
    const int stride = hd + 2;
#pragma unroll
    for (int k = 0; k < MAXO; k++) {
        const int o = tid + k * NCT;
        if (o < nout) {
            const int h = o / hd, i = o % hd;
            a.part[((size_t)(g * group + h) * a.nsplit + y) * stride + i] = acc[k];
        }
    }
    if (tid < group) {
        float *ph = a.part + ((size_t)(g * group + tid) * a.nsplit + y) * stride;
        ph[hd] = sm[tid];
        ph[hd + 1] = sl[tid];
    }
    __threadfence();
    consumer_sync();
    if (tid == 0) *flag = atomicAdd(&a.att_counter[g], 1u) == (unsigned)active - 1;
    consumer_sync();
    if (!*flag) return;
    __threadfence();
    float *wts = sp;   /* [group][ATT_TILE >= nsplit] */
    for (int h = warp; h < group; h += NCW) {
        const float *ph = a.part + (size_t)(g * group + h) * a.nsplit * stride;
        const float m = lane < active ? __ldcg(ph + (size_t)lane * stride + hd) : -INFINITY;
        const float l = lane < active ? __ldcg(ph + (size_t)lane * stride + hd + 1) : 0.0f;
        const float M = warp_max(m);
        const float e = lane < active ? expf(m - M) : 0.0f;
        const float Ls = warp_sum(l * e);
        wts[h * ATT_TILE + lane] = e / Ls;
    }
    consumer_sync();
    for (int o = tid; o < nout; o += NCT) {
        const int h = o / hd, i = o % hd;
        const float *base = a.part + (size_t)(g * group + h) * a.nsplit * stride + i;
        const float *w = wts + h * ATT_TILE;
        float num = 0.0f;
#pragma unroll 8
        for (int s2 = 0; s2 < active; s2++) num = fmaf(__ldcg(base + (size_t)s2 * stride), w[s2], num);
        a.ao[(size_t)(g * group + h) * hd + i] = num;
    }
    if (tid == 0) a.att_counter[g] = 0u;
}

/* ------------------------------------------------------------ shared layout */

/* Dynamic shared memory of a streaming CTA: mbarriers [2][nstage], psum
 * [2][128], per-warp argmax [NCW], flag, reduction scratch [32], activation
 * (or attention scratch) of act_bytes, then the ring (128 B aligned). */
struct Smem {
    uint64_t *full, *empty;
    float *psum;
    unsigned long long *cta_best;
    int *flag;
    float *red;
    unsigned char *act;
    uint8_t *ring;
};

__host__ __device__ inline int smem_fixed_bytes(int nstage, int act_bytes) {
    return 16 * nstage + 1024 + 8 * NCW + 16 + 128 + act_bytes + 128;
}

__device__ __forceinline__ Smem carve(unsigned char *smem, int nstage, int act_bytes) {
    Smem s;
    s.full = (uint64_t *)smem;
    s.empty = s.full + nstage;
    s.psum = (float *)(smem + 16 * nstage);
    s.cta_best = (unsigned long long *)(s.psum + 256);
    s.flag = (int *)(s.cta_best + NCW);
    s.red = (float *)(s.flag + 4);
    s.act = (unsigned char *)(s.red + 32);
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

__device__ void producer(const StepArgs &a, Ring rg) {
    const int j = blockIdx.x, G = gridDim.x;
    int r0, r1;
    for (int s = 0; s < a.nsteps; s++) {
        for (int l = 0; l < a.n_layers; l++) {
            const LayerPlan &L = a.layers[l];
            share_rows(L.wq.rows, j, G, r0, r1); produce_rows(rg, L.wq, nullptr, a.dim, r0, r1, a.err);
            share_rows(L.wk.rows, j, G, r0, r1); produce_rows(rg, L.wk, nullptr, a.dim, r0, r1, a.err);
            share_rows(L.wv.rows, j, G, r0, r1); produce_rows(rg, L.wv, nullptr, a.dim, r0, r1, a.err);
            share_rows(L.wo.rows, j, G, r0, r1); produce_rows(rg, L.wo, nullptr, a.q_dim, r0, r1, a.err);
            share_rows(L.w1.rows, j, G, r0, r1); produce_rows(rg, L.w1, &L.w3, a.dim, r0, r1, a.err);
            share_rows(L.w2.rows, j, G, r0, r1); produce_rows(rg, L.w2, nullptr, a.hidden, r0, r1, a.err);
        }
        if (a.run_cls) {
            share_rows(a.cls.rows, j, G, r0, r1);
            produce_rows(rg, a.cls, nullptr, a.dim, r0, r1, a.err);
        }
    }
}

__global__ void __launch_bounds__(STEP_THREADS, 1) step_kernel(const __grid_constant__ StepArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const Smem sh = carve(smem, a.nstage, a.act_bytes);
    ev_init(true);
    init_ring(sh, a.nstage);
    Ring rg{ sh.full, sh.empty, sh.ring, a.nstage, a.slot_bytes, 0u };
    if ((threadIdx.x >> 5) == NCW) {
        if ((threadIdx.x & 31) == 0) producer(a, rg);
        return;
    }
    const int j = blockIdx.x, G = gridDim.x;
    unsigned expect = 0;
    int8_t *xq = (int8_t *)sh.act;
    if (threadIdx.x == 0) timeline_mark(a);
    for (int step = 0; step < a.nsteps; step++) {
        const int tok = __ldcg(&a.ls->token), pos = __ldcg(&a.ls->pos);
        const bool ok = tok >= 0 && tok < a.vocab && pos >= 0 && pos < a.max_seq;
        if (!ok && threadIdx.x == 0) atomicOr(&a.ls->err, 1u);
        const int tk = ok ? tok : 0, ps = ok ? pos : 0;
        const int logit_row0 = (__ldcg(&a.ls->step) % LOGITS_RING) * a.vocab;
        unsigned long long best = 0;
        int r0, r1;
        for (int l = 0; l < a.n_layers; l++) {
            const LayerPlan &L = a.layers[l];
            int cols = a.dim, nb = cols / QK;
            float *xd = (float *)(sh.act + cols);
            int *xs = (int *)(xd + nb);
            /* A: Q/K/V */
            if (l == 0) {
                load_activation(a, SRC_EMBED, nullptr, tk, L.attn_norm, a.inv0[tk], nullptr, cols, nullptr, nullptr, xq, xd, xs,
                                sh.red);
                /* the residual stream starts as the embedding row: this CTA's rows of x */
                share_rows(a.dim, j, G, r0, r1);
                for (int r = r0 + (int)threadIdx.x; r < r1; r += NCT) {
                    const int b = r / QK, jj = r % QK;
                    const float sc = a.emb.d16 ? __half2float(((const __half *)a.emb.d)[(size_t)tk * nb + b])
                                               : ((const float *)a.emb.d)[(size_t)tk * nb + b];
                    int v;
                    if (a.emb.type == T_Q8) {
                        v = ((const int8_t *)a.emb.q)[(size_t)tk * a.dim + r];
                    } else {
                        const uint8_t byte = a.emb.q[((size_t)tk * nb + b) * (QK / 2) + (jj & 15)];
                        v = (jj < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
                    }
                    float o = __fmul_rn((float)v, sc);
                    if (a.embed_scale != 1.0f) o = __fmul_rn(o, a.embed_scale);
                    a.x[r] = o;
                }
            } else {
                load_activation(a, SRC_GLOBAL, a.x, tk, L.attn_norm, 0.0f, a.ssp, cols, nullptr, nullptr, xq, xd, xs, sh.red);
            }
            trace_mark(a, expect / G, 0);
            if (threadIdx.x == 0) ev(0, EV_PRO_DONE);
            {
                const Act x{ xq, xd, xs };
                share_rows(L.wq.rows, j, G, r0, r1);
                consume(rg, L.wq, nullptr, cols, r0, r1, Epi{ EPI_STORE, a.qkv, L.bq, 0, 0.0f, 0 }, x, sh.psum, a.err, best);
                share_rows(L.wk.rows, j, G, r0, r1);
                consume(rg, L.wk, nullptr, cols, r0, r1, Epi{ EPI_STORE, a.qkv + a.q_dim, L.bk, 0, 0.0f, 0 }, x, sh.psum,
                        a.err, best);
                share_rows(L.wv.rows, j, G, r0, r1);
                consume(rg, L.wv, nullptr, cols, r0, r1, Epi{ EPI_STORE, a.qkv + a.q_dim + a.kv_dim, L.bv, 0, 0.0f, 0 }, x,
                        sh.psum, a.err, best);
            }
            grid_barrier(a, expect);
            /* B: attention */
            trace_mark(a, expect / G, 0);
            if (threadIdx.x == 0) ev(0, EV_PRO_DONE);
            for (int it = j; it < a.n_kv_heads * a.nsplit; it += G)
                attention_item(a, L, it / a.nsplit, it % a.nsplit, ps, (float *)sh.act, sh.flag);
            grid_barrier(a, expect);
            /* C: O projection + residual */
            cols = a.q_dim; nb = cols / QK;
            xd = (float *)(sh.act + cols); xs = (int *)(xd + nb);
            load_activation(a, SRC_GLOBAL, a.ao, tk, nullptr, 1.0f, nullptr, cols, nullptr, nullptr, xq, xd, xs, sh.red);
            trace_mark(a, expect / G, 0);
            if (threadIdx.x == 0) ev(0, EV_PRO_DONE);
            share_rows(L.wo.rows, j, G, r0, r1);
            consume(rg, L.wo, nullptr, cols, r0, r1, Epi{ EPI_RESID, a.x, nullptr, 0, 0.0f, 0 }, Act{ xq, xd, xs },
                    sh.psum, a.err, best);
            publish_ssq(a, r0, r1, sh.red);
            grid_barrier(a, expect);
            /* D: gate/up + activation */
            cols = a.dim; nb = cols / QK;
            xd = (float *)(sh.act + cols); xs = (int *)(xd + nb);
            load_activation(a, SRC_GLOBAL, a.x, tk, L.ffn_norm, 0.0f, a.ssp, cols, nullptr, nullptr, xq, xd, xs, sh.red);
            trace_mark(a, expect / G, 0);
            if (threadIdx.x == 0) ev(0, EV_PRO_DONE);
            share_rows(L.w1.rows, j, G, r0, r1);
            consume(rg, L.w1, &L.w3, cols, r0, r1, Epi{ EPI_PAIR, a.hb, nullptr, a.act, 0.0f, 0 }, Act{ xq, xd, xs },
                    sh.psum, a.err, best);
            grid_barrier(a, expect);
            /* E: down + residual */
            cols = a.hidden; nb = cols / QK;
            xd = (float *)(sh.act + cols); xs = (int *)(xd + nb);
            load_activation(a, SRC_GLOBAL, a.hb, tk, nullptr, 1.0f, nullptr, cols, nullptr, nullptr, xq, xd, xs, sh.red);
            trace_mark(a, expect / G, 0);
            if (threadIdx.x == 0) ev(0, EV_PRO_DONE);
            share_rows(L.w2.rows, j, G, r0, r1);
            consume(rg, L.w2, nullptr, cols, r0, r1, Epi{ EPI_RESID, a.x, nullptr, 0, 0.0f, 0 }, Act{ xq, xd, xs },
                    sh.psum, a.err, best);
            publish_ssq(a, r0, r1, sh.red);
            grid_barrier(a, expect);
        }
        /* F: classifier + argmax */
        if (a.run_cls) {
            const int cols = a.dim, nb = cols / QK;
            float *xd = (float *)(sh.act + cols);
            int *xs = (int *)(xd + nb);
            load_activation(a, SRC_GLOBAL, a.x, tk, a.final_norm, 0.0f, a.ssp, cols, nullptr, nullptr, xq, xd, xs, sh.red);
            trace_mark(a, expect / G, 0);
            if (threadIdx.x == 0) ev(0, EV_PRO_DONE);
            share_rows(a.cls.rows, j, G, r0, r1);
            consume(rg, a.cls, nullptr, cols, r0, r1, Epi{ EPI_LOGITS, a.logits, nullptr, 0, a.final_softcap, logit_row0 },
                    Act{ xq, xd, xs }, sh.psum, a.err, best);
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                best = other > best ? other : best;
            }
            if ((threadIdx.x & 31) == 0) sh.cta_best[threadIdx.x >> 5] = best;
            consumer_sync();
            if (threadIdx.x == 0) {
                unsigned long long b = 0;
                for (int w = 0; w < NCW; w++) b = sh.cta_best[w] > b ? sh.cta_best[w] : b;
                if (b) atomicMax(&a.ls->best, b);
            }
        }
        /* every CTA arrives; the last one advances the loop state, then
         * releases the others with one more arrival */
        consumer_sync();
        const unsigned pfin = expect / gridDim.x;
        expect += gridDim.x;
        if (threadIdx.x == 0) {
            trace_mark(a, pfin, 1);
            __threadfence();
            const unsigned prev = atomicAdd(a.bar, 1u);
            if (prev == expect - 1) {
                LoopState *ls = a.ls;
                const int st = ls->step;
                if (a.run_cls) {
                    const unsigned long long b = atomicAdd(&ls->best, 0ull);
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
 * kernel's producer and consumers over rows [0, rows), CTA j of G owning its
 * share, the activation copied in (SRC_PREQUANT). */
struct MatvecArgs {
    PMat m;
    int cols;
    const int8_t *xq;
    const float *xd;
    float *y;
    unsigned *err;
    int nstage, slot_bytes, act_bytes;
};

__global__ void __launch_bounds__(STEP_THREADS, 1) matvec_kernel(const __grid_constant__ MatvecArgs p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const Smem sh = carve(smem, p.nstage, p.act_bytes);
    ev_init(false);
    init_ring(sh, p.nstage);
    Ring rg{ sh.full, sh.empty, sh.ring, p.nstage, p.slot_bytes, 0u };
    int r0, r1;
    share_rows(p.m.rows, blockIdx.x, gridDim.x, r0, r1);
    if ((threadIdx.x >> 5) == NCW) {
        if ((threadIdx.x & 31) == 0) produce_rows(rg, p.m, nullptr, p.cols, r0, r1, p.err);
        return;
    }
    const int nb = p.cols / QK;
    int8_t *xq = (int8_t *)sh.act;
    float *xd = (float *)(sh.act + p.cols);
    int *xs = (int *)(xd + nb);
    StepArgs dummy{};
    load_activation(dummy, SRC_PREQUANT, nullptr, 0, nullptr, 1.0f, nullptr, p.cols, p.xq, p.xd, xq, xd, xs, sh.red);
    unsigned long long best = 0;
    consume(rg, p.m, nullptr, p.cols, r0, r1, Epi{ EPI_STORE, p.y, nullptr, 0, 0.0f, 0 }, Act{ xq, xd, xs }, sh.psum,
            p.err, best);
}

/* The activation prologue alone (kc_quantize_q8_dev, kc_rmsnorm_quantize_dev):
 * one CTA of consumer threads writes its shared arrays out. */
__global__ void __launch_bounds__(NCT, 1) activation_kernel(const float *x, const float *w, float eps, int n, int8_t *q,
                                                           float *d, float *xn) {
    extern __shared__ __align__(128) unsigned char smem[];
    float *red = (float *)smem;
    int8_t *xq = (int8_t *)(smem + 128);
    float *xd = (float *)(smem + 128 + n);
    int *xs = (int *)(xd + n / QK);
    StepArgs a{};
    a.eps = eps;
    load_activation(a, SRC_GLOBAL, x, 0, w, 0.0f, nullptr, n, nullptr, nullptr, xq, xd, xs, red);
    for (int i = threadIdx.x; i < n; i += NCT) q[i] = xq[i];
    for (int b = threadIdx.x; b < n / QK; b += NCT) d[b] = xd[b];
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
