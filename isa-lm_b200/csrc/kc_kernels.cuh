/* Device kernels of the decode token loop (sm_100a).
 *
 * Decode is HBM-bound: every weight byte is read once per token. The
 * projections run in one GEMV kernel with three parts:
 *   prologue  each CTA rebuilds the Q8_0 activation in shared memory from the
 *             float vector (RMSNorm first where the reference normalizes), with
 *             the reference's bit-exact rule (kernels/scalar/k_scalar.c:39-57);
 *   body      each warp streams whole weight rows with 16-byte non-allocating
 *             loads, int32 block dots by dp4a (exact), float scale-accumulate
 *             (k_scalar.c:4-37), warp-shuffle reduction;
 *   epilogue  fused per row: bias, residual add, SiLU/GELU * up, logits with
 *             the first-index argmax (model/sampler.c:57-61) and the device
 *             token-loop advance.
 * Attention is a split-K flash-decode kernel per KV head that also applies
 * RoPE and writes this position's K/V row (model/transformer.c:280-283,
 * ops/ops.c:124-155); the last CTA of each KV head combines the splits.
 */
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace kc {

constexpr int QK = 32;
constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int MAX_SEGS = 4;
constexpr int GEMV_NSTAGE = 4;          /* pipeline depth of the weight stream */
constexpr int GEMV_STAGE_Q = 16 * 1024;  /* bytes of quants per stage (at least one row) */
constexpr int ATT_THREADS = 128;
constexpr int ATT_TILE = 32;
constexpr int ATT_MAX_OUT = 16;   /* outputs per thread: group * head_dim <= 2048 */
constexpr int LOGITS_RING = 128;  /* logits rows kept on the device per call */

enum { T_Q8 = 1, T_Q4 = 2 };
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_PAIR = 2, EPI_LOGITS = 3 };
enum { PRO_PREQUANT = 0, PRO_QUANT = 1, PRO_RMSNORM_QUANT = 2 };

/* Device-resident token-loop state: one graph replays every step. */
struct LoopState {
    int token, pos, step, feed_mode;
    unsigned long long best;   /* argmax key: ordered logit << 32 | (~index) */
    unsigned done;             /* CTAs of the classifier that finished */
    unsigned err;              /* bit 0: token/pos out of range seen by a kernel */
};

struct Seg {
    const uint8_t *q;
    const void *d;
    const uint8_t *q2;   /* EPI_PAIR: the up matrix (w3) */
    const void *d2;
    const float *bias;
    float *out;
    int rows, type, d16, epi;
    int cta0, ctas;     /* the CTAs that work on this segment (rows split evenly among them) */
};

struct GemvParams {
    Seg seg[MAX_SEGS];
    int nseg, cols;
    int pro;
    const float *x;
    const float *norm_w;
    float eps;
    const int8_t *xq;   /* PRO_PREQUANT */
    const float *xd;
    const float *inv_tab;    /* PRO_RMSNORM_QUANT: when set, 1/rms of x is inv_tab[*inv_token] */
    const int *inv_token;
    int act;            /* EPI_PAIR: 0 SiLU, 1 GELU (tanh) */
    float softcap;      /* EPI_LOGITS: final soft-cap, 0 = none */
    LoopState *ls;      /* EPI_LOGITS */
    const int *feed;
    int *out_tokens;
    int vocab;
    unsigned *err;      /* bit 1: a bounded wait gave up */
};

struct AttnParams {
    const float *qkv;          /* q [q_dim] | k [kv_dim] | v [kv_dim] of this step, before RoPE */
    float *kc, *vc;            /* this layer's F32 cache [max_seq][kv_dim] */
    const float *rcos, *rsin;  /* [max_seq][head_dim/2] */
    float *ao;                 /* [q_dim] */
    float *part;               /* [n_heads][nsplit][head_dim + 2] */
    unsigned *counter;         /* [n_kv_heads], zero between launches */
    LoopState *ls;
    int n_heads, n_kv_heads, hd, q_dim, kv_dim, max_seq, window, nsplit;
    float scale, softcap;
};

/* ------------------------------------------------------------ helpers */

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <bool D16>
__device__ __forceinline__ float load_scale(const void *d, size_t i) {
    if constexpr (D16) {
        const unsigned short h = __ldg((const unsigned short *)d + i);
        return __half2float(__ushort_as_half(h));
    } else {
        return __ldg((const float *)d + i);
    }
}

/* Q4_0 block: byte j = element j (low nibble) | element j+16 (high nibble);
 * the nibbles n = w + 8 go through dp4a as they are and 8 * sum(x) is taken
 * off in int32 (exact). xlo/xhi: activation elements 0..15 / 16..31. */
__device__ __forceinline__ int dot_q4(uint4 w, int4 xlo, int4 xhi) {
    const unsigned m = 0x0F0F0F0Fu;
    int s = 0;
    s = __dp4a((int)(w.x & m), xlo.x, s);
    s = __dp4a((int)((w.x >> 4) & m), xhi.x, s);
    s = __dp4a((int)(w.y & m), xlo.y, s);
    s = __dp4a((int)((w.y >> 4) & m), xhi.y, s);
    s = __dp4a((int)(w.z & m), xlo.z, s);
    s = __dp4a((int)((w.z >> 4) & m), xhi.z, s);
    s = __dp4a((int)(w.w & m), xlo.w, s);
    s = __dp4a((int)((w.w >> 4) & m), xhi.w, s);
    return s;
}

/* Q8_0 half block: 16 int8 weights against 16 int8 activations. */
__device__ __forceinline__ int dot_q8(uint4 w, int4 x) {
    int s = 0;
    s = __dp4a((int)w.x, x.x, s);
    s = __dp4a((int)w.y, x.y, s);
    s = __dp4a((int)w.z, x.z, s);
    s = __dp4a((int)w.w, x.w, s);
    return s;
}

/* The reference's Q8_0 rule for 4 values held by each lane of an 8-lane group
 * (one block of 32): d = amax/127, q = trunc(x*(127/amax) + copysign(.5, x))
 * clamped to +-127, blocks with amax < 1e-30 -> 0. Every op is IEEE round to
 * nearest without contraction, as the reference builds with -ffp-contract=off.
 * Returns the 4 quants packed in a word; *d and *sum (sum of the 32 quants)
 * are valid on every lane of the group. */
__device__ __forceinline__ unsigned quant4(const float v[4], float *d, int *sum) {
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    unsigned word = 0;
    int s = 0;
    if (amax < 1e-30f) {
        *d = 0.0f;
    } else {
        const float id = __fdiv_rn(127.0f, amax);
        *d = __fdiv_rn(amax, 127.0f);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float t = truncf(__fadd_rn(__fmul_rn(v[i], id), copysignf(0.5f, v[i])));
            t = fminf(fmaxf(t, -127.0f), 127.0f);
            const int qi = (int)t;
            s += qi;
            word |= ((unsigned)qi & 0xffu) << (8 * i);
        }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    *sum = s;
    return word;
}

/* Named barrier of the GEMV_THREADS consumer threads (the GEMV's producer warp
 * never joins it; standalone kernels launch exactly GEMV_THREADS threads). */
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(GEMV_THREADS) : "memory"); }

/* Float sum over the consumer threads into red[0]. */
__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    consumer_sync();
    if (lane == 0) red[warp] = v;
    consumer_sync();
    if (warp == 0) {
        float t = lane < GEMV_WARPS ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    consumer_sync();
    return red[0];
}

/* Activation prologue (consumer threads): xq[cols] int8, xd[nb] scales, xs[nb]
 * = 8 * sum(block quants) in shared memory. RMSNorm (k_scalar.c:59-64):
 * o = (x * inv) * w with inv = 1 / sqrt(ss / n + eps), ss in tree order. */
__device__ __forceinline__ void gemv_prologue(const GemvParams &p, int8_t *xq, float *xd, int *xs, float *red) {
    const int cols = p.cols, nb = cols / QK, tid = threadIdx.x;
    if (p.pro == PRO_PREQUANT) {
        for (int i = tid; i < cols / 16; i += GEMV_THREADS) ((int4 *)xq)[i] = ((const int4 *)p.xq)[i];
        for (int b = tid; b < nb; b += GEMV_THREADS) xd[b] = p.xd[b];
        consumer_sync();
        for (int b = tid; b < nb; b += GEMV_THREADS) {
            int s = 0;
            for (int j = 0; j < QK; j++) s += xq[b * QK + j];
            xs[b] = 8 * s;
        }
        consumer_sync();
        return;
    }
    float inv = 1.0f;
    if (p.pro == PRO_RMSNORM_QUANT && p.inv_tab) {
        /* the first layer's input is an embedding row: its 1/rms was computed on
         * the host in the reference's sequential order (see embed_inv_table) */
        inv = p.inv_tab[*p.inv_token];
    } else if (p.pro == PRO_RMSNORM_QUANT) {
        float ss = 0.0f;
        for (int i = tid; i < cols / 4; i += GEMV_THREADS) {
            const float4 v = ((const float4 *)p.x)[i];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        ss = block_sum(ss, red);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), p.eps)));
    }
    constexpr int per_pass = GEMV_THREADS / 8;   /* blocks per pass: 8 lanes x 4 values each */
    for (int b0 = 0; b0 < nb; b0 += per_pass) {
        const int b = b0 + tid / 8, j0 = (tid & 7) * 4;
        float v[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
        if (b < nb) {
            const float4 xv = *(const float4 *)(p.x + b * QK + j0);
            v[0] = xv.x; v[1] = xv.y; v[2] = xv.z; v[3] = xv.w;
            if (p.pro == PRO_RMSNORM_QUANT) {
                const float4 wv = *(const float4 *)(p.norm_w + b * QK + j0);
                v[0] = __fmul_rn(__fmul_rn(v[0], inv), wv.x);
                v[1] = __fmul_rn(__fmul_rn(v[1], inv), wv.y);
                v[2] = __fmul_rn(__fmul_rn(v[2], inv), wv.z);
                v[3] = __fmul_rn(__fmul_rn(v[3], inv), wv.w);
            }
        }
        float d;
        int sum;
        const unsigned word = quant4(v, &d, &sum);
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

/* ---- mbarrier / bulk-copy primitives (PTX ISA: mbarrier, cp.async.bulk) ---- */

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
/* Waits for the phase with the given parity to complete; gives up (false)
 * after a bounded number of polls so that no wait can hang the GPU. */
__device__ __forceinline__ bool mbar_wait(uint64_t *b, unsigned parity) {
    const uint32_t a = smem_u32(b);
    for (unsigned it = 0; it < (1u << 22); it++) {
        unsigned ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}
/* Global -> shared bulk copy (16-byte aligned addresses and size) completing
 * on the mbarrier's transaction count. */
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

/* Stage geometry of a segment: R rows (a power of two, <= 64) per pipeline
 * stage with at most GEMV_STAGE_Q bytes of quants per stage (one row when a
 * row alone is larger); qbytes / dbytes: the quant and scale room of one
 * matrix in a stage (the scales with 16 bytes of alignment slack). */
__host__ __device__ inline void stage_geom(int type, int d16, int cols, int pair, int &R, int &qbytes, int &dbytes) {
    const int qrow = type == T_Q4 ? cols / 2 : cols, drow = (cols / QK) * (d16 ? 2 : 4);
    const int unit = qrow * (pair ? 2 : 1);
    R = 1;
    while (R * 2 <= 64 && R * 2 * unit <= GEMV_STAGE_Q) R *= 2;
    qbytes = R * qrow;
    dbytes = (R * drow + 16 + 15) & ~15;
}
__host__ __device__ inline int stage_slot_bytes(int type, int d16, int cols, int pair) {
    int R, qb, db;
    stage_geom(type, d16, cols, pair, R, qb, db);
    return (((qb + db) * (pair ? 2 : 1)) + 127) & ~127;
}

/* Partial dot of one weight row held in shared memory (qr: quants, dr: its
 * scales) over the 32-chunk slices s0, s0 + sstep, ... of the row; chunks are
 * 16 bytes (a Q4 block or half a Q8 block). Exact int32 block sums, float
 * scale-accumulate as (float)s * d_w * d_x (k_scalar.c:4-37). Warp-reduced. */
template <int TYPE, bool D16, bool PAIR>
__device__ __forceinline__ void slice_dot(const uint8_t *qr, const uint8_t *dr, const uint8_t *qr2, const uint8_t *dr2,
                                          int s0, int sstep, int nch, const int8_t *xq, const float *xd,
                                          const int *xs, int lane, float &out0, float &out1) {
    constexpr int CPB = TYPE == T_Q4 ? 1 : 2;
    const int4 *x4 = (const int4 *)xq;
    float a0 = 0.0f, a1 = 0.0f;
    for (int s = s0; s * 32 < nch; s += sstep) {
        const int c = s * 32 + lane;
        const bool ok = c < nch;
        const int b = c / CPB;
        if constexpr (TYPE == T_Q4) {
            if (ok) {
                const int4 xlo = x4[2 * b], xhi = x4[2 * b + 1];
                const float dx = xd[b];
                const int corr = xs[b];
                const uint4 w = *(const uint4 *)(qr + 16 * c);
                float dw;
                if constexpr (D16) dw = __half2float(((const __half *)dr)[b]);
                else dw = ((const float *)dr)[b];
                a0 += __fmul_rn((float)(dot_q4(w, xlo, xhi) - corr), dw) * dx;
                if constexpr (PAIR) {
                    const uint4 w2 = *(const uint4 *)(qr2 + 16 * c);
                    float dw2;
                    if constexpr (D16) dw2 = __half2float(((const __half *)dr2)[b]);
                    else dw2 = ((const float *)dr2)[b];
                    a1 += __fmul_rn((float)(dot_q4(w2, xlo, xhi) - corr), dw2) * dx;
                }
            }
        } else {
            const int4 xv = ok ? x4[c] : make_int4(0, 0, 0, 0);
            int t0 = ok ? dot_q8(*(const uint4 *)(qr + 16 * c), xv) : 0;
            int t1 = 0;
            if constexpr (PAIR) t1 = ok ? dot_q8(*(const uint4 *)(qr2 + 16 * c), xv) : 0;
            t0 += __shfl_xor_sync(0xffffffffu, t0, 1);   /* both halves of the block */
            if constexpr (PAIR) t1 += __shfl_xor_sync(0xffffffffu, t1, 1);
            if (ok && !(lane & 1)) {
                const float dx = xd[b];
                float dw;
                if constexpr (D16) dw = __half2float(((const __half *)dr)[b]);
                else dw = ((const float *)dr)[b];
                a0 += __fmul_rn((float)t0, dw) * dx;
                if constexpr (PAIR) {
                    float dw2;
                    if constexpr (D16) dw2 = __half2float(((const __half *)dr2)[b]);
                    else dw2 = ((const float *)dr2)[b];
                    a1 += __fmul_rn((float)t1, dw2) * dx;
                }
            }
        }
    }
    out0 = warp_sum(a0);
    out1 = PAIR ? warp_sum(a1) : 0.0f;
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    unsigned u = __float_as_uint(v == 0.0f ? 0.0f : v);   /* -0 and +0 compare equal */
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (unsigned)idx);
}

__device__ __forceinline__ float act_mul(int act, float g, float u) {
    if (act == 1) {   /* GELU, tanh form (k_scalar.c:100-105) */
        const float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, g), g), g);
        const float t = tanhf(__fmul_rn(0.7978845608f, __fadd_rn(g, x3)));
        return __fmul_rn(__fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, t)), u);
    }
    /* SiLU * up (k_scalar.c:96-98): g / (1 + exp(-g)) * u */
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

/* The consumer side of one CTA for a segment of fixed type/scale format. */
template <int TYPE, bool D16, bool PAIR>
__device__ __forceinline__ void gemv_consume(const GemvParams &p, const Seg &sg, int r_begin, int r_end, uint64_t *full,
                                             uint64_t *empty, uint8_t *ring, int slot_bytes, const int8_t *xq,
                                             const float *xd, const int *xs, float *psum, unsigned long long &best,
                                             int logit_row0) {
    const int cols = p.cols, nb = cols / QK, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int CPB = TYPE == T_Q4 ? 1 : 2;
    const int nch = nb * CPB;
    const int qrow = TYPE == T_Q4 ? cols / 2 : cols, drow = nb * (D16 ? 2 : 4);
    int R, qbytes, dbytes;
    stage_geom(TYPE, D16, cols, PAIR, R, qbytes, dbytes);
    const int G = R >= GEMV_WARPS ? 1 : GEMV_WARPS / R;   /* warps per row */
    const int nst = (r_end - r_begin + R - 1) / R;
    for (int st = 0; st < nst; st++) {
        const int slot = st % GEMV_NSTAGE;
        if (!mbar_wait(&full[slot], (unsigned)(st / GEMV_NSTAGE) & 1u) && lane == 0) atomicOr(p.err, 2u);
        const int ra = r_begin + st * R, nr = min(R, r_end - ra);
        const uint8_t *sq = ring + (size_t)slot * slot_bytes;
        const uint8_t *sd = sq + qbytes;
        const int doff = (int)(((size_t)ra * drow) & 15);
        const uint8_t *sq2 = sq + qbytes + dbytes, *sd2 = sq2 + qbytes;
        float *ps = psum + (st & 1) * 128;
        if (G == 1) {
            for (int r = warp; r < nr; r += GEMV_WARPS) {
                float a0, a1;
                slice_dot<TYPE, D16, PAIR>(sq + (size_t)r * qrow, sd + doff + r * drow, sq2 + (size_t)r * qrow,
                                           sd2 + doff + r * drow, 0, 1, nch, xq, xd, xs, lane, a0, a1);
                if (lane == 0) {
                    ps[r] = a0;
                    ps[64 + r] = a1;
                }
            }
        } else {
            const int r = warp / G, g = warp % G;
            if (r < nr) {
                float a0, a1;
                slice_dot<TYPE, D16, PAIR>(sq + (size_t)r * qrow, sd + doff + r * drow, sq2 + (size_t)r * qrow,
                                           sd2 + doff + r * drow, g, G, nch, xq, xd, xs, lane, a0, a1);
                if (lane == 0) {
                    ps[r * G + g] = a0;
                    ps[64 + r * G + g] = a1;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);   /* the slot's bytes are no longer read */
        consumer_sync();
        const int t = threadIdx.x;
        if (t < nr) {
            float acc = 0.0f, acc2 = 0.0f;
            for (int g = 0; g < G; g++) {   /* fixed order: the result does not depend on timing */
                acc += ps[t * G + g];
                acc2 += ps[64 + t * G + g];
            }
            const int row = ra + t;
            switch (sg.epi) {
            case EPI_STORE: sg.out[row] = sg.bias ? __fadd_rn(acc, sg.bias[row]) : acc; break;
            case EPI_RESID: sg.out[row] = __fadd_rn(sg.out[row], acc); break;
            case EPI_PAIR: sg.out[row] = act_mul(p.act, acc, acc2); break;
            case EPI_LOGITS: {
                float v = acc;
                if (p.softcap > 0.0f) v = __fmul_rn(p.softcap, tanhf(__fdiv_rn(v, p.softcap)));
                sg.out[logit_row0 + row] = v;
                const unsigned long long k = argmax_key(v, row);
                best = k > best ? k : best;
                break;
            }
            }
        }
    }
}

/* Decode GEMV: GEMV_WARPS consumer warps + 1 producer warp per CTA. Each CTA
 * owns a contiguous range of rows of one segment; the producer streams its
 * quants and scales through a GEMV_NSTAGE-deep shared-memory ring with bulk
 * copies while the consumers build the activation and compute. */
__global__ void __launch_bounds__(GEMV_THREADS + 32, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int cols = p.cols, nb = cols / QK;
    uint64_t *full = (uint64_t *)smem, *empty = full + GEMV_NSTAGE;
    float *psum = (float *)(smem + 16 * GEMV_NSTAGE);                 /* [2][128] */
    unsigned long long *cta_best = (unsigned long long *)(psum + 256); /* [GEMV_WARPS] */
    int *is_last = (int *)(cta_best + GEMV_WARPS);
    float *red = (float *)(is_last + 4);                               /* [32] */
    int8_t *xq = (int8_t *)(red + 32);
    float *xd = (float *)((unsigned char *)xq + cols);
    int *xs = (int *)(xd + nb);
    uint8_t *ring = (uint8_t *)(((uintptr_t)(xs + nb) + 127) & ~(uintptr_t)127);

    int si = 0;
    while (si + 1 < p.nseg && (int)blockIdx.x >= p.seg[si + 1].cta0) si++;
    const Seg &sg = p.seg[si];
    const int j = (int)blockIdx.x - sg.cta0;
    const int r_begin = (int)((long long)sg.rows * j / sg.ctas), r_end = (int)((long long)sg.rows * (j + 1) / sg.ctas);
    const int pair = sg.epi == EPI_PAIR;
    int slot_bytes = 0;
    for (int i = 0; i < p.nseg; i++) {
        const int b = stage_slot_bytes(p.seg[i].type, p.seg[i].d16, cols, p.seg[i].epi == EPI_PAIR);
        slot_bytes = b > slot_bytes ? b : slot_bytes;
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < GEMV_NSTAGE; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], GEMV_WARPS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == GEMV_WARPS) {   /* producer */
        if (lane == 0) {
            int R, qbytes, dbytes;
            stage_geom(sg.type, sg.d16, cols, pair, R, qbytes, dbytes);
            const int qrow = sg.type == T_Q4 ? cols / 2 : cols, drow = nb * (sg.d16 ? 2 : 4);
            const int nst = (r_end - r_begin + R - 1) / R;
            for (int st = 0; st < nst; st++) {
                const int slot = st % GEMV_NSTAGE;
                if (st >= GEMV_NSTAGE && !mbar_wait(&empty[slot], (unsigned)(st / GEMV_NSTAGE - 1) & 1u))
                    atomicOr(p.err, 2u);
                const int ra = r_begin + st * R, nr = min(R, r_end - ra);
                const size_t ds = (size_t)ra * drow, de = (size_t)(ra + nr) * drow;
                const size_t das = ds & ~(size_t)15, dae = (de + 15) & ~(size_t)15;
                const unsigned qb = (unsigned)(nr * qrow), db = (unsigned)(dae - das);
                uint8_t *dst = ring + (size_t)slot * slot_bytes;
                mbar_expect_tx(&full[slot], (qb + db) * (pair ? 2u : 1u));
                bulk_g2s(dst, sg.q + (size_t)ra * qrow, qb, &full[slot]);
                bulk_g2s(dst + qbytes, (const uint8_t *)sg.d + das, db, &full[slot]);
                if (pair) {
                    bulk_g2s(dst + qbytes + dbytes, sg.q2 + (size_t)ra * qrow, qb, &full[slot]);
                    bulk_g2s(dst + 2 * qbytes + dbytes, (const uint8_t *)sg.d2 + das, db, &full[slot]);
                }
            }
        }
        return;
    }
    gemv_prologue(p, xq, xd, xs, red);
    unsigned long long best = 0;
    const int logit_row0 = p.ls ? (*(volatile int *)&p.ls->step % LOGITS_RING) * p.vocab : 0;
    if (sg.type == T_Q4) {
        if (pair) {
            if (sg.d16) gemv_consume<T_Q4, true, true>(p, sg, r_begin, r_end, full, empty, ring, slot_bytes, xq, xd, xs, psum, best, logit_row0);
            else gemv_consume<T_Q4, false, true>(p, sg, r_begin, r_end, full, empty, ring, slot_bytes, xq, xd, xs, psum, best, logit_row0);
        } else {
            if (sg.d16) gemv_consume<T_Q4, true, false>(p, sg, r_begin, r_end, full, empty, ring, slot_bytes, xq, xd, xs, psum, best, logit_row0);
            else gemv_consume<T_Q4, false, false>(p, sg, r_begin, r_end, full, empty, ring, slot_bytes, xq, xd, xs, psum, best, logit_row0);
        }
    } else {
        if (pair) {
            if (sg.d16) gemv_consume<T_Q8, true, true>(p, sg, r_begin, r_end, full, empty, ring, slot_bytes, xq, xd, xs, psum, best, logit_row0);
            else gemv_consume<T_Q8, false, true>(p, sg, r_begin, r_end, full, empty, ring, slot_bytes, xq, xd, xs, psum, best, logit_row0);
        } else {
            if (sg.d16) gemv_consume<T_Q8, true, false>(p, sg, r_begin, r_end, full, empty, ring, slot_bytes, xq, xd, xs, psum, best, logit_row0);
            else gemv_consume<T_Q8, false, false>(p, sg, r_begin, r_end, full, empty, ring, slot_bytes, xq, xd, xs, psum, best, logit_row0);
        }
    }
    if (!p.ls) return;
    /* classifier: CTA argmax -> global max; the last CTA advances the loop */
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if (lane == 0) cta_best[warp] = best;
    consumer_sync();
    if (threadIdx.x == 0) {
        unsigned long long b = 0;
        for (int w = 0; w < GEMV_WARPS; w++) b = cta_best[w] > b ? cta_best[w] : b;
        atomicMax(&p.ls->best, b);
        __threadfence();
        *is_last = atomicAdd(&p.ls->done, 1u) == gridDim.x - 1;
    }
    consumer_sync();
    if (threadIdx.x == 0 && *is_last) {
        __threadfence();
        LoopState *ls = p.ls;
        const unsigned long long b = atomicAdd(&ls->best, 0ull);
        const int tok = (int)(0xffffffffu - (unsigned)(b & 0xffffffffull));
        const int step = ls->step;
        p.out_tokens[step] = tok;
        ls->step = step + 1;
        ls->pos = ls->pos + 1;
        ls->token = ls->feed_mode ? p.feed[step + 1] : tok;
        ls->best = 0ull;
        ls->done = 0u;
    }
}

/* Dynamic shared memory of gemv_kernel for a launch. */
__host__ inline int gemv_smem_bytes(const GemvParams &p) {
    int slot = 0;
    for (int i = 0; i < p.nseg; i++) {
        const int b = stage_slot_bytes(p.seg[i].type, p.seg[i].d16, p.cols, p.seg[i].epi == EPI_PAIR);
        slot = b > slot ? b : slot;
    }
    const int head = 16 * GEMV_NSTAGE + 256 * 4 + 8 * GEMV_WARPS + 16 + 32 * 4;
    const int act = p.cols + 8 * (p.cols / QK);
    return head + act + 128 + GEMV_NSTAGE * slot;
}

/* The loop advance when a step has no classifier (prefill without logits). */
__global__ void advance_kernel(LoopState *ls, const int *feed) {
    const int step = ls->step;
    ls->step = step + 1;
    ls->pos = ls->pos + 1;
    if (ls->feed_mode) ls->token = feed[step + 1];
}

/* x = dequant(tok_emb[token]) * embed_scale (model/transformer.c:226-230,
 * core/quant_ref.c:4-19). */
template <bool D16>
__global__ void embed_kernel(float *x, const uint8_t *q, const void *d, int type, int dim, int vocab, int max_seq,
                             float embed_scale, LoopState *ls) {
    const int tok = ls->token, pos = ls->pos;
    if (tok < 0 || tok >= vocab || pos < 0 || pos >= max_seq) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(&ls->err, 1u);
        return;
    }
    const int nb = dim / QK;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
        const int b = i / QK, j = i % QK;
        const float sc = load_scale<D16>(d, (size_t)tok * nb + b);
        int v;
        if (type == T_Q8) {
            v = ((const int8_t *)q)[(size_t)tok * dim + i];
        } else {
            const uint8_t byte = q[((size_t)tok * nb + b) * (QK / 2) + (j & 15)];
            v = (j < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
        }
        float o = __fmul_rn((float)v, sc);
        if (embed_scale != 1.0f) o = __fmul_rn(o, embed_scale);
        x[i] = o;
    }
}

/* Split-K flash decode for one KV head and one range of positions; F32 cache.
 * grid (n_kv_heads, nsplit), ATT_THREADS threads. */
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float fsm[];
    const int hd = p.hd, group = p.n_heads / p.n_kv_heads, h2 = hd / 2;
    const int g = blockIdx.x, y = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int pos = p.ls->pos;
    if (pos < 0 || pos >= p.max_seq) return;
    const int first = p.window && pos >= p.window ? pos + 1 - p.window : 0;
    const int n = pos + 1 - first;
    int C = (n + p.nsplit - 1) / p.nsplit;
    C = C < ATT_TILE ? ATT_TILE : (C + ATT_TILE - 1) / ATT_TILE * ATT_TILE;
    const int active = (n + C - 1) / C;
    if (y >= active) return;
    const int t_begin = first + y * C, t_end = min(t_begin + C, pos + 1);

    float *sq = fsm;                          /* [group][hd] */
    float *sk = sq + group * hd;              /* [ATT_TILE][hd + 1] */
    float *sv = sk + ATT_TILE * (hd + 1);     /* [ATT_TILE][hd] */
    float *sp = sv + ATT_TILE * hd;           /* [group][ATT_TILE] */
    float *sm = sp + group * ATT_TILE;        /* [group] running max */
    float *sl = sm + group;                   /* [group] running sum */
    float *sa = sl + group;                   /* [group] rescale of this tile */
    __shared__ int is_last;

    const float *cs = p.rcos + (size_t)pos * h2, *sn = p.rsin + (size_t)pos * h2;
    /* RoPE on adjacent pairs (k_scalar.c:79-94) */
    for (int idx = tid; idx < group * h2; idx += ATT_THREADS) {
        const int h = idx / h2, i = idx % h2;
        const float *qh = p.qkv + (size_t)(g * group + h) * hd;
        const float a = qh[2 * i], b = qh[2 * i + 1], c = cs[i], s = sn[i];
        sq[h * hd + 2 * i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        sq[h * hd + 2 * i + 1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
    if (t_end == pos + 1) {   /* this split holds the new position: store its K (roped) and V */
        const float *kn = p.qkv + p.q_dim + (size_t)g * hd, *vn = p.qkv + p.q_dim + p.kv_dim + (size_t)g * hd;
        float *kr = p.kc + (size_t)pos * p.kv_dim + (size_t)g * hd, *vr = p.vc + (size_t)pos * p.kv_dim + (size_t)g * hd;
        for (int i = tid; i < h2; i += ATT_THREADS) {
            const float a = kn[2 * i], b = kn[2 * i + 1], c = cs[i], s = sn[i];
            kr[2 * i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
            kr[2 * i + 1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
        }
        for (int i = tid; i < hd; i += ATT_THREADS) vr[i] = vn[i];
    }
    if (tid < group) {
        sm[tid] = -INFINITY;
        sl[tid] = 0.0f;
    }
    const int nout = group * hd;
    float acc[ATT_MAX_OUT];
#pragma unroll
    for (int k = 0; k < ATT_MAX_OUT; k++) acc[k] = 0.0f;
    __syncthreads();

    for (int t0 = t_begin; t0 < t_end; t0 += ATT_TILE) {
        const int nt = min(ATT_TILE, t_end - t0);
        const int h4 = hd / 4;
        for (int idx = tid; idx < nt * h4; idx += ATT_THREADS) {
            const int t = idx / h4, c4 = idx % h4;
            const size_t off = (size_t)(t0 + t) * p.kv_dim + (size_t)g * hd + 4 * c4;
            const float4 kv = __ldcg((const float4 *)(p.kc + off));
            const float4 vv = __ldcg((const float4 *)(p.vc + off));
            float *kd = sk + t * (hd + 1) + 4 * c4;
            kd[0] = kv.x; kd[1] = kv.y; kd[2] = kv.z; kd[3] = kv.w;
            *(float4 *)(sv + t * hd + 4 * c4) = vv;
        }
        __syncthreads();
        for (int idx = tid; idx < group * ATT_TILE; idx += ATT_THREADS) {
            const int h = idx / ATT_TILE, t = idx % ATT_TILE;
            float s = -INFINITY;
            if (t < nt) {
                const float *qh = sq + h * hd, *kt = sk + t * (hd + 1);
                float dot = 0.0f;
                for (int i = 0; i < hd; i++) dot = fmaf(qh[i], kt[i], dot);
                s = __fmul_rn(dot, p.scale);
                if (p.softcap > 0.0f) s = __fmul_rn(p.softcap, tanhf(__fdiv_rn(s, p.softcap)));
            }
            sp[h * ATT_TILE + t] = s;
        }
        __syncthreads();
        for (int h = warp; h < group; h += ATT_THREADS / 32) {
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
        __syncthreads();
#pragma unroll
        for (int k = 0; k < ATT_MAX_OUT; k++) {
            const int o = tid + k * ATT_THREADS;
            if (o < nout) {
                const int h = o / hd, i = o % hd;
                float a = acc[k] * sa[h];
                const float *ph = sp + h * ATT_TILE;
                for (int t = 0; t < nt; t++) a = fmaf(ph[t], sv[t * hd + i], a);
                acc[k] = a;
            }
        }
        __syncthreads();
    }
    const int stride = hd + 2;
#pragma unroll
    for (int k = 0; k < ATT_MAX_OUT; k++) {
        const int o = tid + k * ATT_THREADS;
        if (o < nout) {
            const int h = o / hd, i = o % hd;
            p.part[((size_t)(g * group + h) * p.nsplit + y) * stride + i] = acc[k];
        }
    }
    if (tid < group) {
        float *ph = p.part + ((size_t)(g * group + tid) * p.nsplit + y) * stride;
        ph[hd] = sm[tid];
        ph[hd + 1] = sl[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&p.counter[g], 1u) == (unsigned)active - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    /* combine: per head the split weights exp(m_s - M) / L into shared memory
     * (one lane per split), then every output sums its splits with the loads
     * of all splits in flight at once */
    float *wts = sp;   /* [group][ATT_TILE >= nsplit] (the score tile is free now) */
    for (int h = warp; h < group; h += ATT_THREADS / 32) {
        const float *ph = p.part + (size_t)(g * group + h) * p.nsplit * stride;
        const float m = lane < active ? __ldcg(ph + (size_t)lane * stride + hd) : -INFINITY;
        const float l = lane < active ? __ldcg(ph + (size_t)lane * stride + hd + 1) : 0.0f;
        const float M = warp_max(m);
        const float e = lane < active ? expf(m - M) : 0.0f;
        const float L = warp_sum(l * e);
        wts[h * ATT_TILE + lane] = e / L;
    }
    __syncthreads();
    for (int o = tid; o < nout; o += ATT_THREADS) {
        const int h = o / hd, i = o % hd;
        const float *base = p.part + (size_t)(g * group + h) * p.nsplit * stride + i;
        const float *w = wts + h * ATT_TILE;
        float num = 0.0f;
#pragma unroll 8
        for (int s2 = 0; s2 < active; s2++) num = fmaf(__ldcg(base + (size_t)s2 * stride), w[s2], num);
        p.ao[(size_t)(g * group + h) * hd + i] = num;
    }
    if (tid == 0) p.counter[g] = 0u;
}

/* Standalone activation quantization (kc_quantize_q8_dev / kc_rmsnorm_quantize_dev):
 * one CTA runs the GEMV prologue and writes the shared arrays out. */
__global__ void __launch_bounds__(GEMV_THREADS) quantize_kernel(const __grid_constant__ GemvParams p, int8_t *q,
                                                                float *d, float *xn) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int cols = p.cols, nb = cols / QK;
    int8_t *xq = (int8_t *)smem;
    float *xd = (float *)(smem + cols);
    int *xs = (int *)(smem + cols + 4 * nb);
    float *red = (float *)(smem + cols + 8 * nb);
    gemv_prologue(p, xq, xd, xs, red);
    for (int i = threadIdx.x; i < cols; i += blockDim.x) q[i] = xq[i];
    for (int b = threadIdx.x; b < nb; b += blockDim.x) d[b] = xd[b];
    if (xn && p.pro == PRO_RMSNORM_QUANT) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) {
            const float4 v = ((const float4 *)p.x)[i];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        ss = block_sum(ss, red);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), p.eps)));
        for (int i = threadIdx.x; i < cols; i += blockDim.x) xn[i] = __fmul_rn(__fmul_rn(p.x[i], inv), p.norm_w[i]);
    }
}

/* int32 block sums through dot_q4 / dot_q8 (the GEMV's integer path). */
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
