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
constexpr int NCW = 8;                   /* consumer warps of a streaming CTA: 288 threads with the
                                            producer, so that a thread gets up to 224 registers and the
                                            decode step runs without spills or call frames */
constexpr int NCT = NCW * 32;            /* consumer threads */
constexpr int STEP_THREADS = NCT + 32;   /* + the producer warp */
constexpr int STAGE_Q = 32 * 1024;       /* bytes of quants per ring stage (at least one row) */
constexpr int ATT_TILE = 64;             /* positions per attention tile (two per lane in the softmax) */
constexpr int ATT_MAX_OUT = 2048;        /* outputs per KV head group: group * head_dim */
constexpr int LOGITS_RING = 128;         /* logits rows kept on the device per call */
constexpr int MAX_NSPLIT = 32;           /* attention splits per KV head (one lane each in the combine) */

enum { T_Q8 = 1, T_Q4 = 2 };
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_PAIR = 2, EPI_LOGITS = 3 };

/* Device-resident token-loop state: one graph replays every step. */
struct LoopState {
    int token, pos, step, feed_mode;
    unsigned long long best;   /* argmax key: ordered logit << 32 | (~index) */
    unsigned done;             /* CTAs of the classifier that finished */
    unsigned err;              /* bit 0: token/pos out of range seen by a kernel */
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

__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

/* Q4_0 block: byte j = element j (low nibble) | element j+16 (high nibble),
 * nibble n = w + 8. Returns sum(n * x) exactly: the low nibbles go through
 * dp4a (unsigned x signed) as they are, the high nibbles masked in place (16 n)
 * and the sum divided by 16 once (an exact multiple of 16). The caller takes
 * off 8 * sum(x) (xs) in int32. xlo/xhi: activation elements 0..15 / 16..31. */
__device__ __forceinline__ int dot_q4(uint4 w, int4 xlo, int4 xhi) {
    const unsigned ml = 0x0F0F0F0Fu, mh = 0xF0F0F0F0u;
    int lo = 0, hi = 0;
    lo = dp4a_us(w.x & ml, xlo.x, lo);
    hi = dp4a_us(w.x & mh, xhi.x, hi);
    lo = dp4a_us(w.y & ml, xlo.y, lo);
    hi = dp4a_us(w.y & mh, xhi.y, hi);
    lo = dp4a_us(w.z & ml, xlo.z, lo);
    hi = dp4a_us(w.z & mh, xhi.z, hi);
    lo = dp4a_us(w.w & ml, xlo.w, lo);
    hi = dp4a_us(w.w & mh, xhi.w, hi);
    return lo + (hi >> 4);
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
/* quant4's rule with 4 lanes per block, 8 values per lane (lane groups of 4
 * consecutive lanes): the same block maximum, d, 127/amax and rounding, so
 * the bits are the same; half the shuffles and divisions per value. Returns
 * the 8 int8 values packed in a uint2. */
__device__ __forceinline__ uint2 quant8(const float v[8], float *d, int *sum) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    uint2 word = make_uint2(0u, 0u);
    int s = 0;
    if (amax < 1e-30f) {
        *d = 0.0f;
    } else {
        const float id = __fdiv_rn(127.0f, amax);
        *d = __fdiv_rn(amax, 127.0f);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float t = truncf(__fadd_rn(__fmul_rn(v[i], id), copysignf(0.5f, v[i])));
            t = fminf(fmaxf(t, -127.0f), 127.0f);
            const int qi = (int)t;
            s += qi;
            if (i < 4) word.x |= ((unsigned)qi & 0xffu) << (8 * i);
            else word.y |= ((unsigned)qi & 0xffu) << (8 * (i - 4));
        }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    *sum = s;
    return word;
}

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

/* The reference's single-scale row quantization (ops/ops.c:81-96) of the n
 * values x[0, n) by one warp (lane i takes elements i, i+32, ...): the quants
 * into out, and as floats into back when given; returns the scale. */
__device__ __forceinline__ float warp_quantize_row(const float *x, int n, int8_t *out, float *back, int lane) {
    float amax = 0.0f;
    for (int i = lane; i < n; i += 32) amax = fmaxf(amax, fabsf(x[i]));
    amax = warp_max(amax);
    const bool tiny = amax < 1e-30f;
    const float id = tiny ? 0.0f : __fdiv_rn(127.0f, amax);
    for (int i = lane; i < n; i += 32) {
        int qi = 0;
        if (!tiny) {
            const float t = truncf(__fadd_rn(__fmul_rn(x[i], id), copysignf(0.5f, x[i])));
            qi = (int)fminf(fmaxf(t, -127.0f), 127.0f);
        }
        out[i] = (int8_t)qi;
        if (back) back[i] = (float)qi;
    }
    return tiny ? 0.0f : __fdiv_rn(amax, 127.0f);
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
/* Polls of an mbarrier wait before it gives up (about a second under load). */
constexpr unsigned WAIT_POLLS = 1u << 22;

/* Waits for the phase with the given parity to complete; gives up (false)
 * after `limit` polls so that no wait can hang the GPU, or as soon as the
 * error word (when given) is non-zero. */
__device__ __forceinline__ bool mbar_wait(uint64_t *b, unsigned parity, const unsigned *err = nullptr,
                                          unsigned limit = WAIT_POLLS) {
    const uint32_t a = smem_u32(b);
    for (unsigned it = 0; it < limit; it++) {
        if (err && (it & 255) == 255 && *(volatile const unsigned *)err) return false;
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
/* 16-byte asynchronous global -> shared copy (no register staging); the
 * issuing thread waits for its own copies with cp_async_wait_all. */
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

/* Stage geometry of a matrix: R rows (a power of two, <= 64) per ring stage
 * with at most STAGE_Q bytes of quants (one row when a row alone is larger);
 * qbytes / dbytes: the quant and scale room of one matrix in a stage (the
 * scales with 16 bytes of alignment slack). pair: two matrices per stage. */
__host__ __device__ inline void stage_geom(int type, int d16, int cols, int pair, int &R, int &qbytes, int &dbytes) {
    const int qrow = type == T_Q4 ? cols / 2 : cols, drow = (cols / QK) * (d16 ? 2 : 4);
    const int unit = qrow * (pair ? 2 : 1);
    R = 1;
    while (R * 2 <= 64 && R * 2 * unit <= STAGE_Q) R *= 2;
    qbytes = R * qrow;
    dbytes = (R * drow + 16 + 15) & ~15;
}
__host__ __device__ inline int stage_slot_bytes(int type, int d16, int cols, int pair) {
    int R, qb, db;
    stage_geom(type, d16, cols, pair, R, qb, db);
    return (((qb + db) * (pair ? 2 : 1)) + 127) & ~127;
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

}  // namespace kc
