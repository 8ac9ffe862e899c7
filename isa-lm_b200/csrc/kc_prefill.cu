/* Batched prompt prefill on sm_100a: ml_prefill / prefill_step
 * (model/transformer.c:385-438) with the matrix products on the tensor cores.
 *
 * A chunk of up to `batch` prompt tokens goes through each layer as the
 * reference's prefill_step takes it: per token RMSNorm and the Q8_0 activation
 * rule, one matrix product per projection shared by every token of the chunk,
 * per token bias / RoPE / KV store, the batched attention (ops/ops.c:186-238)
 * and the residual adds.
 *
 * Projections: int8 GEMMs on tcgen05 (kind::i8, s8 x s8 -> s32 in TMEM). One
 * MMA covers one 32-wide K block, so every (row, token) block dot is an exact
 * int32, as the reference's dpbusd sums are; the epilogue warps read it from
 * TMEM and accumulate in float in block order, acc = fma(s, d_w * d_x, acc),
 * the per-row chain of the reference's packed kernels
 * (kernels/avx512vnni/k_avx512vnni.c:128-186). Weights are repacked once per
 * model into the MMA's shared-memory operand layout (Q4 nibbles widened to
 * int8, scales to float), and each quantized activation chunk is written in
 * the same layout, so a pipeline stage is one bulk copy per operand.
 *
 * CTA of the GEMM: warp 0 issues the bulk copies, warp 1 owns TMEM and issues
 * the MMAs, warps 2..9 are the epilogue (two per TMEM lane quarter, each 16
 * token columns of a 128-row x 32-token tile).
 */
#include <cmath>
#include <cstring>
#include <algorithm>
#include <string>
#include <vector>

#include "kc_internal.h"
#include "kc_kernels.cuh"
#include "kc_prefill.h"

namespace kc {

constexpr int PF_M = 128;                              /* weight rows per tile: the TMEM lanes */
constexpr int PF_N = 32;                               /* tokens per tile: TMEM columns per buffer */
constexpr int PF_KB = 4;                               /* K blocks per pipeline stage */
constexpr int PF_NST = 4;                              /* pipeline stages */
constexpr int PF_NBUF = 4;                             /* TMEM buffers, each two K blocks x PF_N columns */
constexpr int PF_EPI_WARPS = 8;                        /* two per TMEM lane quarter */
constexpr int PF_THREADS = 32 * (2 + PF_EPI_WARPS);
constexpr int PF_COLS = PF_N * 4 / PF_EPI_WARPS;       /* token columns per epilogue warp */
constexpr int PF_A_BLK = PF_M * QK;                    /* bytes of one K block of a weight tile */
constexpr int PF_B_BLK = PF_N * QK;                    /* bytes of one K block of a token tile */
constexpr int PF_DW_BLK = PF_M * 4;                    /* weight scales of one K block (float) */
constexpr int PF_DX_BLK = PF_N * 4;                    /* token scales of one K block (float) */
constexpr int PF_STAGE = PF_KB * (PF_A_BLK + PF_B_BLK + PF_DW_BLK + PF_DX_BLK);
constexpr int PF_TMEM_COLS = PF_NBUF * 2 * PF_N;
constexpr int PF_SMEM = 1024 + PF_NST * PF_STAGE + 256;
static_assert(PF_TMEM_COLS >= 32 && (PF_TMEM_COLS & (PF_TMEM_COLS - 1)) == 0, "TMEM columns: a power of two");
static_assert(PF_COLS == 16, "the epilogue loads 16 TMEM columns at a time");
static_assert(PF_STAGE % 256 == 0, "stage alignment");
static_assert(PF_KB % 2 == 0, "a stage holds whole K-block pairs");
static_assert((2 * PF_NST + 2 * PF_NBUF) * 8 + 4 <= 256, "barrier room");

/* Byte (r, k) of one K block (rows x 32 bytes) in the MMA's K-major layout
 * without swizzle: core matrices of 8 rows x 16 bytes (128 contiguous bytes),
 * the two 16-byte K halves of a row group 128 bytes apart, row groups 256
 * bytes apart. */
__host__ __device__ inline int tile_off(int r, int k) { return (r >> 3) * 256 + (k >> 4) * 128 + (r & 7) * 16 + (k & 15); }

/* Shared-memory matrix descriptor of a K block in that layout (tcgen05
 * descriptor: start >> 4, leading-dimension offset 128 >> 4 (between the K
 * halves), stride offset 256 >> 4 (between row groups), version 1, no swizzle). */
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
           (1ull << 46);
}
/* Instruction descriptor: s32 accumulators, A and B signed 8-bit, both K-major,
 * N = PF_N, M = PF_M. */
constexpr uint32_t PF_IDESC =
    (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PF_N >> 3) << 17) | ((uint32_t)(PF_M >> 4) << 24);

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_alloc(uint32_t *slot, int ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, int ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_st16(uint32_t taddr, uint32_t v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(
            taddr),
        "r"(v)
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

/* Pairs of floats in one 64-bit register for the paired FP32 instructions
 * (add/sub/mul/fma .f32x2): each lane of the pair rounds as the scalar
 * instruction does. */
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2sub(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
/* An int32 with |s| < 2^22 as a float, exactly, without the conversion unit:
 * the bits 0x4B400000 + s are the float 1.5 * 2^23 + s (the mantissa of
 * 1.5 * 2^23 has ulp 1 and room for s on either side), and subtracting
 * 1.5 * 2^23 leaves s. A 32-element int8 block dot is at most 32 * 127 * 127.
 * The GEMM's TMEM accumulators start at these bits, so the MMA itself adds s. */
constexpr int PF_MAGIC_BITS = 0x4B400000;
constexpr float PF_MAGIC = 12582912.0f;

/* Error bit of the prefill kernels: a pipeline wait gave up. */
constexpr unsigned PF_ERR_WAIT = 4u;

enum { PF_STORE = 0, PF_RESID = 1 };

struct PfGemm {
    const int8_t *wq;    /* [mt][nbk] K blocks of PF_A_BLK bytes */
    const float *wd;     /* [mt][nbk][PF_M] */
    const float *bias;   /* [rows] or null */
    const int8_t *xq;    /* [nt][nbk] K blocks of PF_B_BLK bytes */
    const float *xd;     /* [nt][nbk][PF_N] */
    float *out;          /* out[t * ldo + row] */
    int ldo, rows, T, nbk, mode;
    float softcap;
    unsigned *err;
};

/* Y[t][row] = sum_b s(row, t, b) * (d_w[row][b] * d_x[t][b]) over one
 * 128-row x 32-token tile (blockIdx.y, blockIdx.x): stored, or added to out
 * (residual), with the row's bias and the logit soft-cap when given.
 * A pipeline stage holds PF_KB K blocks: weight quants, token quants, weight
 * scales, token scales, each one bulk copy. The stage is released when its
 * MMAs have completed (tcgen05.commit) and every epilogue warp has read its
 * scales; a TMEM buffer when every epilogue warp has loaded it. */
__global__ void __launch_bounds__(PF_THREADS, 2) pf_gemm_kernel(const __grid_constant__ PfGemm g) {
    extern __shared__ unsigned char pf_smem_raw[];
    unsigned char *sm = (unsigned char *)(((uintptr_t)pf_smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(sm + PF_NST * PF_STAGE), *empty = full + PF_NST;
    uint64_t *tfull = empty + PF_NST, *tempty = tfull + PF_NBUF;
    uint32_t *tslot = (uint32_t *)(tempty + PF_NBUF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x, m = blockIdx.y, nbk = g.nbk;
    constexpr int OFF_B = PF_KB * PF_A_BLK, OFF_DW = OFF_B + PF_KB * PF_B_BLK, OFF_DX = OFF_DW + PF_KB * PF_DW_BLK;
    if (threadIdx.x == 0) {
        for (int i = 0; i < PF_NST; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1 + PF_EPI_WARPS);
        }
        for (int i = 0; i < PF_NBUF; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], PF_EPI_WARPS);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tc_alloc(tslot, PF_TMEM_COLS);
        tc_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (warp == 0) {
        if (lane == 0) {
            const int nst = (nbk + PF_KB - 1) / PF_KB;
            for (int st = 0; st < nst; st++) {
                const int s = st % PF_NST;
                if (!mbar_wait(&empty[s], ((st / PF_NST) & 1) ^ 1, g.err)) {
                    atomicOr(g.err, PF_ERR_WAIT);
                    break;
                }
                const int kbs = min(PF_KB, nbk - st * PF_KB);
                const size_t wb = (size_t)m * nbk + (size_t)st * PF_KB, xb = (size_t)n * nbk + (size_t)st * PF_KB;
                unsigned char *stage = sm + s * PF_STAGE;
                mbar_expect_tx(&full[s], (unsigned)(kbs * (PF_A_BLK + PF_B_BLK + PF_DW_BLK + PF_DX_BLK)));
                bulk_g2s(stage, g.wq + wb * PF_A_BLK, kbs * PF_A_BLK, &full[s]);
                bulk_g2s(stage + OFF_B, g.xq + xb * PF_B_BLK, kbs * PF_B_BLK, &full[s]);
                bulk_g2s(stage + OFF_DW, g.wd + wb * PF_M, kbs * PF_DW_BLK, &full[s]);
                bulk_g2s(stage + OFF_DX, g.xd + xb * PF_N, kbs * PF_DX_BLK, &full[s]);
            }
        }
    } else if (warp == 1) {
        /* MMA issue: K blocks in pairs, one TMEM buffer (2 x PF_N columns) and
         * one commit per pair */
        if (lane == 0) {
            for (int ks = 0; 2 * ks < nbk; ks++) {
                const int kb = 2 * ks, st = kb / PF_KB, j = kb - st * PF_KB, s = st % PF_NST, buf = ks % PF_NBUF;
                if (j == 0 && !mbar_wait(&full[s], (st / PF_NST) & 1, g.err)) {
                    atomicOr(g.err, PF_ERR_WAIT);
                    break;
                }
                /* the epilogue fills each buffer with the bias before its every use */
                if (!mbar_wait(&tempty[buf], (ks / PF_NBUF) & 1, g.err)) {
                    atomicOr(g.err, PF_ERR_WAIT);
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(sm + s * PF_STAGE) + j * PF_A_BLK;
                const uint32_t b = smem_u32(sm + s * PF_STAGE + OFF_B) + j * PF_B_BLK;
                const uint32_t d = tmem + (uint32_t)(buf * 2 * PF_N);
                tc_mma_i8(d, umma_desc(a), umma_desc(b), PF_IDESC, 1u);
                if (kb + 1 < nbk) tc_mma_i8(d + PF_N, umma_desc(a + PF_A_BLK), umma_desc(b + PF_B_BLK), PF_IDESC, 1u);
                tc_commit(&tfull[buf]);
                if (j + 2 == PF_KB || kb + 2 >= nbk) tc_commit(&empty[s]);
            }
        }
    } else {
        /* epilogue: TMEM lane quarter q (the warp's rank in its warpgroup),
         * token columns c0 .. c0+15 of the tile; K blocks in pairs, the TMEM
         * loads of pair ks + 1 in flight while pair ks is accumulated */
        const int e = warp - 2, q = warp & 3, c0 = (e >> 2) * PF_COLS;
        const int row = m * PF_M + q * 32 + lane;
        const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
        uint64_t acc[PF_COLS / 2];   /* column pairs */
#pragma unroll
        for (int c = 0; c < PF_COLS / 2; c++) acc[c] = 0ull;
        const uint64_t magic2 = f2pack(PF_MAGIC, PF_MAGIC);
        const int nks = (nbk + 1) / 2;
        bool ok = true;
        /* every TMEM buffer starts as the int32 bits of 1.5 * 2^23: the MMAs add
         * their block dots to it, so each word read back is the float 1.5 * 2^23 + s */
        for (int b = 0; b < PF_NBUF; b++) {
            tc_st16(tq + (uint32_t)(b * 2 * PF_N), (uint32_t)PF_MAGIC_BITS);
            tc_st16(tq + (uint32_t)(b * 2 * PF_N + PF_N), (uint32_t)PF_MAGIC_BITS);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int b = 0; b < PF_NBUF; b++) mbar_arrive(&tempty[b]);
        /* acc = fma((float)s, d_w * d_x, acc) for K block j of the stage, two columns per instruction */
        auto accumulate = [&](const uint32_t (&v)[PF_COLS], const unsigned char *stage, int j) {
            const float dw = ((const float *)(stage + OFF_DW))[j * PF_M + q * 32 + lane];
            const uint64_t dw2 = f2pack(dw, dw);
            const float4 *dx4 = (const float4 *)(stage + OFF_DX + j * PF_DX_BLK) + c0 / 4;
#pragma unroll
            for (int i = 0; i < PF_COLS / 4; i++) {
                const float4 x = dx4[i];
                const uint64_t m01 = f2mul(dw2, f2pack(x.x, x.y)), m23 = f2mul(dw2, f2pack(x.z, x.w));
                const uint64_t s01 = f2sub(f2pack(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])), magic2);
                const uint64_t s23 = f2sub(f2pack(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])), magic2);
                acc[2 * i] = f2fma(s01, m01, acc[2 * i]);
                acc[2 * i + 1] = f2fma(s23, m23, acc[2 * i + 1]);
            }
        };
        for (int ks = 0; ks < nks; ks++) {
            const int kb = 2 * ks, st = kb / PF_KB, j = kb - st * PF_KB, s = st % PF_NST, buf = ks % PF_NBUF;
            if (j == 0 && !__all_sync(0xffffffffu, mbar_wait(&full[s], (st / PF_NST) & 1, g.err))) {
                ok = false;
                break;
            }
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (ks / PF_NBUF) & 1, g.err))) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t va[PF_COLS], vb[PF_COLS];
            tc_ld16(tq + (uint32_t)(buf * 2 * PF_N), va);
            tc_ld16(tq + (uint32_t)(buf * 2 * PF_N + PF_N), vb);
            tc_wait_ld();
            tc_st16(tq + (uint32_t)(buf * 2 * PF_N), (uint32_t)PF_MAGIC_BITS);
            tc_st16(tq + (uint32_t)(buf * 2 * PF_N + PF_N), (uint32_t)PF_MAGIC_BITS);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            const unsigned char *stage = sm + s * PF_STAGE;
            accumulate(va, stage, j);
            if (kb + 1 < nbk) accumulate(vb, stage, j + 1);
            if (j + 2 == PF_KB || kb + 2 >= nbk) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
        }
        if (!ok) {
            tc_wait_ld();
            if (lane == 0) atomicOr(g.err, PF_ERR_WAIT);
        } else if (row < g.rows) {
            const float bias = g.bias ? g.bias[row] : 0.0f;
            float res[PF_COLS];
#pragma unroll
            for (int c = 0; c < PF_COLS / 2; c++) f2unpack(acc[c], res[2 * c], res[2 * c + 1]);
#pragma unroll
            for (int c = 0; c < PF_COLS; c++) {
                const int t = n * PF_N + c0 + c;
                if (t < g.T) {
                    float y = res[c];
                    if (g.bias) y = __fadd_rn(y, bias);
                    if (g.softcap > 0.0f) y = __fmul_rn(g.softcap, tanhf(__fdiv_rn(y, g.softcap)));
                    float *o = g.out + (size_t)t * g.ldo + row;
                    *o = g.mode == PF_RESID ? __fadd_rn(*o, y) : y;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tc_dealloc(tmem, PF_TMEM_COLS);
}

/* ------------------------------------------------------------ activations */

enum { PQ_NORM = 0, PQ_PLAIN = 1, PQ_GATED = 2 };

struct PfQuant {
    const float *x;      /* x[t * ldx + i] */
    int ldx;
    const float *w;      /* norm weights (PQ_NORM) */
    float eps;
    int mode, act, cols, T, nbk;
    int8_t *xq;          /* [nt][nbk] K blocks of PF_B_BLK bytes */
    float *xd;           /* [nt][nbk][PF_N] */
};

/* One token per CTA (grid: the token tiles' rows, padding tokens quantize to
 * zero): v = RMSNorm(x) * w (k_scalar.c:59-64, o = (x * inv) * w), x itself,
 * or act(g) * u from a [g | u] row (model/transformer.c:233-236); then the
 * Q8_0 rule per 32-block (k_scalar.c:39-57) into the GEMM's token-tile layout. */
__global__ void __launch_bounds__(256) pf_quant_kernel(const PfQuant a) {
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nt = t / PF_N, tr = t - nt * PF_N;
    __shared__ float red[8];
    const bool live = t < a.T;
    const float *xr = a.x + (size_t)(live ? t : 0) * a.ldx;
    float inv = 1.0f;
    if (a.mode == PQ_NORM) {
        float ss = 0.0f;
        if (live)
            for (int i = tid; i < a.cols; i += 256) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        ss = red[0];
        for (int w = 1; w < 8; w++) ss = __fadd_rn(ss, red[w]);
        inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)a.cols), a.eps)));
    }
    for (int b0 = warp * 4; b0 < a.nbk; b0 += 32) {
        const int b = b0 + (lane >> 3), j0 = (lane & 7) * 4;
        float v[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
        if (live && b < a.nbk) {
            const int i = b * QK + j0;
            if (a.mode == PQ_GATED) {
#pragma unroll
                for (int k = 0; k < 4; k++) v[k] = act_mul(a.act, xr[i + k], xr[a.cols + i + k]);
            } else {
                const float4 x4 = *(const float4 *)(xr + i);
                v[0] = x4.x; v[1] = x4.y; v[2] = x4.z; v[3] = x4.w;
                if (a.mode == PQ_NORM) {
                    const float4 w4 = *(const float4 *)(a.w + i);
                    v[0] = __fmul_rn(__fmul_rn(v[0], inv), w4.x);
                    v[1] = __fmul_rn(__fmul_rn(v[1], inv), w4.y);
                    v[2] = __fmul_rn(__fmul_rn(v[2], inv), w4.z);
                    v[3] = __fmul_rn(__fmul_rn(v[3], inv), w4.w);
                }
            }
        }
        float d;
        int sum;
        const unsigned word = quant4(v, &d, &sum);
        if (b < a.nbk) {
            int8_t *blk = a.xq + ((size_t)nt * a.nbk + b) * PF_B_BLK;
            *(unsigned *)(blk + tile_off(tr, j0)) = word;
            if ((lane & 7) == 0) a.xd[((size_t)nt * a.nbk + b) * PF_N + tr] = d;
        }
    }
}

struct PfEmbed {
    const uint8_t *q;
    const void *d;
    int type, d16;
    float scale;
    const int *tok;
    int cols;
    float *x;
};

/* x[t] = dequant(tok_emb[tok[t]]) * embed_scale (model/transformer.c:226-230,
 * core/quant_ref.c:4-19). */
__global__ void __launch_bounds__(256) pf_embed_kernel(const PfEmbed a) {
    const int t = blockIdx.x, tok = a.tok[t], nb = a.cols / QK;
    for (int i = threadIdx.x; i < a.cols; i += 256) {
        const int b = i / QK, j = i % QK;
        const float sc = a.d16 ? __half2float(((const __half *)a.d)[(size_t)tok * nb + b])
                               : ((const float *)a.d)[(size_t)tok * nb + b];
        int v;
        if (a.type == T_Q8) {
            v = ((const int8_t *)a.q)[(size_t)tok * a.cols + i];
        } else {
            const uint8_t byte = a.q[((size_t)tok * nb + b) * (QK / 2) + (j & 15)];
            v = (j < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
        }
        float o = __fmul_rn((float)v, sc);
        if (a.scale != 1.0f) o = __fmul_rn(o, a.scale);
        a.x[(size_t)t * a.cols + i] = o;
    }
}

/* Post-norm models: x += RMSNorm(y) * w for every token (model/transformer.c:238-243), one token per CTA. */
__global__ void __launch_bounds__(256) pf_post_kernel(float *x, const float *y, const float *w, int cols, float eps) {
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ float red[8];
    const float *yr = y + (size_t)t * cols;
    float *xr = x + (size_t)t * cols;
    float ss = 0.0f;
    for (int i = tid; i < cols; i += 256) ss = __fadd_rn(ss, __fmul_rn(yr[i], yr[i]));
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    ss = red[0];
    for (int k = 1; k < 8; k++) ss = __fadd_rn(ss, red[k]);
    const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)cols), eps)));
    for (int i = tid; i < cols; i += 256) xr[i] = __fadd_rn(xr[i], __fmul_rn(__fmul_rn(yr[i], inv), w[i]));
}

struct PfRope {
    float *qkv;                  /* [T][q_dim + 2 kv_dim], q | k | v */
    int ldq;
    const float *rcos, *rsin;    /* [max_seq][hd / 2] */
    void *kc, *vc;               /* this layer's cache rows [max_seq][kv_dim] */
    float *kd, *vd;              /* Q8 cache: row scales [max_seq][n_kv] */
    int8_t *qq;                  /* Q8 cache: quantized query heads [T][q_dim] */
    float *qd;                   /* their scales [T][n_heads] */
    int pos0, hd, n_heads, n_kv, q_dim, kv_dim, kv_type;
    const float *q_norm, *k_norm;   /* per-head RMSNorm weights [hd] (qk_norm), or null */
    float eps;
};

constexpr int PR_MAX_HEADS = 512;   /* query + KV heads a rope CTA normalizes */

/* One token per CTA: with qk_norm the per-head RMSNorm of every q and k head
 * (model/transformer.c:244-248, before RoPE); RoPE on adjacent pairs of every q and k head
 * (k_scalar.c:79-94) at position pos0 + t, then the K and V rows into the
 * cache in its type (model/transformer.c:188-205: f16 rounding, or the
 * single-scale row quantization per KV head, ops/ops.c:81-96) and, for a Q8
 * cache, the query heads quantized the same way (ops/ops.c:229-233). */
__global__ void __launch_bounds__(256) pf_rope_kernel(const PfRope a) {
    const int t = blockIdx.x, p = a.pos0 + t, h2 = a.hd / 2;
    float *q = a.qkv + (size_t)t * a.ldq, *k = q + a.q_dim, *v = k + a.kv_dim;
    const float *cs = a.rcos + (size_t)p * h2, *sn = a.rsin + (size_t)p * h2;
    const int nq = a.n_heads * h2, nk = a.n_kv * h2;
    __shared__ float hinv[PR_MAX_HEADS];
    if (a.q_norm) {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int h = warp; h < a.n_heads + a.n_kv; h += 8) {
            const float *x = h < a.n_heads ? q + h * a.hd : k + (h - a.n_heads) * a.hd;
            float t = 0.0f;
            for (int i = lane; i < a.hd; i += 32) t = __fadd_rn(t, __fmul_rn(x[i], x[i]));
            t = warp_sum(t);
            if (lane == 0) hinv[h] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(t, (float)a.hd), a.eps)));
        }
        __syncthreads();
    }
    for (int idx = threadIdx.x; idx < nq + nk; idx += 256) {
        const bool isq = idx < nq;
        const int r = isq ? idx : idx - nq, h = r / h2, i = r - h * h2;
        float *e = (isq ? q : k) + h * a.hd + 2 * i;
        float xa = e[0], xb = e[1];
        const float c = cs[i], s = sn[i];
        if (a.q_norm) {
            const float inv = hinv[isq ? h : a.n_heads + h], *w = isq ? a.q_norm : a.k_norm;
            xa = __fmul_rn(__fmul_rn(xa, inv), w[2 * i]);
            xb = __fmul_rn(__fmul_rn(xb, inv), w[2 * i + 1]);
        }
        e[0] = __fsub_rn(__fmul_rn(xa, c), __fmul_rn(xb, s));
        e[1] = __fadd_rn(__fmul_rn(xa, s), __fmul_rn(xb, c));
    }
    __syncthreads();
    const size_t row = (size_t)p * a.kv_dim;
    if (a.kv_type == KC_F32) {
        for (int i = threadIdx.x; i < a.kv_dim; i += 256) {
            ((float *)a.kc)[row + i] = k[i];
            ((float *)a.vc)[row + i] = v[i];
        }
    } else if (a.kv_type == KC_F16) {
        for (int i = threadIdx.x; i < a.kv_dim; i += 256) {
            ((__half *)a.kc)[row + i] = __float2half_rn(k[i]);
            ((__half *)a.vc)[row + i] = __float2half_rn(v[i]);
        }
    } else {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int j = warp; j < 2 * a.n_kv + a.n_heads; j += 8) {
            if (j < 2 * a.n_kv) {
                const bool isv = j >= a.n_kv;
                const int g = isv ? j - a.n_kv : j;
                int8_t *dst = (int8_t *)(isv ? a.vc : a.kc) + row + (size_t)g * a.hd;
                const float d = warp_quantize_row((isv ? v : k) + g * a.hd, a.hd, dst, nullptr, lane);
                if (lane == 0) (isv ? a.vd : a.kd)[(size_t)p * a.n_kv + g] = d;
            } else {
                const int h = j - 2 * a.n_kv;
                const float d =
                    warp_quantize_row(q + h * a.hd, a.hd, a.qq + (size_t)t * a.q_dim + h * a.hd, nullptr, lane);
                if (lane == 0) a.qd[(size_t)t * a.n_heads + h] = d;
            }
        }
    }
}

/* ------------------------------------------------------------ attention */

constexpr int PA_THREADS = 256;
constexpr int PA_ROWS = 32;                          /* query rows (tokens x heads of one KV group) per CTA */
constexpr int PA_MAXG = 16;                          /* query heads per KV head */

struct PfAttn {
    const float *qkv;            /* rotated query heads at qkv[t * ldq + h * hd] */
    int ldq;
    const int8_t *qq;            /* Q8 cache: quantized query heads */
    const float *qd;
    const void *kc, *vc;
    const float *kd, *vd;
    float *out;                  /* [T][q_dim] */
    int T, pos0, hd, n_heads, n_kv, q_dim, kv_dim, window, tq;   /* tq: tokens per CTA */
    float scale, softcap;
};

/* Shared memory of pf_attn_kernel: the CTA's query rows, K and V tiles of pt
 * positions (double-buffered, rows at a pitch of the row's bytes + 16 so that
 * 16-byte reads of different rows hit different banks), the tile's scores /
 * probabilities per row, the rows' running max, sum and rescale, and the Q8
 * row scales of the tiles. */
__host__ __device__ inline int pa_pitch(int hd, int es) { return hd * es + 16; }
__host__ __device__ inline size_t pa_smem_bytes(int hd, int es, int pt) {
    return sizeof(float) * (size_t)PA_ROWS * hd + 4 * (size_t)pt * pa_pitch(hd, es) +
           sizeof(float) * ((size_t)PA_ROWS * pt + 3 * PA_ROWS + 4 * (size_t)pt);
}

__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

/* Attention of tq consecutive tokens (positions pos0 + t) for the query heads
 * of KV head g: ops/ops.c:124-180 (attend) for each of their rows, the cache
 * read once per CTA for all of them in tiles of PT positions staged through
 * shared memory (cp.async, one tile ahead). Per row and tile: scores q.k *
 * scale summed over the head dimension in order (Q8 cache: int32 dot of the
 * quantized query and row, (float)s * (qd * scale) * kd), the optional
 * soft-cap, the causal (and sliding-window) mask of the row's position; then
 * the running softmax (max, exp(s - max), sum) rescales the row's output,
 * out += sum_t p_t * V_t in position order (Q8: (p_t * vd_t) * v), and the
 * output is divided by the row's sum at the end. */
template <int KV, int HD>
__global__ void __launch_bounds__(PA_THREADS) pf_attn_kernel(const PfAttn a) {
    extern __shared__ __align__(16) unsigned char pa_raw[];
    constexpr int ES = KV == KC_F32 ? 4 : (KV == KC_F16 ? 2 : 1);
    constexpr int PT = HD <= 64 ? 64 : 32, hd = HD;
    const int g = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int group = a.n_heads / a.n_kv;
    const int t0 = blockIdx.x * a.tq, ntok = min(a.tq, a.T - t0), R = ntok * group;
    const int rowb = hd * ES, pitch = rowb + 16, upr = rowb / 16;
    float *sq = (float *)pa_raw;                                   /* [PA_ROWS][hd] (Q8: int8 rows) */
    unsigned char *tiles = (unsigned char *)(sq + PA_ROWS * hd);   /* K0 V0 K1 V1, PT rows each */
    float *sp = (float *)(tiles + 4 * PT * pitch);                 /* [PA_ROWS][PT] */
    float *smx = sp + PA_ROWS * PT, *ssum = smx + PA_ROWS, *salpha = ssum + PA_ROWS;
    float *srd = salpha + PA_ROWS;                                 /* [2 buffers][K, V][PT] Q8 row scales */
    __shared__ float cq[PA_ROWS];
    /* row r: token t0 + r / group, query head g * group + r % group */
    if constexpr (KV == KC_Q8_0) {
        for (int i = tid; i < R * hd / 4; i += PA_THREADS) {
            const int r = i / (hd / 4), w = i % (hd / 4);
            const int8_t *qq = a.qq + (size_t)(t0 + r / group) * a.q_dim + (size_t)(g * group + r % group) * hd;
            ((int *)sq)[i] = ((const int *)qq)[w];
        }
        if (tid < R)
            cq[tid] = __fmul_rn(a.qd[(size_t)(t0 + tid / group) * a.n_heads + g * group + tid % group], a.scale);
    } else {
        for (int i = tid; i < R * hd; i += PA_THREADS) {
            const int r = i / hd, d = i % hd;
            sq[i] = a.qkv[(size_t)(t0 + r / group) * a.ldq + (size_t)(g * group + r % group) * hd + d];
        }
    }
    if (tid < PA_ROWS) {
        smx[tid] = -INFINITY;
        ssum[tid] = 0.0f;
    }
    const int p_first = a.pos0 + t0, p_last = p_first + ntok - 1;
    const int lo = a.window && p_first >= a.window ? p_first + 1 - a.window : 0;   /* the rows' first position */
    const int ntiles = (p_last + 1 - lo + PT - 1) / PT;
    const size_t ld = (size_t)a.kv_dim * ES;
    const uint8_t *kbase = (const uint8_t *)a.kc + (size_t)g * rowb, *vbase = (const uint8_t *)a.vc + (size_t)g * rowb;
    auto load_tile = [&](int k) {
        const int tp = lo + k * PT, nt = min(PT, p_last + 1 - tp);
        unsigned char *kd = tiles + (size_t)(2 * (k & 1)) * PT * pitch, *vd = kd + (size_t)PT * pitch;
        for (int u = tid; u < nt * upr; u += PA_THREADS) {
            const int r = u / upr, c = u - r * upr;
            cp_async16(kd + r * pitch + 16 * c, kbase + (size_t)(tp + r) * ld + 16 * c);
            cp_async16(vd + r * pitch + 16 * c, vbase + (size_t)(tp + r) * ld + 16 * c);
        }
        cp_async_commit();
        if (KV == KC_Q8_0 && tid < nt) {
            srd[(k & 1) * 2 * PT + tid] = a.kd[(size_t)(tp + tid) * a.n_kv + g];
            srd[(k & 1) * 2 * PT + PT + tid] = a.vd[(size_t)(tp + tid) * a.n_kv + g];
        }
    };
    /* outputs of this thread: dimension tid % hd of rows tid / hd + k * (PA_THREADS / hd) */
    constexpr int rp = PA_THREADS / HD, NO = PA_ROWS / rp;
    const int od = tid % hd, or0 = tid / hd;
    float acc[NO];
#pragma unroll
    for (int k = 0; k < NO; k++) acc[k] = 0.0f;
    load_tile(0);
    for (int k = 0; k < ntiles; k++) {
        if (k + 1 < ntiles) {
            load_tile(k + 1);
            cp_async_wait_one();
        } else {
            cp_async_wait_all();
        }
        __syncthreads();
        const int tp = lo + k * PT, nt = min(PT, p_last + 1 - tp);
        const unsigned char *K = tiles + (size_t)(2 * (k & 1)) * PT * pitch, *V = K + (size_t)PT * pitch;
        const float *rkd = srd + (k & 1) * 2 * PT, *rvd = rkd + PT;
        /* scores of every (row, position) of the tile, masked by the row's position: thread ->
         * position tid % PT of rows tid / PT + j * (PA_THREADS / PT), their chains interleaved */
        {
            constexpr int RPS = PA_THREADS / PT, NS = PA_ROWS / RPS;
            const int p = tid % PT, r0 = tid / PT, t = tp + p;
            const unsigned char *row = K + (size_t)p * pitch;
            float sc[NS];
            bool live[NS];
#pragma unroll
            for (int j = 0; j < NS; j++) {
                const int r = r0 + j * RPS, pos = p_first + r / group;
                const int first = a.window && pos >= a.window ? pos + 1 - a.window : 0;
                live[j] = r < R && p < nt && t <= pos && t >= first;
            }
            if constexpr (KV == KC_Q8_0) {
                int isum[NS];
#pragma unroll
                for (int j = 0; j < NS; j++) isum[j] = 0;
                for (int w = 0; w < hd / 4; w++) {
                    const int kw = p < nt ? ((const int *)row)[w] : 0;
#pragma unroll
                    for (int j = 0; j < NS; j++)
                        if (r0 + j * RPS < R) isum[j] = __dp4a(((const int *)sq)[(r0 + j * RPS) * hd / 4 + w], kw, isum[j]);
                }
#pragma unroll
                for (int j = 0; j < NS; j++)
                    sc[j] = live[j] ? __fmul_rn(__fmul_rn((float)isum[j], cq[r0 + j * RPS]), rkd[p]) : 0.0f;
            } else {
                /* q.k over the head dimension in order, rows in pairs (fma.f32x2) */
                uint64_t sc2[NS / 2];
#pragma unroll
                for (int j = 0; j < NS / 2; j++) sc2[j] = 0ull;
                for (int d0 = 0; d0 < hd; d0 += 4) {
                    float k4[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
                    if (p < nt) {
                        if constexpr (KV == KC_F32) {
                            const float4 v = *(const float4 *)(row + 4 * d0);
                            k4[0] = v.x; k4[1] = v.y; k4[2] = v.z; k4[3] = v.w;
                        } else {
                            const uint2 u = *(const uint2 *)(row + 2 * d0);
                            const float2 l0 = __half22float2(*(const __half2 *)&u.x), h0 = __half22float2(*(const __half2 *)&u.y);
                            k4[0] = l0.x; k4[1] = l0.y; k4[2] = h0.x; k4[3] = h0.y;
                        }
                    }
                    const uint64_t kk0 = f2pack(k4[0], k4[0]), kk1 = f2pack(k4[1], k4[1]);
                    const uint64_t kk2 = f2pack(k4[2], k4[2]), kk3 = f2pack(k4[3], k4[3]);
#pragma unroll
                    for (int j = 0; j < NS / 2; j++) {
                        const float4 qa = *(const float4 *)(sq + (r0 + 2 * j * RPS) * hd + d0);
                        const float4 qb = *(const float4 *)(sq + (r0 + (2 * j + 1) * RPS) * hd + d0);
                        sc2[j] = f2fma(f2pack(qa.x, qb.x), kk0, sc2[j]);
                        sc2[j] = f2fma(f2pack(qa.y, qb.y), kk1, sc2[j]);
                        sc2[j] = f2fma(f2pack(qa.z, qb.z), kk2, sc2[j]);
                        sc2[j] = f2fma(f2pack(qa.w, qb.w), kk3, sc2[j]);
                    }
                }
#pragma unroll
                for (int j = 0; j < NS / 2; j++) f2unpack(sc2[j], sc[2 * j], sc[2 * j + 1]);
#pragma unroll
                for (int j = 0; j < NS; j++) sc[j] = __fmul_rn(sc[j], a.scale);
            }
#pragma unroll
            for (int j = 0; j < NS; j++) {
                const int r = r0 + j * RPS;
                if (r < R) {
                    float v = sc[j];
                    if (live[j] && a.softcap > 0.0f) v = __fmul_rn(a.softcap, tanhf(__fdiv_rn(v, a.softcap)));
                    sp[r * PT + p] = live[j] ? v : -INFINITY;
                }
            }
        }
        __syncthreads();
        /* running softmax: one warp per row */
        for (int r = warp; r < R; r += PA_THREADS / 32) {
            float v[PT / 32], mt = -INFINITY;
#pragma unroll
            for (int j = 0; j < PT / 32; j++) {
                v[j] = sp[r * PT + lane + 32 * j];
                mt = fmaxf(mt, v[j]);
            }
            mt = warp_max(mt);
            const float m_old = smx[r], m_new = fmaxf(m_old, mt);
            float part = 0.0f;
#pragma unroll
            for (int j = 0; j < PT / 32; j++) {
                const float e = m_new == -INFINITY || v[j] == -INFINITY ? 0.0f : expf(__fsub_rn(v[j], m_new));
                sp[r * PT + lane + 32 * j] = e;
                part += e;
            }
            part = warp_sum(part);
            const float alpha = m_new == -INFINITY ? 1.0f : (m_old == -INFINITY ? 0.0f : expf(__fsub_rn(m_old, m_new)));
            if (lane == 0) {
                smx[r] = m_new;
                ssum[r] = __fadd_rn(__fmul_rn(ssum[r], alpha), part);
                salpha[r] = alpha;
            }
        }
        __syncthreads();
        /* out = out * alpha + sum_t p_t V_t over the tile, positions in order; the thread's
         * rows share each V element, their chains interleaved, probabilities read 4 at a time */
#pragma unroll
        for (int k2 = 0; k2 < NO; k2++) {
            const int r = or0 + k2 * rp;
            if (r < R) acc[k2] = __fmul_rn(acc[k2], salpha[r]);
        }
        auto vval = [&](int p) {
            const unsigned char *row = V + (size_t)p * pitch;
            if constexpr (KV == KC_F32) return ((const float *)row)[od];
            else if constexpr (KV == KC_F16) return __half2float(((const __half *)row)[od]);
            else return (float)((const int8_t *)row)[od];
        };
        /* rows in pairs: acc2 = fma((p_r0, p_r1), (v, v), acc2), positions in order */
        uint64_t acc2[NO / 2];
#pragma unroll
        for (int k2 = 0; k2 < NO / 2; k2++) acc2[k2] = f2pack(acc[2 * k2], acc[2 * k2 + 1]);
        const int n4 = nt & ~3;
        for (int p = 0; p < n4; p += 4) {
            const float v0 = vval(p), v1 = vval(p + 1), v2 = vval(p + 2), v3 = vval(p + 3);
            const uint64_t vv0 = f2pack(v0, v0), vv1 = f2pack(v1, v1), vv2 = f2pack(v2, v2), vv3 = f2pack(v3, v3);
#pragma unroll
            for (int k2 = 0; k2 < NO / 2; k2++) {
                const int ra = min(or0 + 2 * k2 * rp, R - 1), rb = min(or0 + (2 * k2 + 1) * rp, R - 1);
                float4 wa = *(const float4 *)(sp + ra * PT + p), wb = *(const float4 *)(sp + rb * PT + p);
                if constexpr (KV == KC_Q8_0) {
                    wa.x = __fmul_rn(wa.x, rvd[p]); wa.y = __fmul_rn(wa.y, rvd[p + 1]);
                    wa.z = __fmul_rn(wa.z, rvd[p + 2]); wa.w = __fmul_rn(wa.w, rvd[p + 3]);
                    wb.x = __fmul_rn(wb.x, rvd[p]); wb.y = __fmul_rn(wb.y, rvd[p + 1]);
                    wb.z = __fmul_rn(wb.z, rvd[p + 2]); wb.w = __fmul_rn(wb.w, rvd[p + 3]);
                }
                acc2[k2] = f2fma(f2pack(wa.x, wb.x), vv0, acc2[k2]);
                acc2[k2] = f2fma(f2pack(wa.y, wb.y), vv1, acc2[k2]);
                acc2[k2] = f2fma(f2pack(wa.z, wb.z), vv2, acc2[k2]);
                acc2[k2] = f2fma(f2pack(wa.w, wb.w), vv3, acc2[k2]);
            }
        }
        for (int p = n4; p < nt; p++) {
            const float vv = vval(p);
            const uint64_t v2 = f2pack(vv, vv);
#pragma unroll
            for (int k2 = 0; k2 < NO / 2; k2++) {
                const int ra = min(or0 + 2 * k2 * rp, R - 1), rb = min(or0 + (2 * k2 + 1) * rp, R - 1);
                float wa = sp[ra * PT + p], wb = sp[rb * PT + p];
                if constexpr (KV == KC_Q8_0) {
                    wa = __fmul_rn(wa, rvd[p]);
                    wb = __fmul_rn(wb, rvd[p]);
                }
                acc2[k2] = f2fma(f2pack(wa, wb), v2, acc2[k2]);
            }
        }
#pragma unroll
        for (int k2 = 0; k2 < NO / 2; k2++) f2unpack(acc2[k2], acc[2 * k2], acc[2 * k2 + 1]);
        __syncthreads();
    }
#pragma unroll
    for (int k2 = 0; k2 < NO; k2++) {
        const int r = or0 + k2 * rp;
        if (r < R)
            a.out[(size_t)(t0 + r / group) * a.q_dim + (size_t)(g * group + r % group) * hd + od] =
                __fdiv_rn(acc[k2], ssum[r]);
    }
}

/* ------------------------------------------------------------ weight repack */

/* Row r, block b of a matrix (Q8: int8 rows; Q4: 16 bytes per block, byte j =
 * element j low nibble and j+16 high nibble, value nibble - 8) into row
 * row0 + r of the packed matrix: int8 quants in the MMA tile layout and the
 * block scale as float. Row r's quants start at q + r * qstride and its
 * scales at d + r * dstride, or, with row_off, both at row_off[r] bytes into
 * q and d (the weight stream's records: quants, then scales). */
__global__ void pf_pack_kernel(const uint8_t *q, size_t qstride, const uint8_t *d, size_t dstride,
                               const unsigned long long *row_off, int type, int d16, int rows, int cols, int row0,
                               int nbk, int8_t *wq, float *wd) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int nb = cols / QK;
    if (i >= (size_t)rows * nb) return;
    const int r = (int)(i / nb), b = (int)(i - (size_t)r * nb);
    const int R = row0 + r, m = R / PF_M, rr = R - m * PF_M;
    const uint8_t *qr = q + (row_off ? row_off[r] : (size_t)r * qstride);
    const uint8_t *dr = d + (row_off ? row_off[r] : (size_t)r * dstride);
    alignas(16) int8_t v[QK];
    if (type == T_Q8) {
        const uint4 *src = (const uint4 *)(qr + (size_t)b * QK);
        *(uint4 *)v = src[0];
        *(uint4 *)(v + 16) = src[1];
    } else {
        const uint8_t *src = qr + (size_t)b * (QK / 2);
        for (int j = 0; j < 16; j++) {
            v[j] = (int8_t)((src[j] & 15) - 8);
            v[j + 16] = (int8_t)((src[j] >> 4) - 8);
        }
    }
    int8_t *dst = wq + ((size_t)m * nbk + b) * PF_A_BLK;
    *(uint4 *)(dst + tile_off(rr, 0)) = *(const uint4 *)v;
    *(uint4 *)(dst + tile_off(rr, 16)) = *(const uint4 *)(v + 16);
    wd[((size_t)m * nbk + b) * PF_M + rr] = d16 ? __half2float(((const __half *)dr)[b]) : ((const float *)dr)[b];
}

/* Token t's quantized activation row (int8 [cols], scales [cols/32]) into
 * the GEMM's token-tile layout. */
__global__ void pf_pack_act_kernel(const int8_t *xq, const float *xd, int n, int cols, int8_t *tq, float *td) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int nb = cols / QK, tpad = (n + PF_N - 1) / PF_N * PF_N;
    if (i >= (size_t)tpad * nb) return;
    const int t = (int)(i / nb), b = (int)(i - (size_t)t * nb), nt = t / PF_N, tr = t - nt * PF_N;
    uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
    float d = 0.0f;
    if (t < n) {
        const uint4 *src = (const uint4 *)(xq + (size_t)t * cols + (size_t)b * QK);
        lo = src[0];
        hi = src[1];
        d = xd[(size_t)t * nb + b];
    }
    int8_t *blk = tq + ((size_t)nt * nb + b) * PF_B_BLK;
    *(uint4 *)(blk + tile_off(tr, 0)) = lo;
    *(uint4 *)(blk + tile_off(tr, 16)) = hi;
    td[((size_t)nt * nb + b) * PF_N + tr] = d;
}

/* ------------------------------------------------------------ host side */

namespace {

int cuda_err(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return KC_OK;
    set_error(std::string("prefill: ") + what + ": " + cudaGetErrorString(e));
    (void)cudaGetLastError();
    return e == cudaErrorMemoryAllocation ? KC_E_NOMEM : KC_E_IO;
}
#define PCK(call, what)                                    \
    do {                                                   \
        const cudaError_t e_ = (call);                     \
        if (e_ != cudaSuccess) return cuda_err(e_, what);  \
    } while (0)

size_t up256(size_t n) { return (n + 255) & ~(size_t)255; }

/* One packed GEMM operand. */
struct PfMat {
    int8_t *q = nullptr;
    float *d = nullptr;
    float *bias = nullptr;
    int rows = 0, cols = 0, mt = 0, nbk = 0;
};

struct PfLayerW {
    PfMat qkv, wo, w13, w2;
};

}  // namespace

struct PfModel {
    std::vector<PfLayerW> layers;
    PfMat cls;
    bool have_cls = false;
    std::vector<void *> allocs;
    size_t bytes = 0;
    ~PfModel() {
        for (void *p : allocs) cudaFree(p);
    }
};

struct PfScratch {
    int tc = 0;                  /* tokens per chunk (a multiple of PF_N) */
    size_t npos = 0;
    void *base = nullptr;
    float *x = nullptr, *qkv = nullptr, *ao = nullptr, *gu = nullptr, *xd = nullptr, *qd = nullptr, *y = nullptr;
    int8_t *xq = nullptr, *qq = nullptr;
    int *tok = nullptr;
    ~PfScratch() {
        if (base) cudaFree(base);
    }
};

namespace {

/* Bytes of one packed operand: quants [mt][nbk][PF_A_BLK], scales [mt][nbk][PF_M] (each 256-aligned). */
size_t mat_bytes(int rows, int cols) {
    const size_t mt = (size_t)(rows + PF_M - 1) / PF_M, nbk = (size_t)cols / QK;
    return up256(mt * nbk * PF_A_BLK) + up256(mt * nbk * PF_M * sizeof(float));
}

/* A packed operand of rows x cols, carved from *arena (advanced) or, without
 * one, in its own allocation. The padding rows of the last row tile stay
 * unwritten: they only feed output rows the GEMM never stores. */
int alloc_mat(PfModel &P, PfMat &M, int rows, int cols, uint8_t **arena = nullptr) {
    M.rows = rows;
    M.cols = cols;
    M.mt = (rows + PF_M - 1) / PF_M;
    M.nbk = cols / QK;
    const size_t qb = up256((size_t)M.mt * M.nbk * PF_A_BLK);
    uint8_t *base = nullptr;
    if (arena) {
        base = *arena;
        *arena += mat_bytes(rows, cols);
    } else {
        void *b = nullptr;
        PCK(cudaMalloc(&b, mat_bytes(rows, cols)), "packed weights");
        P.allocs.push_back(b);
        P.bytes += mat_bytes(rows, cols);
        base = (uint8_t *)b;
    }
    M.q = (int8_t *)base;
    M.d = (float *)(base + qb);
    return KC_OK;
}

/* Packs rows [0, rows) of one weight-stream matrix (records at the offsets
 * row_off, in the stream's types) into rows row0.. of M. */
int pack_rows(const uint8_t *stream, const unsigned long long *row_off, int rows, int type, int d16, int row0, PfMat &M,
              cudaStream_t st) {
    if (row0 + rows > M.rows || (type != T_Q8 && type != T_Q4)) {
        set_error("prefill: a matrix does not fit its packed operand");
        return KC_E_SHAPE;
    }
    const int qrow = type == T_Q4 ? M.cols / 2 : M.cols;
    const size_t items = (size_t)rows * (M.cols / QK);
    pf_pack_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(stream, 0, stream + qrow, 0, row_off, type, d16,
                                                                     rows, M.cols, row0, M.nbk, M.q, M.d);
    PCK(cudaGetLastError(), "pack kernel");
    return KC_OK;
}

/* The stacked bias of a packed operand from the layer's host arrays. */
int stack_bias(PfModel &P, PfMat &M, const std::vector<std::pair<const float *, int>> &parts, cudaStream_t st) {
    void *b = nullptr;
    PCK(cudaMalloc(&b, sizeof(float) * (size_t)M.rows), "bias");
    P.allocs.push_back(b);
    size_t off = 0;
    for (const auto &pr : parts) {
        PCK(cudaMemcpyAsync((float *)b + off, pr.first, sizeof(float) * (size_t)pr.second, cudaMemcpyHostToDevice, st),
            "bias copy");
        off += (size_t)pr.second;
    }
    M.bias = (float *)b;
    return KC_OK;
}

int pack_all(kc_model *m, const uint8_t *stream, const PfRowTable &t, PfModel &P, cudaStream_t st) {
    const kc_config &c = m->cfg;
    const HostLayer &H0 = m->layers[0];
    const HostMat &cls = m->shared ? m->tok_emb : m->wcls;
    auto ty = [](const HostMat &h) { return h.type == KC_Q4_0 ? T_Q4 : T_Q8; };
    const size_t nq = (size_t)c.q_dim + 2 * (size_t)c.kv_dim, nd = (size_t)c.dim, nh = 2 * (size_t)c.hidden_dim;
    P.layers.resize((size_t)c.n_layers);
    /* one allocation for every operand */
    const size_t per_layer = mat_bytes((int)nq, c.dim) + mat_bytes(c.dim, c.q_dim) + mat_bytes((int)nh, c.dim) +
                             mat_bytes(c.dim, c.hidden_dim);
    const size_t total = per_layer * (size_t)c.n_layers + mat_bytes(c.vocab, c.dim);
    void *base = nullptr;
    PCK(cudaMalloc(&base, total), "packed weights");
    P.allocs.push_back(base);
    P.bytes += total;
    uint8_t *arena = (uint8_t *)base;
    int r;
    for (int l = 0; l < c.n_layers; l++) {
        const HostLayer &H = m->layers[(size_t)l];
        PfLayerW &W = P.layers[(size_t)l];
        const unsigned long long *q = t.qkv + l * nq;
        if ((r = alloc_mat(P, W.qkv, (int)nq, c.dim, &arena)) != KC_OK) return r;
        if ((r = pack_rows(stream, q, c.q_dim, ty(H0.wq), t.d16, 0, W.qkv, st)) != KC_OK) return r;
        if ((r = pack_rows(stream, q + c.q_dim, c.kv_dim, ty(H0.wk), t.d16, c.q_dim, W.qkv, st)) != KC_OK) return r;
        if ((r = pack_rows(stream, q + c.q_dim + c.kv_dim, c.kv_dim, ty(H0.wv), t.d16, c.q_dim + c.kv_dim, W.qkv,
                           st)) != KC_OK)
            return r;
        if (H.bq && (r = stack_bias(P, W.qkv, { { H.bq, c.q_dim }, { H.bk, c.kv_dim }, { H.bv, c.kv_dim } }, st)) != KC_OK)
            return r;
        if ((r = alloc_mat(P, W.wo, c.dim, c.q_dim, &arena)) != KC_OK) return r;
        if ((r = pack_rows(stream, t.wo + l * nd, c.dim, ty(H0.wo), t.d16, 0, W.wo, st)) != KC_OK) return r;
        if ((r = alloc_mat(P, W.w13, (int)nh, c.dim, &arena)) != KC_OK) return r;
        if ((r = pack_rows(stream, t.w13 + l * nh, (int)nh, ty(H0.w1), t.d16, 0, W.w13, st)) != KC_OK) return r;
        if ((r = alloc_mat(P, W.w2, c.dim, c.hidden_dim, &arena)) != KC_OK) return r;
        if ((r = pack_rows(stream, t.w2 + l * nd, c.dim, ty(H0.w2), t.d16, 0, W.w2, st)) != KC_OK) return r;
    }
    if ((r = alloc_mat(P, P.cls, c.vocab, c.dim, &arena)) != KC_OK) return r;
    if ((r = pack_rows(stream, t.cls, c.vocab, ty(cls), t.d16, 0, P.cls, st)) != KC_OK) return r;
    P.have_cls = true;
    return KC_OK;
}

size_t kv_es(int kv_type) { return kv_type == KC_F32 ? 4 : (kv_type == KC_F16 ? 2 : 1); }
int attn_tile(const kc_config &c) { return c.head_dim <= 64 ? 64 : 32; }
bool attn_hd_ok(int hd) { return hd == 16 || hd == 32 || hd == 64 || hd == 128; }
int attn_smem_bytes(const kc_config &c, int kv_type) {
    return (int)pa_smem_bytes(c.head_dim, (int)kv_es(kv_type), attn_tile(c));
}

int ensure_scratch(PfScratch *&S, const kc_config &c, int tc, size_t npos) {
    if (S && S->tc >= tc && S->npos >= npos) return KC_OK;
    delete S;
    S = new (std::nothrow) PfScratch();
    if (!S) return KC_E_NOMEM;
    const size_t T = (size_t)tc, wide = (size_t)std::max(std::max(c.dim, c.q_dim), c.hidden_dim);
    struct B { void **p; size_t bytes; };
    std::vector<B> bufs = {
        { (void **)&S->x, sizeof(float) * T * c.dim },
        { (void **)&S->y, sizeof(float) * T * c.dim },
        { (void **)&S->qkv, sizeof(float) * T * (size_t)(c.q_dim + 2 * c.kv_dim) },
        { (void **)&S->ao, sizeof(float) * T * c.q_dim },
        { (void **)&S->gu, sizeof(float) * T * 2 * (size_t)c.hidden_dim },
        { (void **)&S->xq, T * wide },
        { (void **)&S->xd, sizeof(float) * T * (wide / QK) },
        { (void **)&S->qq, T * c.q_dim },
        { (void **)&S->qd, sizeof(float) * T * c.n_heads },
        { (void **)&S->tok, sizeof(int) * T },
    };
    size_t total = 0;
    for (const B &b : bufs) total += up256(b.bytes);
    PCK(cudaMalloc(&S->base, total), "prefill scratch");
    size_t off = 0;
    for (const B &b : bufs) {
        *b.p = (uint8_t *)S->base + off;
        off += up256(b.bytes);
    }
    S->tc = tc;
    S->npos = npos;
    return KC_OK;
}

void launch_quant(const PfScratch &S, const float *x, int ldx, const float *w, float eps, int mode, int act, int cols,
                  int T, cudaStream_t st) {
    PfQuant q{ x, ldx, w, eps, mode, act, cols, T, cols / QK, S.xq, S.xd };
    const int tpad = (T + PF_N - 1) / PF_N * PF_N;
    pf_quant_kernel<<<tpad, 256, 0, st>>>(q);
}

void launch_gemm(const PfMat &W, const PfScratch &S, int T, float *out, int ldo, int mode, float softcap,
                 unsigned *err, cudaStream_t st, int tok0 = 0) {
    PfGemm g;
    g.wq = W.q; g.wd = W.d; g.bias = W.bias;
    g.xq = S.xq + (size_t)(tok0 / PF_N) * W.nbk * PF_B_BLK;
    g.xd = S.xd + (size_t)(tok0 / PF_N) * W.nbk * PF_N;
    g.out = out; g.ldo = ldo; g.rows = W.rows; g.T = T; g.nbk = W.nbk; g.mode = mode; g.softcap = softcap; g.err = err;
    const dim3 grid((unsigned)((T + PF_N - 1) / PF_N), (unsigned)W.mt);
    pf_gemm_kernel<<<grid, PF_THREADS, PF_SMEM, st>>>(g);
}

int set_attributes(int attn_smem) {
    static int done_gemm = 0;
    if (!done_gemm) {
        PCK(cudaFuncSetAttribute(pf_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM), "gemm smem");
        done_gemm = 1;
    }
    const cudaFuncAttribute A = cudaFuncAttributeMaxDynamicSharedMemorySize;
#define PA_ATTR(KV, HD) PCK(cudaFuncSetAttribute(pf_attn_kernel<KV, HD>, A, attn_smem), "attn")
    PA_ATTR(KC_F32, 16); PA_ATTR(KC_F32, 32); PA_ATTR(KC_F32, 64); PA_ATTR(KC_F32, 128);
    PA_ATTR(KC_F16, 16); PA_ATTR(KC_F16, 32); PA_ATTR(KC_F16, 64); PA_ATTR(KC_F16, 128);
    PA_ATTR(KC_Q8_0, 16); PA_ATTR(KC_Q8_0, 32); PA_ATTR(KC_Q8_0, 64); PA_ATTR(KC_Q8_0, 128);
#undef PA_ATTR
    return KC_OK;
}

template <int HD>
void launch_attn(const PfAttn &at, dim3 grid, int smem, int kv_type, cudaStream_t st) {
    if (kv_type == KC_F32) pf_attn_kernel<KC_F32, HD><<<grid, PA_THREADS, smem, st>>>(at);
    else if (kv_type == KC_F16) pf_attn_kernel<KC_F16, HD><<<grid, PA_THREADS, smem, st>>>(at);
    else pf_attn_kernel<KC_Q8_0, HD><<<grid, PA_THREADS, smem, st>>>(at);
}

}  // namespace

/* Shared memory the batched attention needs for a chunk reaching position
 * last_pos; > PF_ATTN_SMEM_MAX means the batched path cannot take it. */
bool pf_fits(const kc_config &c, int kv_type, int last_pos) {
    const int group = c.n_heads / c.n_kv_heads;
    if (group > PA_MAXG || group > PA_ROWS || c.head_dim % 4) return false;
    if (c.qk_norm && c.n_heads + c.n_kv_heads > PR_MAX_HEADS) return false;
    if (c.dim % QK || c.q_dim % QK || c.hidden_dim % QK) return false;
    (void)last_pos;
    if ((c.head_dim * (int)kv_es(kv_type)) % 16 || !attn_hd_ok(c.head_dim)) return false;
    return attn_smem_bytes(c, kv_type) <= PF_ATTN_SMEM_MAX;
}

int pf_pack_model(kc_model *m, const uint8_t *stream, const PfRowTable &t, cudaStream_t st) {
    PfModel *P = new (std::nothrow) PfModel();
    if (!P) return KC_E_NOMEM;
    int rc = pack_all(m, stream, t, *P, st);
    if (rc == KC_OK) {
        const cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_err(e, "weight repack");
    }
    if (rc != KC_OK) {
        delete P;
        return rc;
    }
    pf_free_model(m->pf);
    m->pf = P;
    return KC_OK;
}

void pf_free_model(PfModel *p) { delete p; }
void pf_free_scratch(PfScratch *p) { delete p; }
size_t pf_model_bytes(const PfModel *p) { return p ? p->bytes : 0; }

int pf_prefill(const PfRun &r, const int *tokens, int n, int pos0, float *logits) {
    const kc_config &c = r.m->cfg;
    cudaStream_t st = r.st;
    if (!r.m->pf || !r.m->pf->have_cls) {
        set_error("prefill: the model's GEMM operands were not packed at upload");
        return KC_E_SHAPE;
    }
    PfModel &P = *r.m->pf;
    const int tc = std::max(PF_N, std::min(r.batch, n) + PF_N - 1) / PF_N * PF_N;
    const size_t npos = (size_t)pos0 + n;
    int rc = ensure_scratch(*r.scratch, c, tc, npos);
    if (rc != KC_OK) return rc;
    PfScratch &S = **r.scratch;
    const int asmem = attn_smem_bytes(c, r.kv_type);
    rc = set_attributes(asmem);
    if (rc != KC_OK) return rc;
    const int group = c.n_heads / c.n_kv_heads, ldq = c.q_dim + 2 * c.kv_dim;
    PCK(cudaMemsetAsync(r.err, 0, sizeof(unsigned), st), "error word");
    for (int i0 = 0; i0 < n; i0 += tc) {
        const int T = std::min(tc, n - i0), p0 = pos0 + i0;
        PCK(cudaMemcpyAsync(S.tok, tokens + i0, sizeof(int) * (size_t)T, cudaMemcpyHostToDevice, st), "tokens");
        PfEmbed e{ r.emb_q, r.emb_d, r.emb_type, r.emb_d16, c.embed_scale, S.tok, c.dim, S.x };
        pf_embed_kernel<<<T, 256, 0, st>>>(e);
        for (int l = 0; l < c.n_layers; l++) {
            const PfLayerW &W = P.layers[(size_t)l];
            const PfLayerRun &L = r.layers[l];
            launch_quant(S, S.x, c.dim, L.attn_norm, c.norm_eps, PQ_NORM, c.act, c.dim, T, st);
            launch_gemm(W.qkv, S, T, S.qkv, ldq, PF_STORE, 0.0f, r.err, st);
            PfRope ro{ S.qkv, ldq, L.rcos, L.rsin, L.kc, L.vc, L.kd, L.vd, S.qq, S.qd,
                       p0, c.head_dim, c.n_heads, c.n_kv_heads, c.q_dim, c.kv_dim, r.kv_type,
                       L.q_norm, L.k_norm, c.norm_eps };
            pf_rope_kernel<<<T, 256, 0, st>>>(ro);
            const int tq = std::max(1, PA_ROWS / group);
            PfAttn at{ S.qkv, ldq, S.qq, S.qd, L.kc, L.vc, L.kd, L.vd, S.ao,
                       T, p0, c.head_dim, c.n_heads, c.n_kv_heads, c.q_dim, c.kv_dim, L.window, tq,
                       c.attn_scale, c.attn_softcap };
            const dim3 ag((unsigned)((T + tq - 1) / tq), (unsigned)c.n_kv_heads);
            if (c.head_dim == 16) launch_attn<16>(at, ag, asmem, r.kv_type, st);
            else if (c.head_dim == 32) launch_attn<32>(at, ag, asmem, r.kv_type, st);
            else if (c.head_dim == 64) launch_attn<64>(at, ag, asmem, r.kv_type, st);
            else launch_attn<128>(at, ag, asmem, r.kv_type, st);
            launch_quant(S, S.ao, c.q_dim, nullptr, 0.0f, PQ_PLAIN, c.act, c.q_dim, T, st);
            if (L.post_attn) {
                launch_gemm(W.wo, S, T, S.y, c.dim, PF_STORE, 0.0f, r.err, st);
                pf_post_kernel<<<T, 256, 0, st>>>(S.x, S.y, L.post_attn, c.dim, c.norm_eps);
            } else {
                launch_gemm(W.wo, S, T, S.x, c.dim, PF_RESID, 0.0f, r.err, st);
            }
            launch_quant(S, S.x, c.dim, L.ffn_norm, c.norm_eps, PQ_NORM, c.act, c.dim, T, st);
            launch_gemm(W.w13, S, T, S.gu, 2 * c.hidden_dim, PF_STORE, 0.0f, r.err, st);
            launch_quant(S, S.gu, 2 * c.hidden_dim, nullptr, 0.0f, PQ_GATED, c.act, c.hidden_dim, T, st);
            if (L.post_ffn) {
                launch_gemm(W.w2, S, T, S.y, c.dim, PF_STORE, 0.0f, r.err, st);
                pf_post_kernel<<<T, 256, 0, st>>>(S.x, S.y, L.post_ffn, c.dim, c.norm_eps);
            } else {
                launch_gemm(W.w2, S, T, S.x, c.dim, PF_RESID, 0.0f, r.err, st);
            }
        }
        (void)group;
        PCK(cudaGetLastError(), "prefill launch");
        if (logits) {
            launch_quant(S, S.x, c.dim, r.final_norm, c.norm_eps, PQ_NORM, c.act, c.dim, T, st);
            for (int s0 = 0; s0 < T; s0 += r.logits_rows) {
                const int k = std::min(r.logits_rows, T - s0);
                launch_gemm(P.cls, S, k, r.logits_dev, c.vocab, PF_STORE, c.final_softcap, r.err, st, s0);
                PCK(cudaGetLastError(), "classifier launch");
                PCK(cudaMemcpyAsync(logits + (size_t)(i0 + s0) * c.vocab, r.logits_dev, sizeof(float) * (size_t)k * c.vocab,
                                    cudaMemcpyDeviceToHost, st),
                    "logits copy");
            }
        }
    }
    unsigned err = 0;
    PCK(cudaMemcpyAsync(&err, r.err, sizeof err, cudaMemcpyDeviceToHost, st), "error word");
    PCK(cudaStreamSynchronize(st), "prefill");
    if (err) {
        set_error("prefill: a pipeline wait gave up (error word " + std::to_string(err) + ")");
        return KC_E_IO;
    }
    return KC_OK;
}

}  // namespace kc

using namespace kc;

/* ml_matmul (ops/ops.c:51-79) on device buffers: y[t * rows + r] = W x_t for n
 * quantized activation rows, through the prefill's packed weights and tensor-core
 * GEMM (weights repacked per call into temporary device memory). */
extern "C" int kc_matmul_dev(float *y, int type, int d_f16, const void *wq, const void *wd, int rows, int cols,
                             const int8_t *xq, const float *xd, int n, void *stream) {
    clear_error();
    if (rows <= 0 || cols <= 0 || n <= 0 || cols % QK || (type != KC_Q8_0 && type != KC_Q4_0)) return KC_E_SHAPE;
    cudaStream_t st = (cudaStream_t)stream;
    PfModel P;
    PfMat W;
    int rc = alloc_mat(P, W, rows, cols);
    if (rc != KC_OK) return rc;
    const size_t items = (size_t)rows * (cols / QK);
    const size_t qrow = type == KC_Q4_0 ? (size_t)cols / 2 : (size_t)cols, drow = (size_t)(cols / QK) * (d_f16 ? 2 : 4);
    pf_pack_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>((const uint8_t *)wq, qrow, (const uint8_t *)wd, drow,
                                                                     nullptr, type == KC_Q4_0 ? T_Q4 : T_Q8, d_f16, rows,
                                                                     cols, 0, W.nbk, W.q, W.d);
    const int tpad = (n + PF_N - 1) / PF_N * PF_N;
    PfScratch S;
    void *buf = nullptr;
    const size_t qb = up256((size_t)tpad * cols), db = sizeof(float) * (size_t)tpad * (cols / QK);
    PCK(cudaMalloc(&buf, qb + db), "activation tiles");
    S.base = buf;
    S.xq = (int8_t *)buf;
    S.xd = (float *)((uint8_t *)buf + qb);
    const size_t aitems = (size_t)tpad * (cols / QK);
    pf_pack_act_kernel<<<(unsigned)((aitems + 255) / 256), 256, 0, st>>>(xq, xd, n, cols, S.xq, S.xd);
    unsigned *err = nullptr;
    PCK(cudaMalloc(&err, sizeof(unsigned)), "error word");
    rc = set_attributes(48 * 1024);
    if (rc == KC_OK) {
        cudaMemsetAsync(err, 0, sizeof(unsigned), st);
        launch_gemm(W, S, n, y, rows, PF_STORE, 0.0f, err, st);
        unsigned h = 0;
        cudaMemcpyAsync(&h, err, sizeof h, cudaMemcpyDeviceToHost, st);
        const cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_err(e, "matmul");
        else if (h) {
            set_error("matmul: a pipeline wait gave up");
            rc = KC_E_IO;
        }
    }
    cudaFree(err);
    return rc;
}
