/* Device-side next-token sampler: ml_sample (model/sampler.c:39-165) over a
 * logits row in device memory, one CTA, so that sampled generation needs no
 * logits copy to the host.
 *
 * Steps, as the reference takes them:
 *   penalty       each distinct token of the recent ring once: a positive logit
 *                 divided by repeat_penalty, a negative one multiplied (:30-42);
 *   greedy        temperature 0: first index of the maximum (:57-61);
 *   softmax       logits / temperature, max, exp(x - max), sum, times 1/sum
 *                 (kernels/scalar/k_scalar.c:66-77, all -inf -> uniform);
 *   coin          xorshift64* (:44-49), the same integer stream as the host;
 *   top-k / top-p the tokens ordered by probability, ties by lower id
 *                 (cmp_desc, :73-78): the k best (top-k), or the tokens at
 *                 or above the top-p cutoff (top-p alone), by a radix select
 *                 of the k-th key and a bitonic sort of the k; past 2048 of
 *                 them, a stable LSD radix sort of all tokens on the
 *                 probability's bits; then the reference's sample_sorted by
 *                 one thread, or sample_topp's running sums in blocks;
 *   multinomial   neither: the first token whose cumulative probability
 *                 exceeds the coin (:63-70).
 * The sums over all tokens (softmax, the multinomial prefix) are block
 * reductions and blocked scans, not the reference's single running sum; with
 * CUDA's expf that moves a probability by an ulp or so, which changes a choice
 * only when the coin lies that close to a cumulative boundary. */
#pragma once
#include <cstdint>

#include "kc_kernels.cuh"

namespace kc {

constexpr int SM_THREADS = 1024;
constexpr int SM_WARPS = SM_THREADS / 32;

struct SamplerDev {
    unsigned long long rng;   /* xorshift64* state */
    int n_recent, recent_at;  /* the ring of the last repeat_last_n accepted tokens */
};

struct SampleArgs {
    const float *logits;      /* [vocab] */
    int vocab;
    float temperature, topp, repeat_penalty;
    int topk, repeat_last_n;
    SamplerDev *st;
    int *recent;              /* [repeat_last_n] */
    float *p;                 /* [vocab] scratch */
    unsigned *ka, *kb;        /* [vocab] sort keys (ping-pong) */
    int *va, *vb;             /* [vocab] token ids */
    int *token_out;           /* the sampled token */
    LoopState *ls;            /* optional: the device loop, advanced to the token */
    int *out_tokens;          /* optional, with ls: the step's slot */
};

__device__ __forceinline__ float sm_block_max(float v, float *red) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < SM_WARPS; i++) r = fmaxf(r, red[i]);
    return r;
}

__device__ __forceinline__ float sm_block_sum(float v, float *red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < SM_WARPS; i++) r = __fadd_rn(r, red[i]);
    return r;
}

/* Stable ascending LSD radix sort of (key, id) over n entries by the whole
 * block, 8-bit digits; result in (ka, va). hist: [SM_WARPS][256] shared. */
__device__ void sm_radix_sort(unsigned *ka, int *va, unsigned *kb, int *vb, int n, int *hist, int *tot) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int chunk = (n + SM_WARPS - 1) / SM_WARPS, lo = w * chunk, hi = min(n, lo + chunk);
    const unsigned lt = (1u << lane) - 1u;
    for (int shift = 0; shift < 32; shift += 8) {
        for (int i = threadIdx.x; i < SM_WARPS * 256; i += SM_THREADS) hist[i] = 0;
        __syncthreads();
        for (int i = lo + lane; i < hi; i += 32) atomicAdd(&hist[w * 256 + ((ka[i] >> shift) & 255u)], 1);
        __syncthreads();
        /* offsets digit-major, then warp order within a digit: stable */
        if (threadIdx.x < 256) {
            int s = 0;
            for (int k = 0; k < SM_WARPS; k++) s += hist[k * 256 + threadIdx.x];
            tot[threadIdx.x] = s;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int s = 0;
            for (int d = 0; d < 256; d++) {
                const int t = tot[d];
                tot[d] = s;
                s += t;
            }
        }
        __syncthreads();
        if (threadIdx.x < 256) {
            int s = tot[threadIdx.x];
            for (int k = 0; k < SM_WARPS; k++) {
                const int c = hist[k * 256 + threadIdx.x];
                hist[k * 256 + threadIdx.x] = s;
                s += c;
            }
        }
        __syncthreads();
        /* each warp scatters its range in order, lanes of equal digit by lane */
        for (int base = lo; base < hi; base += 32) {
            const int i = base + lane;
            const bool live = i < hi;
            const unsigned key = live ? ka[i] : 0u;
            const int id = live ? va[i] : 0;
            const unsigned d = live ? ((key >> shift) & 255u) : 256u;
            const unsigned peers = __match_any_sync(0xffffffffu, d);
            const int rank = __popc(peers & lt);
            int pos = 0;
            if (live) pos = hist[w * 256 + d] + rank;
            __syncwarp();
            if (live && rank == 0) hist[w * 256 + d] += __popc(peers);
            __syncwarp();
            if (live) {
                kb[pos] = key;
                vb[pos] = id;
            }
        }
        __syncthreads();
        unsigned *tk = ka; ka = kb; kb = tk;
        int *tv = va; va = vb; vb = tv;
    }
    /* four passes: the result is back in the caller's (ka, va) */
}

constexpr int SM_TOPK_MAX = 2048;   /* top-k by selection up to this k; the full sort beyond */

/* The k smallest keys (ties by lower id) of ka[0, n), ascending by (key, id),
 * into cand[0, k) as key << 32 | id: an MSB-first radix select of the k-th key
 * (4 histogram passes), every key below it and the lowest ids equal to it, then
 * a bitonic sort in shared memory. k <= SM_TOPK_MAX. */
__device__ void sm_topk_select(const unsigned *ka, int n, int k, unsigned long long *cand, int *hist, int *s_cnt) {
    const int tid = threadIdx.x;
    __shared__ unsigned s_prefix, s_mask;
    __shared__ int s_k;
    if (tid == 0) {
        s_prefix = 0u;
        s_mask = 0u;
        s_k = k;
    }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += SM_THREADS) hist[i] = 0;
        __syncthreads();
        const unsigned prefix = s_prefix, mask = s_mask;
        for (int i = tid; i < n; i += SM_THREADS) {
            const unsigned key = ka[i];
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
        }
        __syncthreads();
        if (tid == 0) {
            int kk = s_k, d = 0;
            for (; d < 255 && hist[d] < kk; d++) kk -= hist[d];
            s_k = kk;
            s_prefix = prefix | ((unsigned)d << shift);
            s_mask = mask | (255u << shift);
        }
        __syncthreads();
    }
    const unsigned T = s_prefix;
    const int kk = s_k;   /* ids with key == T to take, the lowest first */
    /* keys below T: any order (sorted below); keys equal to T: the first kk by id */
    if (tid == 0) *s_cnt = 0;
    const int chunk = (n + SM_THREADS - 1) / SM_THREADS, lo = tid * chunk, hi = min(n, lo + chunk);
    int eq = 0;
    for (int i = lo; i < hi; i++) eq += ka[i] == T;
    __syncthreads();
    int *eqs = hist;   /* per-thread counts of keys equal to T, then their exclusive prefix */
    eqs[tid] = eq;
    __syncthreads();
    if (tid == 0) {
        int s = 0;
        for (int t = 0; t < SM_THREADS; t++) {
            const int c = eqs[t];
            eqs[t] = s;
            s += c;
        }
    }
    __syncthreads();
    int rank = eqs[tid];
    for (int i = lo; i < hi; i++) {
        const unsigned key = ka[i];
        if (key < T || (key == T && rank++ < kk)) {
            const int at = atomicAdd(s_cnt, 1);
            if (at < SM_TOPK_MAX) cand[at] = ((unsigned long long)key << 32) | (unsigned)i;
        }
    }
    __syncthreads();
    int m = 1;
    while (m < k) m <<= 1;
    for (int i = k + tid; i < m; i += SM_THREADS) cand[i] = ~0ull;
    __syncthreads();
    for (int size = 2; size <= m; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < m; i += SM_THREADS) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    const unsigned long long x = cand[i], y = cand[j];
                    if ((x > y) == up) {
                        cand[i] = y;
                        cand[j] = x;
                    }
                }
            }
            __syncthreads();
        }
}

/* xorshift64*, uniform in [0, 1): model/sampler.c:44-49 */
__device__ __forceinline__ float sm_random_f32(unsigned long long *st) {
    unsigned long long x = *st;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *st = x;
    return (float)((unsigned)((x * 0x2545F4914F6CDD1Dull) >> 32) >> 8) / 16777216.0f;
}

__global__ void __launch_bounds__(SM_THREADS, 1) sample_kernel(const SampleArgs a) {
    __shared__ float red[SM_WARPS];
    __shared__ int hist[SM_WARPS * 256];
    __shared__ int tot[256];
    __shared__ int s_tok;
    __shared__ float s_coin;
    __shared__ unsigned long long s_best;
    const int n = a.vocab, tid = threadIdx.x;
    float *p = a.p;
    /* logits, penalized (each distinct recent token once, :30-42) */
    for (int i = tid; i < n; i += SM_THREADS) p[i] = a.logits[i];
    __syncthreads();
    const SamplerDev st = *a.st;
    if (a.repeat_penalty != 1.0f && st.n_recent > 0) {
        for (int i = tid; i < st.n_recent; i += SM_THREADS) {
            const int t = a.recent[i];
            bool first = t >= 0 && t < n;
            for (int j = 0; j < i && first; j++) first = a.recent[j] != t;
            if (first) {
                const float v = p[t];
                p[t] = v > 0.0f ? __fdiv_rn(v, a.repeat_penalty) : __fmul_rn(v, a.repeat_penalty);
            }
        }
        __syncthreads();
    }
    if (tid == 0) s_best = 0ull;
    __syncthreads();
    if (a.temperature == 0.0f) {
        /* greedy: first index of the maximum */
        unsigned long long best = 0ull;
        for (int i = tid; i < n; i += SM_THREADS) {
            const unsigned long long k = argmax_key(p[i], i);
            best = k > best ? k : best;
        }
        atomicMax(&s_best, best);
        __syncthreads();
        if (tid == 0) s_tok = (int)(0xffffffffu - (unsigned)(s_best & 0xffffffffull));
    } else {
        /* softmax of logits / temperature */
        float mx = -INFINITY;
        for (int i = tid; i < n; i += SM_THREADS) {
            const float q = __fdiv_rn(p[i], a.temperature);
            p[i] = q;
            mx = fmaxf(mx, q);
        }
        mx = sm_block_max(mx, red);
        if (mx == -INFINITY) {
            const float u = __fdiv_rn(1.0f, (float)n);
            for (int i = tid; i < n; i += SM_THREADS) p[i] = u;
        } else {
            float sum = 0.0f;
            for (int i = tid; i < n; i += SM_THREADS) {
                const float e = expf(__fsub_rn(p[i], mx));
                p[i] = e;
                sum = __fadd_rn(sum, e);
            }
            sum = sm_block_sum(sum, red);
            const float inv = __fdiv_rn(1.0f, sum);
            for (int i = tid; i < n; i += SM_THREADS) p[i] = __fmul_rn(p[i], inv);
        }
        if (tid == 0) {
            unsigned long long r = st.rng;
            s_coin = sm_random_f32(&r);
            a.st->rng = r;
        }
        __syncthreads();
        const float coin = s_coin;
        const bool use_k = a.topk > 0 && a.topk < n, use_p = a.topp > 0.0f && a.topp < 1.0f;
        if (use_k || use_p) {
            /* the tokens by probability descending, ties by lower id: the k best by selection,
             * or every token by a full sort. Without top-k only the tokens at or above the
             * top-p cutoff (sample_topp, :133-155) are candidates, counted first. */
            const float cutoff = n > 1 ? __fdiv_rn(__fsub_rn(1.0f, a.topp), (float)(n - 1)) : 0.0f;
            __shared__ int s_m;
            if (tid == 0) s_m = 0;
            __syncthreads();
            int c = 0;
            for (int i = tid; i < n; i += SM_THREADS) {
                const float q = p[i];
                a.ka[i] = ~__float_as_uint(q);
                a.va[i] = i;
                c += q >= cutoff;
            }
            if (!use_k) atomicAdd(&s_m, c);
            __syncthreads();
            const int m_p = s_m;                               /* top-p candidates (top-p only) */
            const int ksel = use_k ? a.topk : max(m_p, 1);     /* one: the argmax when none pass */
            const bool select = ksel <= SM_TOPK_MAX;
            __shared__ int s_cnt;
            if (select) {
                unsigned long long *cand = (unsigned long long *)a.kb;   /* [SM_TOPK_MAX] in the spare key buffer */
                sm_topk_select(a.ka, n, ksel, cand, hist, &s_cnt);
                for (int i = tid; i < ksel; i += SM_THREADS) {
                    a.ka[i] = (unsigned)(cand[i] >> 32);
                    a.va[i] = (int)(unsigned)cand[i];
                }
                __syncthreads();
            } else {
                sm_radix_sort(a.ka, a.va, a.kb, a.vb, n, hist, tot);
            }
            const unsigned *k = a.ka;
            const int *v = a.va;
            auto pr = [&](int i) { return __uint_as_float(~k[i]); };
            if (use_k) {
                if (tid == 0) {
                    /* sample_sorted (:108-131) over the k best */
                    const int m = a.topk;
                    float total = 0.0f;
                    for (int i = 0; i < m; i++) total = __fadd_rn(total, pr(i));
                    int last = m - 1;
                    if (use_p) {
                        float cum = 0.0f;
                        const float lim = __fmul_rn(a.topp, total);
                        for (int i = 0; i < m; i++) {
                            cum = __fadd_rn(cum, pr(i));
                            if (cum > lim) { last = i; break; }
                        }
                        total = cum;
                    }
                    const float r = __fmul_rn(coin, total);
                    float cdf = 0.0f;
                    int tok = v[last];
                    for (int i = 0; i <= last; i++) {
                        cdf = __fadd_rn(cdf, pr(i));
                        if (r < cdf) { tok = v[i]; break; }
                    }
                    s_tok = tok;
                }
            } else {
                /* sample_topp (:133-155): the m tokens at or above the cutoff lead the
                 * order; their running sums in blocks (per-thread ranges in order) */
                const int m = m_p;
                if (m == 0) {
                    if (tid == 0) s_tok = v[0];   /* argmax: the first in this order is the first index of the maximum */
                } else {
                    const int chunk = (m + SM_THREADS - 1) / SM_THREADS, lo = tid * chunk, hi = min(m, lo + chunk);
                    float cs = 0.0f;
                    for (int i = lo; i < hi; i++) cs = __fadd_rn(cs, pr(i));
                    float *csum = (float *)hist;
                    csum[tid] = cs;
                    __syncthreads();
                    if (tid == 0) {
                        float cum = 0.0f;
                        int last = m - 1, t = 0;
                        for (; t < SM_THREADS; t++) {
                            const float nx = __fadd_rn(cum, csum[t]);
                            if (nx > a.topp) break;
                            cum = nx;
                        }
                        if (t < SM_THREADS)
                            for (int i = t * chunk; i < min(m, (t + 1) * chunk); i++) {
                                cum = __fadd_rn(cum, pr(i));
                                if (cum > a.topp) { last = i; break; }
                            }
                        const float r = __fmul_rn(coin, cum);
                        const int tl = last / chunk;
                        float cdf = 0.0f;
                        int u = 0, tok = v[last];
                        for (; u < tl; u++) {
                            const float nx = __fadd_rn(cdf, csum[u]);
                            if (r < nx) break;
                            cdf = nx;
                        }
                        const int l1 = u < tl ? min(m, (u + 1) * chunk) - 1 : last;
                        for (int i = u * chunk; i <= l1; i++) {
                            cdf = __fadd_rn(cdf, pr(i));
                            if (r < cdf) { tok = v[i]; break; }
                        }
                        s_tok = tok;
                    }
                }
            }
        } else {
            /* sample_mult (:63-70): the first token whose running sum passes the
             * coin; each thread sums a contiguous range, the ranges in order */
            const int chunk = (n + SM_THREADS - 1) / SM_THREADS, lo = tid * chunk, hi = min(n, lo + chunk);
            float cs = 0.0f;
            for (int i = lo; i < hi; i++) cs = __fadd_rn(cs, p[i]);
            float *csum = (float *)hist;
            csum[tid] = cs;
            __syncthreads();
            if (tid == 0) {
                float cdf = 0.0f;
                int tok = n - 1, t = 0;
                for (; t < SM_THREADS; t++) {
                    const float next = __fadd_rn(cdf, csum[t]);
                    if (coin < next) break;
                    cdf = next;
                }
                if (t < SM_THREADS) {
                    const int l0 = t * chunk, l1 = min(n, l0 + chunk);
                    for (int i = l0; i < l1; i++) {
                        cdf = __fadd_rn(cdf, p[i]);
                        if (coin < cdf) { tok = i; break; }
                    }
                }
                s_tok = tok;
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        const int tok = s_tok;
        *a.token_out = tok;
        /* ml_sampler_accept (:23-28) */
        if (a.repeat_last_n > 0) {
            SamplerDev u = *a.st;
            a.recent[u.recent_at] = tok;
            u.recent_at = (u.recent_at + 1) % a.repeat_last_n;
            if (u.n_recent < a.repeat_last_n) u.n_recent++;
            a.st->n_recent = u.n_recent;
            a.st->recent_at = u.recent_at;
        }
        if (a.ls) {
            /* the step kernel advanced the loop to the argmax: replace it */
            const int stp = a.ls->step - 1;
            if (a.out_tokens && stp >= 0) a.out_tokens[stp] = tok;
            a.ls->token = tok;
        }
    }
}

}  // namespace kc
