/* Synthetic .mlb model writer (mlb_writer.c): the configuration of one
 * model and the entry points of libkrafla_mlbgen.so and of the mlbgen
 * command. */
#ifndef MLB_WRITER_H
#define MLB_WRITER_H
#include <stddef.h>
#include <stdint.h>

typedef struct {
    int dim, n_layers, n_heads, n_kv_heads, hidden_dim, vocab, max_seq;
    float rope_theta, norm_eps;
    int wtype;           /* 1 = Q8_0, 2 = Q4_0 */
    int shared;          /* tied embedding / classifier */
    int rope_type;       /* 0 none, 1 llama3, 2 linear, 3 yarn */
    float rope_factor, rope_lo, rope_hi;
    int rope_orig;
    int q8_mask;         /* Q4 models: classes kept in Q8 (tools/mlb.py:54) */
    int qkv_bias;
    int head_dim;        /* 0: dim / n_heads */
    int scale_f16;
    double sigma;        /* weight standard deviation */
    double bias_sigma;
    uint64_t seed;
    int nthreads;
} kw_config;

/* Writes the model; 0 or an errno value (the file is removed on failure). */
int kw_write_model(const char *path, const kw_config *c);
/* nblocks blocks of 32 floats of x quantized as `type` (1 Q8_0, 2 Q4_0) with
 * f32 or (f16 != 0) f16 scales; 0, or -1 when an f16 scale overflows. */
int kw_quantize(int type, int f16, const float *x, long nblocks, void *q, void *d);
/* n values of tensor `tid` from element i0 on: seeded N(0, sigma). */
void kw_normal(uint64_t seed, uint64_t tid, uint64_t i0, long n, double sigma, float *out);
size_t kw_config_size(void);

#endif
