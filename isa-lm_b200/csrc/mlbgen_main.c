/* mlbgen: writes one synthetic .mlb with the writer of mlb_writer.c, as a
 * command of its own, so that a process which only reads models (the CPU
 * reference arm of bench.py) never loads a library of this repository.
 *
 *   mlbgen OUT.mlb key=value ...
 *
 * Keys are the fields of kw_config (mlb_writer.h); fields not given are 0,
 * except norm_eps 1e-5, rope_theta 10000, sigma and bias_sigma 0.02,
 * scale_f16 1 and nthreads = the online CPUs. Exit status 0, 2 for a bad
 * argument, else the writer's errno value. */
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "mlb_writer.h"

typedef struct {
    const char *key;
    char kind;   /* i int, f float, d double, u uint64 */
    size_t off;
} arg_field;

#define F(name, kind) { #name, kind, offsetof(kw_config, name) }
static const arg_field FIELDS[] = {
    F(dim, 'i'), F(n_layers, 'i'), F(n_heads, 'i'), F(n_kv_heads, 'i'), F(hidden_dim, 'i'), F(vocab, 'i'),
    F(max_seq, 'i'), F(rope_theta, 'f'), F(norm_eps, 'f'), F(wtype, 'i'), F(shared, 'i'), F(rope_type, 'i'),
    F(rope_factor, 'f'), F(rope_lo, 'f'), F(rope_hi, 'f'), F(rope_orig, 'i'), F(q8_mask, 'i'), F(qkv_bias, 'i'),
    F(head_dim, 'i'), F(scale_f16, 'i'), F(sigma, 'd'), F(bias_sigma, 'd'), F(seed, 'u'), F(nthreads, 'i'),
};
#undef F

static int set_field(kw_config *c, const char *arg) {
    const char *eq = strchr(arg, '=');
    if (!eq) return -1;
    const size_t klen = (size_t)(eq - arg);
    for (size_t i = 0; i < sizeof FIELDS / sizeof FIELDS[0]; i++) {
        const arg_field *f = &FIELDS[i];
        if (strlen(f->key) != klen || strncmp(f->key, arg, klen)) continue;
        char *end = NULL;
        char *dst = (char *)c + f->off;
        errno = 0;
        switch (f->kind) {
        case 'i': *(int *)dst = (int)strtol(eq + 1, &end, 10); break;
        case 'f': *(float *)dst = strtof(eq + 1, &end); break;
        case 'd': *(double *)dst = strtod(eq + 1, &end); break;
        default: *(uint64_t *)dst = strtoull(eq + 1, &end, 10); break;
        }
        return (errno || !end || *end || end == eq + 1) ? -1 : 0;
    }
    return -1;
}

int main(int argc, char **argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: mlbgen OUT.mlb key=value ...\n");
        return 2;
    }
    kw_config c;
    memset(&c, 0, sizeof c);
    c.rope_theta = 10000.0f;
    c.norm_eps = 1e-5f;
    c.sigma = 0.02;
    c.bias_sigma = 0.02;
    c.scale_f16 = 1;
    const long ncpu = sysconf(_SC_NPROCESSORS_ONLN);
    c.nthreads = ncpu > 0 ? (int)ncpu : 1;
    for (int i = 2; i < argc; i++) {
        if (set_field(&c, argv[i])) {
            fprintf(stderr, "mlbgen: bad argument '%s'\n", argv[i]);
            return 2;
        }
    }
    const int rc = kw_write_model(argv[1], &c);
    if (rc) fprintf(stderr, "mlbgen: writing %s failed: %s\n", argv[1], strerror(rc));
    return rc;
}
