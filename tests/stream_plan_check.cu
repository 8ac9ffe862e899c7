/* Host-side check of the step kernel's weight-stream plan (make_plan in
 * kc_step.cuh), run by tests/test_stream_plan.py on the CPU: no kernel is
 * launched and no device is needed.
 *
 * Each line on stdin is one case:
 *   dim q_dim kv_dim hidden vocab t_q t_k t_v t_o t_up t_down t_cls d16 b_q b_k b_v G d_unit chunk
 * (types: 1 Q8_0, 2 Q4_0; chunk 0 = the default size). For every CTA j of G
 * the plan must give each matrix's rows to the CTAs exactly once and in CTA
 * order (the stream's layout and the tagged-word ownership both rely on it),
 * records of the matrix's type, whole records per bulk copy within the chunk
 * size (in multiples of a warp task's rows when more than one task fits),
 * gate|up rows in whole d_unit units, no more x rows per CTA than it can own,
 * and a ring slot (plan_max_chunk) that holds every copy. Prints "ok N" for N
 * cases checked, or the first failure. */
#include <cstdio>
#include <cstring>

#include "kc_step.cuh"

using namespace kc;

static int g_case = 0;

static bool fail(int j, const char *phase, const char *what) {
    std::printf("FAIL case %d cta %d phase %s: %s\n", g_case, j, phase, what);
    return false;
}

/* Segment s of CTA j: record size, copy size, and its place after `next`. */
static bool check_seg(const Seg &s, int j, const char *ph, int type, int d16, int cols, int bias, int pair, int chunk,
                      long long &next) {
    const int rec = rec_bytes(type, d16, cols, bias) * (pair ? 2 : 1);
    if (s.type != type || s.d16 != d16 || s.bias != bias) return fail(j, ph, "segment type, scale type or bias");
    if (s.rec != rec || rec % 16) return fail(j, ph, "record bytes");
    if (s.rows < 0) return fail(j, ph, "negative rows");
    if (s.row0 != next) return fail(j, ph, "rows not contiguous in CTA order (gap or overlap)");
    next += s.rows;
    if (s.rpc < 1) return fail(j, ph, "no record per copy");
    if (rec <= chunk && (long long)s.rpc * rec > chunk) return fail(j, ph, "copy larger than the chunk");
    if (rec > chunk && s.rpc != 1) return fail(j, ph, "records larger than the chunk must go one per copy");
    const int step = pair ? GROUP_ROWS / 2 : GROUP_ROWS;
    if (s.rpc >= step && s.rpc % step) return fail(j, ph, "copy not in whole warp tasks");
    return true;
}

static bool check_case(const StreamGeom &g, int G) {
    const int chunk = g.chunk > 0 ? g.chunk : CHUNK_BYTES;
    const int na = g.q_dim + 2 * g.kv_dim;
    const int lo[3] = { 0, g.q_dim, g.q_dim + g.kv_dim }, hi[3] = { g.q_dim, g.q_dim + g.kv_dim, na };
    const int ty[3] = { g.t_q, g.t_k, g.t_v }, dd[3] = { g.d16_q, g.d16_k, g.d16_v }, bb[3] = { g.b_q, g.b_k, g.b_v };
    long long nA = 0, nC = 0, nD = 0, nE = 0, nF = 0;
    for (int j = 0; j < G; j++) {
        PhasePlan P[NPHASE];
        std::memset(P, 0xff, sizeof(P));   /* every field must be written */
        make_plan(g, j, G, P);
        if (P[PH_A].nseg < 0 || P[PH_A].nseg > 3) return fail(j, "A", "segment count");
        for (int s = 0; s < P[PH_A].nseg; s++) {
            const Seg &S = P[PH_A].seg[s];
            int m = 0;
            while (m < 3 && !(S.row0 >= lo[m] && S.row0 < hi[m])) m++;
            if (m == 3 || S.row0 + S.rows > hi[m]) return fail(j, "A", "segment crosses a matrix or lies outside");
            if (!check_seg(S, j, "A", ty[m], dd[m], g.dim, bb[m], 0, chunk, nA)) return false;
        }
        const struct { int p; const char *name; int type, d16, cols, pair; long long *next; } one[4] = {
            { PH_C, "C", g.t_o, g.d16_o, g.q_dim, 0, &nC },
            { PH_D, "D", g.t_up, g.d16_up, g.dim, 1, &nD },
            { PH_E, "E", g.t_down, g.d16_down, g.hidden, 0, &nE },
            { PH_F, "F", g.t_cls, g.d16_cls, g.dim, 0, &nF },
        };
        for (const auto &o : one) {
            if (P[o.p].nseg != 1) return fail(j, o.name, "segment count");
            if (P[o.p].cols != o.cols) return fail(j, o.name, "columns");
            if (!check_seg(P[o.p].seg[0], j, o.name, o.type, o.d16, o.cols, 0, o.pair, chunk, *o.next)) return false;
        }
        const Seg &D = P[PH_D].seg[0];
        if (D.row0 % g.d_unit || D.rows % g.d_unit) return fail(j, "D", "gate|up rows not in whole units");
        if (P[PH_C].seg[0].rows != P[PH_E].seg[0].rows || P[PH_C].seg[0].row0 != P[PH_E].seg[0].row0)
            return fail(j, "C/E", "the two residual phases own different rows of x");
        if (P[PH_C].seg[0].rows > OWN_MAX) return fail(j, "C", "more rows of x than a CTA can own");
        int slot = 0;
        for (int p = 0; p < NPHASE; p++) {
            long long b = 0;
            for (int s = 0; s < P[p].nseg; s++) {
                const Seg &S = P[p].seg[s];
                b += (long long)S.rows * S.rec;
                const int first = (S.rows < S.rpc ? S.rows : S.rpc) * S.rec;
                slot = first > slot ? first : slot;
            }
            if (P[p].bytes != b) return fail(j, "any", "phase bytes");
        }
        if (plan_max_chunk(P) != slot) return fail(j, "any", "ring slot is not the largest copy");
    }
    if (nA != na) return fail(G, "A", "q|k|v rows not all covered");
    if (nC != g.dim || nE != g.dim) return fail(G, "C/E", "rows of x not all covered");
    if (nD != g.hidden) return fail(G, "D", "gate|up rows not all covered");
    if (nF != g.vocab) return fail(G, "F", "classifier rows not all covered");
    return true;
}

int main() {
    StreamGeom g;
    int d16, G, n = 0;
    while (true) {
        std::memset(&g, 0, sizeof(g));
        const int got = std::scanf("%d %d %d %d %d %d %d %d %d %d %d %d %d %d %d %d %d %d %d", &g.dim, &g.q_dim,
                                   &g.kv_dim, &g.hidden, &g.vocab, &g.t_q, &g.t_k, &g.t_v, &g.t_o, &g.t_up,
                                   &g.t_down, &g.t_cls, &d16, &g.b_q, &g.b_k, &g.b_v, &G, &g.d_unit, &g.chunk);
        if (got != 19) break;
        g.d16_q = g.d16_k = g.d16_v = g.d16_o = g.d16_up = g.d16_down = g.d16_cls = d16;
        g_case = n;
        if (!check_case(g, G)) return 1;
        n++;
    }
    std::printf("ok %d\n", n);
    return n > 0 ? 0 : 1;
}
