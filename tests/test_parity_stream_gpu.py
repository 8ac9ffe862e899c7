"""Free-running greedy parity on the BASELINE shapes (north star: the greedy
stream of 128 tokens against the reference's), three ways from the same seeded
prompts:
  - the reference's scalar build (oracle/_ref, its sources compiled unchanged:
    the semantics the oracle restates bit for bit),
  - the reference's own best SIMD build on this host (oracle/_ref),
  - the B200 build through the C ABI (kc_forward per step, and the device loop
    kc_generate_greedy, which must choose the same tokens).
Each implementation runs its own stream: prefill of the prompt, then greedy
decode (app/ml_bench.c:125-131). A stream leaves the scalar stream at its first
token that differs.

What the reference's own builds show on these shapes (measured here, every
run): its SIMD build is about 1e-2 (config 0) to 6e-2 (config 2) of max|logit|
away from its scalar build from the first decode step on, because a 1-ulp
difference in a sum moves a quantized activation across a rounding boundary
now and then and each such flip moves the logits by about 1%; and random
weights give flat logits (top-2 margins of 1e-3 of max|logit| are common), so
its greedy stream leaves the scalar one within a few to a hundred steps. The
strict bar of 1e-3 therefore cannot hold for any build whose sums run in
another order, the reference's own included; it is held where it does hold
(the reference's golden test models, tests/test_model_gpu.py).

So the B200 stream is held to what the reference's own SIMD build achieves on
the same prompts:
  1. until its first divergence, every step within the largest distance of the
     SIMD build from the scalar one before the SIMD build's own divergences
     (times 1.25, at least the strict 1e-3);
  2. it diverges only where the scalar logits leave the choice within the
     noise: the scalar's top-2 margin at that step is at most twice the B200
     step's logit distance (plus 1e-4 of max|logit|);
  3. over all prompts' steps before their first divergence, its median logit
     distance from the scalar build is at most 1.25 times the SIMD build's;
  4. over the prompts, it stays on the scalar stream at least half as many
     steps as the SIMD build does. The step where a stream leaves is the
     first near-tie that its rounding noise happens to flip, so the sum over a
     few prompts is heavy-tailed: one run measured B200 59 / SIMD 82 steps on
     config 1 (prompt 5: 4 against 25, prompt 1: 24 against 11) with the two
     builds' per-step distances at the same level. Criteria 1-3 compare the
     noise itself; 4 is a floor.
The per-prompt table is printed (pytest -s).
"""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import MODEL_CACHE

import krafla_b200 as kb
import oracle

pytestmark = pytest.mark.gpu

STEPS = 128
CASES = [("cfg0", 16, 8), ("cfg1", 32, 6), ("cfg2", 16, 6)]   # config, prompt length, prompts


@pytest.fixture(scope="module", autouse=True)
def _dev(built):
    kb.device_check()


def _rel(a, b):
    return float(np.abs(a.astype(np.float64) - b).max() / np.abs(b).max())


def _ref_stream(r, path, prompt, vocab):
    h = r.open(path, os.cpu_count() or 1, 0, True)
    p = np.array(prompt[:-1], np.int32)
    assert r.L.ref_prefill(h, p.ctypes.data_as(C.c_void_p), len(p), 0, None) == 0
    lg = np.zeros((STEPS, vocab), np.float32)
    toks, t = [], prompt[-1]
    for i in range(STEPS):
        assert r.L.ref_forward(h, int(t), len(prompt) - 1 + i, lg[i].ctypes.data_as(C.c_void_p)) == 0
        t = int(np.argmax(lg[i]))
        toks.append(t)
    r.L.ref_close(h)
    return np.array(toks), lg


def _gpu_stream(st, prompt):
    st.prefill(prompt[:-1], 0)
    lg, toks, t = [], [], prompt[-1]
    for i in range(STEPS):
        lg.append(st.forward(int(t), len(prompt) - 1 + i))
        t = int(np.argmax(lg[-1]))
        toks.append(t)
    st.prefill(prompt[:-1], 0)
    dev = st.generate_greedy(prompt[-1], len(prompt) - 1, STEPS)
    return np.array(toks), np.stack(lg), dev


def _first_div(a, b):
    d = np.nonzero(a != b)[0]
    return int(d[0]) if len(d) else len(a)


@pytest.mark.parametrize("name,plen,nprompt", CASES)
def test_free_running_greedy_stream(name, plen, nprompt):
    try:
        scalar, simd = oracle.RefBuild("scalar"), oracle.RefBuild()
    except (FileNotFoundError, RuntimeError, OSError) as e:
        pytest.skip(f"the reference's builds are not available here: {e}")
    if simd.isa == "scalar":
        pytest.skip("no SIMD build of the reference runs on this host")
    path = kb.ensure_model(name, MODEL_CACHE)
    vocab = kb.read_header(path)["vocab"]
    m = kb.Model(path)
    st = kb.State(m)
    rows, eg_all, es_all = [], [], []
    for k in range(nprompt):
        prompt = np.random.default_rng(100 + k).integers(0, vocab, plen).tolist()
        st_tok, st_lg = _ref_stream(scalar, path, prompt, vocab)
        sd_tok, sd_lg = _ref_stream(simd, path, prompt, vocab)
        g_tok, g_lg, dev = _gpu_stream(st, prompt)
        assert np.array_equal(dev, g_tok), "the device loop chose other tokens than the host argmax"
        dg, ds = _first_div(g_tok, st_tok), _first_div(sd_tok, st_tok)
        eg = [_rel(g_lg[i], st_lg[i]) for i in range(dg)]
        es = [_rel(sd_lg[i], st_lg[i]) for i in range(ds)]
        eg_all += eg
        es_all += es
        row = dict(prompt=k, d_gpu=dg, d_simd=ds, gpu_err=max(eg, default=0.0), simd_err=max(es, default=0.0),
                   gpu_strict_fail=sum(e > 1e-3 for e in eg), simd_strict_fail=sum(e > 1e-3 for e in es))
        if dg < STEPS:   # the step where the B200 stream leaves the scalar one
            srt = np.sort(st_lg[dg])
            row["margin_rel"] = float((srt[-1] - st_lg[dg][g_tok[dg]]) / np.abs(st_lg[dg]).max())
            row["err_at_div"] = _rel(g_lg[dg], st_lg[dg])
        rows.append(row)
    st.free()
    m.free()
    bar = max(1e-3, 1.25 * max(r["simd_err"] for r in rows))
    print(f"\n{name}: {simd.isa} vs scalar and B200 vs scalar, {nprompt} prompts of {plen} + {STEPS} greedy steps; "
          f"step bar {bar:.2e}")
    for r in rows:
        print("  " + ", ".join(f"{k} {v:.3g}" if isinstance(v, float) else f"{k} {v}" for k, v in r.items()))
    sg, ss = sum(r["d_gpu"] for r in rows), sum(r["d_simd"] for r in rows)
    mg = float(np.median(eg_all)) if eg_all else 0.0
    ms = float(np.median(es_all)) if es_all else 0.0
    print(f"  steps on the scalar stream: B200 {sg}, {simd.isa} {ss}; median step distance B200 {mg:.3g}, "
          f"{simd.isa} {ms:.3g}")
    for r in rows:
        assert r["gpu_err"] <= bar, r
        if "margin_rel" in r:
            assert r["margin_rel"] <= 2 * r["err_at_div"] + 1e-4, r
    assert mg <= max(1e-3, 1.25 * ms), (mg, ms)
    assert sg >= 0.5 * ss, (sg, ss)


def _kl(ref, got):
    """KL(softmax(ref) || softmax(got)) as the reference's tests/compare_logits.py:23-30 computes it."""
    def sm(x):
        e = np.exp(x - x.max())
        return e / e.sum()
    pa, pb = sm(got.astype(np.float64)), sm(ref.astype(np.float64))
    return float((pb * (np.log(pb + 1e-30) - np.log(pa + 1e-30))).sum())


def _ref_logits_at(r, path, toks, positions, vocab):
    """Logits of the reference build r at `positions` of the prompt toks: ml_prefill
    up to each position (no logits), then ml_forward there (the reference's batched
    prefill equals its token-by-token decode bit for bit)."""
    h = r.open(path, os.cpu_count() or 1, 0, True)
    out, done = {}, 0
    for p in sorted(positions):
        if p > done:
            seg = np.ascontiguousarray(toks[done:p], np.int32)
            assert r.L.ref_prefill(h, seg.ctypes.data_as(C.c_void_p), len(seg), done, None) == 0
        lg = np.zeros(vocab, np.float32)
        assert r.L.ref_forward(h, int(toks[p]), p, lg.ctypes.data_as(C.c_void_p)) == 0
        out[p], done = lg, p + 1
    r.L.ref_close(h)
    return out


def test_cfg3_prefill_long_prompt():
    """a 2048-token prompt through the batched tensor-core
    prefill (cfg2 weights) in two calls, the first of 1100 tokens crossing the
    default 1024-token chunk boundary, the second ending at 2048. Logits at
    positions around 512, the chunk boundary, the call boundary and the end
    against the reference's scalar build; the bar is the distance of the
    reference's own SIMD build from its scalar build at the same positions (x
    1.25, at least the reference's 5e-2 / 1e-3 for long runs)."""
    try:
        scalar, simd = oracle.RefBuild("scalar"), oracle.RefBuild()
    except (FileNotFoundError, RuntimeError, OSError) as e:
        pytest.skip(f"the reference's builds are not available here: {e}")
    path = kb.ensure_model("cfg2", MODEL_CACHE)
    vocab = kb.read_header(path)["vocab"]
    toks = np.random.default_rng(7).integers(0, vocab, 2048).astype(np.int32)
    check = [0, 511, 1022, 1023, 1024, 1025, 1099, 1100, 1500, 2047]
    m = kb.Model(path)
    st = kb.State(m)
    got = {}
    for a, b in ((0, 1100), (1100, 2048)):
        lg = st.prefill(toks[a:b], a, logits=True)
        got.update({p: lg[p - a].copy() for p in check if a <= p < b})
        del lg
    st.free()
    m.free()
    want = _ref_logits_at(scalar, path, toks, check, vocab)
    spread = None
    if simd.isa != "scalar":
        other = _ref_logits_at(simd, path, toks, check, vocab)
        spread = (max(_rel(other[p], want[p]) for p in check), max(_kl(want[p], other[p]) for p in check))
    bound, kl_bound = (5e-2, 1e-3) if spread is None else (max(5e-2, 1.25 * spread[0]), max(1e-3, 1.25 * spread[1]))
    print(f"\ncfg3 prefill: {simd.isa} vs scalar spread {spread}; bar {bound:.3g} / KL {kl_bound:.3g}")
    for p in check:
        e, k = _rel(got[p], want[p]), _kl(want[p], got[p])
        print(f"  pos {p}: rel err {e:.3e}, KL {k:.2e}, argmax {int(got[p].argmax())} / {int(want[p].argmax())}")
        assert e <= bound and k <= kl_bound, (p, e, k)
        w = want[p]
        assert got[p].argmax() == w.argmax() or w.max() - w[got[p].argmax()] <= 2 * e * np.abs(w).max() + 1e-4, p
