"""The device sampler (kc_sample, kc_generate_sampled) against the oracle's
restatement of model/sampler.c, pinned to the reference's own sampler by
tests/test_sampler_pin.py, on the same logits (a decode on BASELINE config 0).

Bar: the same xorshift64* state after every draw (exact), and the same token
at every step, except where the oracle's draw lies within 5e-6 (relative to
the mass it was drawn from) of a boundary of the token interval it falls in:
the device sums the probabilities as a tree and in blocks, and uses CUDA's
expf, so its cumulative sums differ from the reference's running sums by float
rounding (a few 1e-7 of the mass here; a synthetic model's flat distribution
gives token intervals of only ~3e-5, so the guard stays well below them)."""
import numpy as np
import pytest

from conftest import MODEL_CACHE

import krafla_b200 as kb
import oracle

pytestmark = pytest.mark.gpu

NEAR = 5e-6
OPTS = [
    dict(temperature=0.0, repeat_penalty=1.3, repeat_last_n=8),
    dict(temperature=0.8, seed=7),
    dict(temperature=1.0, topk=40, seed=11),
    dict(temperature=0.7, topp=0.9, seed=13),
    dict(temperature=0.9, topk=50, topp=0.8, repeat_penalty=1.1, repeat_last_n=16, seed=17),
    dict(temperature=0.6, topp=0.6, topk=200, seed=29),
    # top-p alone with a few hundred tokens above its cutoff: the selection path
    # (the flat cases above have tens of thousands: the full sort)
    dict(temperature=0.05, topp=0.9, seed=19),
]
# Not held: a nucleus of thousands of near-equal probabilities (a flat
# distribution at a high temperature with top-p near 1), where tokens whose
# probabilities differ by an ulp change places between the device's and the
# reference's order.


@pytest.fixture(scope="module")
def model():
    kb.device_check()
    return kb.Model(kb.ensure_model("cfg0", MODEL_CACHE))


@pytest.mark.parametrize("opts", OPTS, ids=[str(i) for i in range(len(OPTS))])
def test_device_sampler_matches_oracle(model, opts):
    vocab = model.config["vocab"]
    prompt = np.random.default_rng(5).integers(0, vocab, 8).tolist()
    st = kb.State(model)
    dev = kb.Sampler(st, **opts)
    orc = oracle.OracleSampler(vocab, oracle.sampler_opts(**opts))
    for t in prompt:
        dev.accept(t)
        orc.accept(t)
    st.prefill(prompt[:-1], 0)
    tok, pos, checked = prompt[-1], len(prompt) - 1, 0
    for _ in range(60):
        lg = st.forward(tok, pos)
        d = dev.sample()
        o, margin = orc.sample(lg)
        assert dev.rng == orc.rng
        if margin > NEAR:
            assert d == o, (pos, d, o, margin)
            checked += 1
        orc.accept(d)          # both streams continue from the device's choice
        tok, pos = d, pos + 1
    assert checked >= 15


def test_generate_sampled_equals_forward_and_sample(model):
    vocab = model.config["vocab"]
    opts = dict(temperature=0.8, topk=40, topp=0.95, repeat_penalty=1.1, repeat_last_n=16, seed=3)
    prompt = np.random.default_rng(6).integers(0, vocab, 8).tolist()
    a = kb.State(model)
    sa = kb.Sampler(a, **opts)
    for t in prompt:
        sa.accept(t)
    a.prefill(prompt[:-1], 0)
    toks = a.generate_sampled(sa, prompt[-1], len(prompt) - 1, 24)
    b = kb.State(model)
    sb = kb.Sampler(b, **opts)
    for t in prompt:
        sb.accept(t)
    b.prefill(prompt[:-1], 0)
    tok, pos, got = prompt[-1], len(prompt) - 1, []
    for _ in range(24):
        b.forward(tok, pos)
        tok, pos = sb.sample(), pos + 1
        got.append(tok)
    assert toks.tolist() == got
    assert sa.rng == sb.rng


def test_greedy_sampler_is_the_argmax(model):
    st = kb.State(model)
    s = kb.Sampler(st, temperature=0.0)
    lg = st.forward(1, 0)
    assert s.sample() == int(np.argmax(lg))


def test_sample_needs_logits(model):
    st = kb.State(model)
    s = kb.Sampler(st, temperature=0.5)
    with pytest.raises(kb.KraflaError):
        s.sample()
