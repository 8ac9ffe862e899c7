"""The oracle's sampler against the reference's own (oracle/_ref scalar build,
model/sampler.c through ml_sampler_init / ml_sampler_accept / ml_sample):
the same tokens and the same final xorshift64* state, bit for bit, for every
option the sampler has (CPU only)."""
import numpy as np
import pytest

import oracle

OPTS = [
    dict(temperature=0.0),
    dict(temperature=0.0, repeat_penalty=1.3, repeat_last_n=8),
    dict(temperature=0.8, seed=7),
    dict(temperature=1.0, topk=40, seed=11),
    dict(temperature=0.7, topp=0.9, seed=13),
    dict(temperature=0.9, topk=50, topp=0.8, repeat_penalty=1.1, repeat_last_n=16, seed=17),
    dict(temperature=1.3, topk=1, seed=19),
    dict(temperature=0.5, topp=0.05, seed=23),
]


def _ref():
    try:
        return oracle.RefBuild("scalar")
    except (FileNotFoundError, RuntimeError, OSError):
        return None


@pytest.mark.parametrize("opts", OPTS, ids=[str(i) for i in range(len(OPTS))])
def test_oracle_sampler_matches_reference(opts):
    ref = _ref()
    if ref is None:
        pytest.skip("the reference's scalar build is not available")
    vocab, rows = 5000, 24
    rng = np.random.default_rng(len(str(opts)))
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    context = rng.integers(0, vocab, 12).tolist()
    want, want_rng = ref.sample_seq(oracle.sampler_opts(**opts), vocab, context, logits)
    s = oracle.OracleSampler(vocab, oracle.sampler_opts(**opts))
    for t in context:
        s.accept(t)
    got = []
    for r in range(rows):
        tok, _ = s.sample(logits[r])
        s.accept(tok)
        got.append(tok)
    assert got == want.tolist()
    assert s.rng == want_rng
