"""Tensor parallelism on the device (two GPUs, one process each): a model
sharded Megatron style across the ranks, the partial O and down outputs summed
on the device over NVLink after each projection, the vocabulary-split
classifier's best logit exchanged. Skipped with fewer than two GPUs.

Bars: the reference's logits (strict, 1e-3 of max|logit|) from every rank, the
same logits bit for bit on every rank, and the same greedy tokens."""
import os
import socket

import numpy as np
import pytest

from conftest import GOLDEN

import krafla_b200 as kb

pytestmark = pytest.mark.gpu

TOKENS = [1, 5, 9, 13, 17, 21, 25, 29, 33, 37, 41, 45, 49, 53, 57, 61]


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, path, kv, out, ffn=-1):
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    states, lg, toks, err = [], None, None, None
    try:
        kb.set_device(rank)
        kb.lib().kc_debug_ffn_split(ffn)
        m = kb.Model(path, upload=False).shard(rank, world)
        st = kb.State(m, kv_type=kv)
        states.append(st)
        st.tp_connect(kb.exchange_handles(st.tp_handle(), dist))
        lg = np.stack([st.forward(t, p) for p, t in enumerate(TOKENS)])
        st2 = kb.State(m, kv_type=kv)
        states.append(st2)
        st2.tp_connect(kb.exchange_handles(st2.tp_handle(), dist))
        st2.prefill(TOKENS[:4], 0)
        toks = st2.generate_greedy(TOKENS[4], 4, 12)
    except Exception as e:      # reported to the test, which fails with it
        err = repr(e) + " " + kb.what_detail()
    # every call above returns after its kernels end; no rank frees its exchange
    # buffer (or exits) before every rank is done, on the error path too
    try:
        dist.barrier()
    except Exception:
        pass
    for st in states:
        st.free()
    try:
        dist.barrier()
    except Exception:
        pass
    out.put((rank, lg, toks, err))
    dist.destroy_process_group()


def _run(path, kv, world=2, ffn=-1):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, path, kv, out, ffn)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r, lg, toks, err = out.get(timeout=300)
        assert err is None, (r, err)
        res[r] = (lg, toks)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name", ["rand_q4", "bias_q4", "mixf16_q4"])
def test_tp2_matches_reference_logits(name):
    path = os.path.join(GOLDEN, "models", f"{name}.mlb")
    res = _run(path, kb.F32)
    want = np.load(os.path.join(GOLDEN, f"{name}.logits.npy"))
    lg0, t0 = res[0]
    lg1, t1 = res[1]
    assert np.array_equal(lg0.view(np.uint32), lg1.view(np.uint32))     # every rank holds the full logits
    assert np.array_equal(t0, t1)                                         # and picks the same tokens
    err = np.abs(lg0.astype(np.float64) - want).max(axis=-1) / np.abs(want).max(axis=-1)
    assert err.max() <= 1e-3, err


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("kv", [kb.F16, kb.Q8_0])
def test_tp2_kv_cache_types(kv):
    path = os.path.join(GOLDEN, "models", "rand_q4.mlb")
    res = _run(path, kv)
    single = kb.State(kb.Model(path), kv_type=kv)
    ref = np.stack([single.forward(t, p) for p, t in enumerate(TOKENS)])
    lg0, t0 = res[0]
    assert np.array_equal(lg0.view(np.uint32), res[1][0].view(np.uint32))
    assert np.array_equal(t0, res[1][1])
    err = np.abs(lg0.astype(np.float64) - ref).max(axis=-1) / np.abs(ref).max(axis=-1)
    assert err.max() <= 1e-3, err


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_tp2_ffn_split_blocks():
    """Each rank's gate|up rows shared in 4-row units with split blocks (the
    mode cfg4's shards take) against whole blocks: equal logits bit for bit,
    on every rank."""
    path = os.path.join(GOLDEN, "models", "rand_q4.mlb")
    whole, split = _run(path, kb.F32, ffn=0), _run(path, kb.F32, ffn=1)
    for r in (0, 1):
        assert np.array_equal(whole[r][0].view(np.uint32), split[r][0].view(np.uint32))
        assert np.array_equal(whole[r][1], split[r][1])
