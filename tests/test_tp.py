"""Tensor parallelism, host side (CPU): the shard plan of kc_model_shard and the
handle exchange over torch.distributed (gloo, two ranks). The device side is
tests/test_tp_gpu.py."""
import os
import socket

import numpy as np
import pytest

from conftest import GOLDEN

import krafla_b200 as kb

RAND_Q4 = os.path.join(GOLDEN, "models", "rand_q4.mlb")


def test_shard_plan_splits_heads_rows_and_vocab():
    full = kb.Model(RAND_Q4, upload=False).config
    infos = [kb.Model(RAND_Q4, upload=False).shard(r, 2).shard_info for r in range(2)]
    for r, s in enumerate(infos):
        assert (s["rank"], s["world"]) == (r, 2)
        assert s["n_heads"] * 2 == full["n_heads"] and s["n_kv_heads"] * 2 == full["n_kv_heads"]
        assert s["q_dim"] * 2 == full["q_dim"] and s["kv_dim"] * 2 == full["kv_dim"]
        assert s["hidden_dim"] * 2 == full["hidden_dim"]
    # the classifier rows of the ranks tile the vocabulary in rank order
    assert infos[0]["cls_row0"] == 0
    assert infos[0]["cls_row0"] + infos[0]["cls_rows"] == infos[1]["cls_row0"]
    assert infos[1]["cls_row0"] + infos[1]["cls_rows"] == full["vocab"]


def test_sharded_model_keeps_the_file_config():
    m = kb.Model(RAND_Q4, upload=False)
    before = m.config
    m.shard(1, 2)
    assert m.config == before


def test_shard_plan_uneven_vocab():
    # vocab split by floor(V * r / world): contiguous, covering, sizes within one
    vocab = kb.Model(RAND_Q4, upload=False).config["vocab"]
    rows = []
    for r in range(2):
        s = kb.Model(RAND_Q4, upload=False).shard(r, 2).shard_info
        rows.append((s["cls_row0"], s["cls_rows"]))
    assert sum(n for _, n in rows) == vocab and abs(rows[0][1] - rows[1][1]) <= 1


@pytest.mark.parametrize("rank,world", [(0, 4), (0, 3), (2, 2), (-1, 2), (0, 9), (0, 0)])
def test_shard_refuses_what_does_not_divide(rank, world):
    with pytest.raises(kb.KraflaError) as e:
        kb.Model(RAND_Q4, upload=False).shard(rank, world)
    assert e.value.status == kb.E_SHAPE


def test_shard_once():
    m = kb.Model(RAND_Q4, upload=False).shard(0, 2)
    with pytest.raises(kb.KraflaError):
        m.shard(0, 2)


def test_world_one_is_the_whole_model():
    s = kb.Model(RAND_Q4, upload=False).shard(0, 1).shard_info
    full = kb.Model(RAND_Q4, upload=False).config
    assert s["world"] == 1 and s["n_heads"] == full["n_heads"] and s["cls_rows"] == full["vocab"]


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _exchange_worker(rank, world, port, out):
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        handle = bytes([rank + 1]) * kb.TP_HANDLE_BYTES
        got = kb.exchange_handles(handle, dist)
        out.put((rank, [h[0] for h in got], [len(h) for h in got]))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_gloo_two_ranks():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_exchange_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(out.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, first_bytes, lens in res:
        assert first_bytes == [1, 2] and lens == [kb.TP_HANDLE_BYTES] * 2
