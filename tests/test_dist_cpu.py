"""CPU tests of the multi-GPU host logic (apex_b200/dist.py) with world-size-2 `gloo`
process groups: shard plans, the KV-split all-gather + LSE merge (the oracle stands in for the
GPU partial kernel), and failure detection on the host (a rank that dies before the
collective makes the surviving rank's collective fail instead of hanging)."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from apex_b200 import dist as adist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_sequences_covers_and_balances():
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 8193, 64).tolist()
    for world in (1, 2, 4, 8):
        shards = adist.shard_sequences(lens, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(64))
        loads = [sum(lens[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(lens)


def test_kv_ranges_cover_and_align():
    for L in (1, 31, 1024, 131072, 131071):
        for world in (1, 2, 4, 8):
            rs = adist.kv_ranges(L, world)
            assert rs[0][0] == 0 and rs[-1][1] == L
            for (b0, e0), (b1, e1) in zip(rs, rs[1:]):
                assert e0 == b1
            for b, e in rs:
                assert b <= e and (b % adist.SPLIT_ALIGN == 0 or b == L)


def _kv_split_worker(rank, world, port, q, K, V, D, L, scale, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    lo, hi = adist.kv_ranges(L, world)[rank]
    splitter = adist.KVSplitDecode(batch=1, q_heads=1, head_dim=D, device="cpu")

    def partial(p):  # the GPU path runs apex_attn_decode_partial_bf16 on the local slice here
        if hi > lo:
            p.view(-1).copy_(torch.from_numpy(oracle.partial_row(q, K, V, D, lo, hi, scale)))
        else:
            p.zero_()

    def merge(parts, out):
        out.copy_(torch.from_numpy(oracle.merge_partials(parts.numpy(), D)).view_as(out))

    out = torch.empty(1, D)
    splitter.step(partial, merge, out)
    if rank == 0:
        np.save(result_path, out.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_kv_split_all_gather_merge_equals_full_attention(tmp_path, world):
    D, L, scale = 64, 1000, 0.125
    rng = np.random.default_rng(3)
    q = rng.standard_normal(D).astype(np.float32)
    K = rng.standard_normal(L * D).astype(np.float32)
    V = rng.standard_normal(L * D).astype(np.float32)
    full = np.zeros(D, np.float32)
    oracle.lib().orc_attention_row(q, K, V, full, D, 0, L - 1, scale)
    res = tmp_path / "out.npy"
    mp.spawn(_kv_split_worker, args=(world, _free_port(), q, K, V, D, L, scale, str(res)), nprocs=world)
    np.testing.assert_allclose(np.load(res)[0], full, rtol=1e-5, atol=1e-6)


def _dying_rank_worker(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the all-gather, with nothing in flight
    splitter = adist.KVSplitDecode(batch=1, q_heads=1, head_dim=8, device="cpu")
    try:
        splitter.step(lambda p: p.zero_(), lambda parts, out: None, torch.empty(1, 8))
        outcome = "completed"
    except Exception as e:  # the surviving rank learns of the failure on the host
        outcome = "error:" + type(e).__name__
    with open(result_path, "w") as f:
        f.write(outcome)
    os._exit(0)


def test_rank_failure_surfaces_as_error_not_hang(tmp_path):
    res = tmp_path / "outcome.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dying_rank_worker, args=(r, 2, port, str(res))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung"
    assert res.read_text().startswith("error:")
