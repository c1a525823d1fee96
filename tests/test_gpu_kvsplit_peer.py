"""GPU parity of the fused KV-split decode (apex_attn_decode_kvsplit_bf16): ranks holding parts of
the key range exchange their partials through NVLink peer memory inside the decode kernel and
merge them there.  The result must match the one-GPU fused decode over the whole range."""
from __future__ import annotations

import ctypes
import dataclasses
import os
import socket

import pytest
import torch

from apex_b200 import _native, ops
from apex_b200.configs import CONFIGS
from helpers import assert_close, bf16_dev_to_f32

from test_gpu_decode import build_decode, run_decode

pytestmark = pytest.mark.gpu

LENS = [9000, 6000]
BOUNDS = [0, 4608, 9000]  # two ranks; split starts on the decode stage (32 positions)


def _cfg():
    return dataclasses.replace(CONFIGS["c1_decode"], batch=2, seed=29, rope_theta=1e6)


def _fused(shape, t, lo, hi, exchange):
    local = ops.KvCache(t["cache"].k[:, :, lo:hi, :].contiguous(), t["cache"].v[:, :, lo:hi, :].contiguous())
    ws = ops.DecodeWorkspace(shape, 2, 9000)
    out = torch.empty(2, shape.q_heads, shape.head_dim, dtype=torch.bfloat16, device="cuda")
    outs = []
    for _ in range(2):  # two steps: both gather slots and the step counters
        ops.attention_decode_kvsplit(shape, t["q_raw"], t["k_new"], t["v_new"], t["qw"], t["kw"], local,
                                     t["lens"], 9000, lo, hi, exchange, out, ws)
        ops.device_status()
        outs.append(bf16_dev_to_f32(out).copy())
    return outs


def test_kvsplit_fused_one_rank_matches_decode():
    """world = 1: the kernel publishes to and waits on its own buffers."""
    cfg = _cfg()
    shape, t = build_decode(cfg, [0, 1], LENS, cap=9000)
    full, _ = run_decode(shape, t)
    lib = _native.load()
    sizes = [ctypes.c_size_t() for _ in range(3)]
    _native.check(lib.apex_attn_peer_exchange_bytes(shape.c(), 2, 1, *map(ctypes.byref, sizes)))
    bufs = []
    for n in sizes:
        p = ctypes.c_void_p()
        _native.check(lib.apex_device_alloc(n.value, ctypes.byref(p)))
        bufs.append(p.value)
    try:
        x = _native.PeerExchange()
        x.rank, x.world, x.gather[0], x.flags[0], x.seq = 0, 1, bufs[0], bufs[1], bufs[2]
        for i, got in enumerate(_fused(shape, t, 0, 9000, x)):
            assert_close(got, full, f"fused one-rank step {i} vs decode", max_abs=4e-3, mean_abs=2e-4)
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            lib.apex_device_free(p)


def _rank_main(rank, world, port):
    import torch.distributed as dist
    from apex_b200 import dist as adist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        cfg = _cfg()
        shape, t = build_decode(cfg, [0, 1], LENS, cap=9000)
        full, _ = run_decode(shape, t)
        bufs = adist.PeerExchangeBuffers(shape, 2)
        try:
            outs = _fused(shape, t, BOUNDS[rank], BOUNDS[rank + 1], bufs.exchange)
        finally:
            bufs.close()
        for i, got in enumerate(outs):
            assert_close(got, full, f"rank {rank} fused step {i} vs one-GPU decode", max_abs=4e-3, mean_abs=2e-4)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_kvsplit_fused_two_gpus_matches_decode():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_rank_main, args=(2, port), nprocs=2, join=True)


def test_kvsplit_wait_gives_up_reports_timeout_and_poisons():
    """world = 2 on one GPU, where "rank 1" is local memory that nothing ever publishes to: the
    bounded wait for its flag (2 ms here) runs out, the status word reports a timeout, the output is
    left as it was, and the pair's counters are poisoned -- a second step publishes and merges
    nothing and reports the timeout again without waiting."""
    cfg = _cfg()
    shape, t = build_decode(cfg, [0, 1], LENS, cap=9000)
    lib = _native.load()
    sizes = [ctypes.c_size_t() for _ in range(3)]
    _native.check(lib.apex_attn_peer_exchange_bytes(shape.c(), 2, 2, *map(ctypes.byref, sizes)))
    g0, f0, s0 = (torch.zeros(max(n.value // 4, 4), dtype=torch.int32, device="cuda") for n in sizes)
    g1, f1 = (torch.zeros(max(n.value // 4, 4), dtype=torch.int32, device="cuda") for n in sizes[:2])
    x = _native.PeerExchange()
    x.rank, x.world = 0, 2
    x.gather[0], x.flags[0], x.gather[1], x.flags[1] = g0.data_ptr(), f0.data_ptr(), g1.data_ptr(), f1.data_ptr()
    x.seq, x.wait_ns = s0.data_ptr(), 2_000_000
    lo, hi = BOUNDS[0], BOUNDS[1]
    local = ops.KvCache(t["cache"].k[:, :, lo:hi, :].contiguous(), t["cache"].v[:, :, lo:hi, :].contiguous())
    ws = ops.DecodeWorkspace(shape, 2, 9000)
    sentinel = torch.full((2, shape.q_heads, shape.head_dim), 0x7F7F, dtype=torch.int16, device="cuda")
    out = sentinel.clone().view(torch.bfloat16)
    poison = -0x80000000  # bit 31 of the uint32 counters, as int32

    ops.attention_decode_kvsplit(shape, t["q_raw"], t["k_new"], t["v_new"], t["qw"], t["kw"], local, t["lens"],
                                 9000, lo, hi, x, out, ws)
    with pytest.raises(_native.ApexError) as e:
        ops.device_status()
    assert e.value.code == _native.APEX_ERR_DEVICE_TIMEOUT
    assert torch.equal(out.view(torch.int16), sentinel), "a step that timed out wrote its output"
    bhkv = 2 * shape.kv_heads
    assert bool(((s0[:bhkv] & poison) != 0).all()), "step counters not poisoned"
    assert bool(((f1[:bhkv] & poison) != 0).all()), "the peer was not told"

    g1_before, g0_before = g1.clone(), g0.clone()
    ops.attention_decode_kvsplit(shape, t["q_raw"], t["k_new"], t["v_new"], t["qw"], t["kw"], local, t["lens"],
                                 9000, lo, hi, x, out, ws)
    with pytest.raises(_native.ApexError) as e:
        ops.device_status()
    assert e.value.code == _native.APEX_ERR_DEVICE_TIMEOUT
    assert torch.equal(g1, g1_before) and torch.equal(g0, g0_before), "a poisoned pair published again"
    assert torch.equal(out.view(torch.int16), sentinel)
    ops.device_status()  # the status word was cleared by the read above


def _gather_rank_main(rank, world, port, result_path):
    """One "rank" of the collective form on a shared GPU: its partial from the decode kernel, the
    real all-gather of the partial records (gloo over host copies stands in for NCCL, which needs
    one GPU per rank), and the merge kernel on the gathered records."""
    from datetime import timedelta

    import numpy as np
    import torch.distributed as dist
    from apex_b200 import dist as adist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        torch.cuda.set_device(0)
        cfg = _cfg()
        shape, t = build_decode(cfg, [0, 1], LENS, cap=9000)
        lo, hi = adist.kv_ranges(9000, world)[rank]
        local = ops.KvCache(t["cache"].k[:, :, lo:hi, :].contiguous(), t["cache"].v[:, :, lo:hi, :].contiguous())
        ws = ops.DecodeWorkspace(shape, 2, 9000)
        part_dev = torch.empty(2, shape.q_heads, shape.head_dim + 2, dtype=torch.float32, device="cuda")
        splitter = adist.KVSplitDecode(2, shape.q_heads, shape.head_dim, "cpu")

        def partial(p):
            ops.attention_decode_partial(shape, t["q_raw"], t["k_new"], t["v_new"], t["qw"], t["kw"], local,
                                         t["lens"], 9000, lo, hi, part_dev, ws)
            p.copy_(part_dev.cpu())

        out = torch.empty(2 * shape.q_heads, shape.head_dim, dtype=torch.bfloat16, device="cuda")

        def merge(parts, o):
            ops.merge_partials(parts.cuda(), o)

        splitter.step(partial, merge, out)
        ops.device_status()
        if rank == 0:
            np.save(result_path, bf16_dev_to_f32(out).reshape(2, shape.q_heads, shape.head_dim))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [3])
def test_kvsplit_collective_form_all_gather_layout_merges_to_full(tmp_path, world):
    import numpy as np
    import torch.multiprocessing as mp
    cfg = _cfg()
    shape, t = build_decode(cfg, [0, 1], LENS, cap=9000)
    full, _ = run_decode(shape, t)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    res = tmp_path / "merged.npy"
    mp.spawn(_gather_rank_main, args=(world, port, str(res)), nprocs=world, join=True)
    assert_close(np.load(res), full, f"{world} partials gathered and merged vs one-GPU decode",
                 max_abs=4e-3, mean_abs=2e-4)
