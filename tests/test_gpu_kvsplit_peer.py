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
