"""Multi-GPU host logic of the attention path: one process per GPU over torch.distributed.

Only these shardings exist, where the work splits naturally:

* batch sharding (ragged decode, batched decode, chunked prefill when the batch divides over the
  ranks): whole sequences go to ranks, balanced by key count (longest first onto the least-loaded
  rank); no collective on the data path.  A chunked prefill whose batch does not divide (4
  sequences over 8 GPUs) shards kv heads with their q heads instead, also with no collective.
* KV-sequence split (one long decode): rank r holds key positions [begin_r, end_r) of every
  sequence.  Fused form (PeerExchangeBuffers + apex_attn_decode_kvsplit_bf16): the decode
  kernel writes each rank's partial (o, m, l) straight into every rank's gather buffer over
  NVLink (CUDA IPC mappings), each value as an 8-byte word carrying the step number, and merges
  once every rank's words carry the step -- one launch per step.  Collective form (KVSplitDecode, the baseline): the partial from
  apex_attn_decode_partial_bf16, ONE NCCL all-gather (16.5 KB per sequence per rank at Hq=16,
  D=256) and apex_attn_merge_partials.

The reference is single-device; these are new (docs/B6_3_attention.md has no parallelism).
"""
from __future__ import annotations

import ctypes
from typing import Callable, List, Sequence, Tuple

import torch

SPLIT_ALIGN = 32  # KV ranges start on multiples of the decode kernel's stage (32 positions)


def shard_sequences(lens: Sequence[int], world: int) -> List[List[int]]:
    """Greedy longest-first assignment of sequence indices to `world` ranks by key count.
    Every index appears exactly once; the result is deterministic."""
    loads = [0] * world
    shards: List[List[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lens)), key=lambda j: (-int(lens[j]), j)):
        r = min(range(world), key=lambda k: (loads[k], k))
        shards[r].append(i)
        loads[r] += int(lens[i])
    return [sorted(s) for s in shards]


def kv_ranges(total_len: int, world: int, align: int = SPLIT_ALIGN) -> List[Tuple[int, int]]:
    """Contiguous [begin, end) key ranges covering 0..total_len, one per rank, starts aligned."""
    per = -(-total_len // world)
    per = -(-per // align) * align
    out = []
    for r in range(world):
        b = min(total_len, r * per)
        e = min(total_len, (r + 1) * per)
        out.append((b, e))
    return out


class KVSplitDecode:
    """One decode step of sequences whose keys are split over the ranks of `group`.

    `partial_fn(partial_out)` computes this rank's partial [B, Hq, D+2] (f32) in place -- on
    the GPU it is apex_attn_decode_partial_bf16 on the local cache slice; `merge_fn(parts,
    out)` merges [world, B*Hq, D+2] partials.  The all-gather is the only collective."""

    def __init__(self, batch: int, q_heads: int, head_dim: int, device, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rows = batch * q_heads
        self.rec = head_dim + 2
        self.partial = torch.empty(batch, q_heads, self.rec, dtype=torch.float32, device=device)
        self.gathered = torch.empty(self.world, self.rows, self.rec, dtype=torch.float32, device=device)

    def step(self, partial_fn: Callable[[torch.Tensor], None],
             merge_fn: Callable[[torch.Tensor, torch.Tensor], None], out: torch.Tensor) -> torch.Tensor:
        partial_fn(self.partial)
        self.dist.all_gather_into_tensor(self.gathered.view(-1), self.partial.view(-1), group=self.group)
        merge_fn(self.gathered, out)
        return out


class PeerExchangeBuffers:
    """Exchange buffers of the fused KV-split decode (apex_attn_decode_kvsplit_bf16) for up to
    `batch` sequences over the ranks of `group` (one process per GPU, all on one NVLink domain).

    Each rank allocates its gather buffer, flag array and step counters with apex_device_alloc
    (zeroed), shares the first two by CUDA IPC handle through one all_gather_object, and maps the
    other ranks' buffers.  `exchange` is the apex_peer_exchange to pass to every decode step;
    every rank must run the same number of steps.  close() unmaps and frees (collective)."""

    def __init__(self, shape, batch: int, group=None):
        import torch.distributed as dist
        from . import _native
        self._native, self.dist, self.group = _native, dist, group
        lib = _native.load()
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > _native.MAX_PEERS:
            raise ValueError(f"PeerExchangeBuffers: at most {_native.MAX_PEERS} ranks")
        self._own, self._opened = [], []
        # Every rank takes the same collective steps whatever fails locally; a failure anywhere
        # releases everything on every rank and raises on every rank.
        handles, err = None, None
        try:
            sizes = [ctypes.c_size_t() for _ in range(3)]
            _native.check(lib.apex_attn_peer_exchange_bytes(shape.c(), batch, self.world,
                                                            *map(ctypes.byref, sizes)))
            gather, flags, seq = (self._alloc(lib, n.value) for n in sizes)
            handles = []
            for ptr in (gather, flags):
                h = (ctypes.c_uint8 * 64)()
                _native.check(lib.apex_ipc_get_handle(ptr, h))
                handles.append(bytes(h))
        except Exception as e:  # noqa: BLE001 -- reported collectively below
            handles, err = None, e
        everyone = [None] * self.world
        dist.all_gather_object(everyone, handles, group=group)
        x = _native.PeerExchange()
        if err is None and all(h is not None for h in everyone):
            try:
                x.rank, x.world, x.seq = self.rank, self.world, seq
                for r in range(self.world):
                    if r == self.rank:
                        x.gather[r], x.flags[r] = gather, flags
                        continue
                    for i, h in enumerate(everyone[r]):
                        ptr = ctypes.c_void_p()
                        buf = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                        _native.check(lib.apex_ipc_open_handle(buf, ctypes.byref(ptr)))
                        self._opened.append(ptr.value)
                        if i == 0:
                            x.gather[r] = ptr.value
                        else:
                            x.flags[r] = ptr.value
            except Exception as e:  # noqa: BLE001
                err = e
        ok = torch.tensor([0 if err is not None else 1], dtype=torch.int32, device="cuda")
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()) == 0:
            self.close()
            raise RuntimeError(f"PeerExchangeBuffers: peer-memory exchange unavailable "
                               f"({err!r} here)" if err else "PeerExchangeBuffers: failed on another rank")
        self.exchange = x
        torch.cuda.synchronize()

    def _alloc(self, lib, nbytes: int) -> int:
        ptr = ctypes.c_void_p()
        self._native.check(lib.apex_device_alloc(max(int(nbytes), 16), ctypes.byref(ptr)))
        self._own.append(ptr.value)
        return ptr.value

    def _release(self, lib) -> None:
        for p in self._opened:
            lib.apex_ipc_close_handle(p)
        self._opened = []
        for p in self._own:
            lib.apex_device_free(p)
        self._own = []

    def close(self) -> None:
        """Unmap the peers' buffers, wait until every rank has done the same, free our own."""
        lib = self._native.load()
        torch.cuda.synchronize()
        for p in self._opened:
            lib.apex_ipc_close_handle(p)
        self._opened = []
        self.dist.barrier(group=self.group)
        for p in self._own:
            lib.apex_device_free(p)
        self._own = []
