"""Multi-GPU host logic of the attention path: one process per GPU over torch.distributed.

Only two shardings exist, where the work splits naturally:

* batch sharding (ragged decode, chunked prefill): whole sequences go to ranks, balanced by
  key count (longest first onto the least-loaded rank); no collective on the data path.
* KV-sequence split (one long decode): rank r holds key positions [begin_r, end_r) of every
  sequence; each rank computes a split-KV partial (o, m, l) per (sequence, q head) with
  apex_attn_decode_partial_bf16, ONE all-gather exchanges the partials (16.5 KB per sequence
  per rank at Hq=16, D=256) and every rank merges them with apex_attn_merge_partials.

The reference is single-device; these are new (docs/B6_3_attention.md has no parallelism).
"""
from __future__ import annotations

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
