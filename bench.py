#!/usr/bin/env python
"""Benchmark of the attention hot path on B200 -- one JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload NAME] [--also NAME,NAME,...|none]

Primary workload (the line's metric / value): c5_long_decode_b8 -- eight decodes over a
131072-key bf16 KV cache, 16 q / 8 kv heads, head_dim 256, QK RMSNorm + RoPE of the new token
fused into the split-KV kernel.  One step = one fused decode call.  At N > 1 the KV sequence is
split over the GPUs and the ranks' partials are merged inside the decode kernel over NVLink peer
memory (one launch per step; NCCL all-gather + merge kernel when peer mapping is unavailable).

Every other configuration is measured in the same run and reported under "workloads" (same
fields): c1_decode, c2_prefill_window (one fused prefill = prep + tcgen05 attention),
c3_ragged_decode, c4_chunked_prefill (one step = the whole 32768-token prefill of 4 sequences in
8 chunks of 4096 appended to the cache in order), c5_long_decode_b1, global_decode (the reference
model's global layers: 8 decodes over 32768 keys of 2 kv heads of head_dim 512, GQA group 8, RoPE on
64 pairs, V norm), global_prefill (the same layers' prefill of one 4096-token chunk) and proj_decode /
proj_prefill (the NVFP4 q/k/v projections and o_proj + post-attention RMSNorm of one decode token /
one 4096-token chunk).  At N > 1: c1 / c2 / global_prefill / proj run replicas (weak scaling); c3 and global_decode shard
sequences; c4 shards sequences where the batch divides over the GPUs and kv heads otherwise; c5 splits
the KV sequence (strong scaling).

Timing: W warm-up steps; then EXACTLY K steps replayed from CUDA graphs over rotating input sets
(more bytes than the 126 MB L2 between reuses), bracketed by barrier + synchronize, CUDA events on
the launching stream, max over ranks.  The dominant kernel's own duration is taken with events
around each of its launches (queued behind a GPU sleep so the events bracket only GPU work).  SM
clocks and throttle reasons are sampled through NVML during the timed region.  `e2e` is the same
metric through the public fused C-ABI call with the step's inputs copied from pinned host memory
and its output copied back inside the timed region.

Parity: before timing, one step of every workload is checked on every rank against a plain
PyTorch fp32 restatement of the path (RMSNorm, RoPE, softmax attention; max |err| <= 2e-2, mean
|err| <= 2e-3), and a KV-split decode also against the one-GPU decode of the whole cache.  The run
exits non-zero, after printing its line, if any check fails.

--impl reference times the reference's own CPU implementation of the path (oracle/_ref: the
reference's cpu_ref.h + docs/B6_3_attention.md CPU functions) on the host cores, rank 0 only, on
bounded samples of the same workloads; its `value` is the sample's throughput.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import pathlib
import statistics
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from apex_b200.configs import CONFIGS, decode_bytes, prefill_flops, visible_pairs  # noqa: E402

PRIMARY = "c5_long_decode_b8"
ALSO = ("c1_decode", "c2_prefill_window", "c3_ragged_decode", "c4_chunked_prefill", "c5_long_decode_b1",
        "global_decode", "global_prefill", "proj_decode", "proj_prefill")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1024 * 1024
TOL_MAX, TOL_MEAN = 2e-2, 2e-3          # against an fp32 reference
TOL_SPLIT_MAX, TOL_SPLIT_MEAN = 4e-3, 2e-4  # KV split vs the one-GPU decode (same bf16 inputs)
# DRAM bytes (read + write) per launch of the dominant kernel from one ncu capture of that
# workload; None where no capture exists.  The 8.6 GB
# c5_long_decode_b8 is too large to capture under the size rule: its figure is the c5_long_decode_b1
# capture (same kernel, same keys per sequence) times the 8 sequences -- the traffic is per-sequence
# K/V streaming and grows in proportion.
_C5_B1_TRAFFIC = 1_073_923_000 + 6_035_712
NCU_TRAFFIC_BYTES = {
    "c2_prefill_window": 33_638_400 + 13_312,
    "c3_ragged_decode": 2_307_200_000,
    "c5_long_decode_b1": _C5_B1_TRAFFIC,
    "c5_long_decode_b8": 8 * _C5_B1_TRAFFIC,
    "global_decode": 1_074_024_000 + 4_393_472,
    "global_prefill": 83_921_920 + 26_314_496,
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {k: float(d[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------------------- clocks (NVML)

class ClockSampler(threading.Thread):
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, torch_device: int, period_s: float = 0.005):
        super().__init__(daemon=True)
        self.period = period_s
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self.stop_evt = threading.Event()
        self.ok = False
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_device).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # reading clocks is best effort; the JSON says when it failed
            self.err = repr(e)

    def sample(self):
        if not self.ok:
            return
        try:
            self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
            self.reasons |= self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            pass

    def run(self):
        while not self.stop_evt.is_set():
            self.sample()
            time.sleep(self.period)

    def finish(self):
        self.stop_evt.set()
        self.join(timeout=1.0)
        self.sample()
        if not self.ok:
            return {"error": getattr(self, "err", "nvml unavailable")}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples),
                "source": "NVML during the timed region"}


# ---------------------------------------------------------------------------- fp32 restatement (checker)

def t_norm_rope(x, w, pos, pairs, base, eps, norm=True):
    """RMSNorm over the last dim (sum of squares in double, weight as stored) and rotate-half RoPE
    on the first `pairs` pairs (i, i + D/2) at positions `pos` (broadcast over the leading dims)."""
    import torch
    D = x.shape[-1]
    y = x.float()
    if norm:
        ms = y.double().pow(2).mean(-1, keepdim=True).float()
        y = y * torch.rsqrt(ms + eps)
        if w is not None:
            y = y * w.float()
    if pairs:
        i = torch.arange(pairs, device=x.device, dtype=torch.float64)
        inv = (float(base) ** (-2.0 * i / D)).float()
        ang = (pos.float().unsqueeze(-1) * inv).double()
        c, s = ang.cos().float(), ang.sin().float()
        a, b = y[..., :pairs].clone(), y[..., D // 2:D // 2 + pairs].clone()
        y = y.clone()
        y[..., :pairs] = a * c - b * s
        y[..., D // 2:D // 2 + pairs] = a * s + b * c
    return y


def t_attend(q, K, V, first, last, scale):
    """q [D] f32, K/V [L, D]: softmax(scale q.K[first..last]) V."""
    import torch
    s = (K[first:last + 1].float() @ q) * scale
    return torch.softmax(s, 0) @ V[first:last + 1].float()


def err_of(got, ref):
    e = (got.float() - ref.float()).abs()
    if not bool(torch_isfinite(got)):
        return float("inf"), float("inf")
    return float(e.max().item()), float(e.mean().item())


def torch_isfinite(t):
    import torch
    return torch.isfinite(t.float()).all()


# ---------------------------------------------------------------------------- workloads

def _randn(g, device, *s, scale=1.0, mean=0.0):
    import torch
    return (torch.randn(*s, generator=g, device=device) * scale + mean).to(torch.bfloat16)


class PrefillWorkload:
    """One step = the configuration's whole prefill: every chunk of every sequence, each chunk one
    fused call (prep kernel: q/k norm + RoPE, K/V appended to the cache; tcgen05 attention kernel)
    appended in order.  At N > 1 c4 shards sequences (batch divides over N) or kv heads."""
    kind = "prefill"

    def __init__(self, cfg, device, rank=0, world=1):
        import torch
        from apex_b200 import ops
        self.cfg0, self.ops, self.torch = cfg, ops, torch
        self.sharding = "replica"
        if cfg.name.startswith("c4") and world > 1:
            if cfg.batch % world == 0:
                self.sharding = "batch-shard"
                cfg = dataclasses.replace(cfg, batch=cfg.batch // world)
            elif cfg.kv_heads % world == 0:
                self.sharding = "kv-head-shard"
                cfg = dataclasses.replace(cfg, q_heads=cfg.q_heads // world, kv_heads=cfg.kv_heads // world)
            else:
                raise SystemExit(f"{cfg.name}: neither the batch nor the kv heads divide over {world} GPUs")
        self.cfg = cfg
        B, T, Hq, Hkv, D = cfg.batch, cfg.chunk, cfg.q_heads, cfg.kv_heads, cfg.head_dim
        self.B, self.T, self.n_chunks = B, T, cfg.seq_len // cfg.chunk
        self.pos0s = [c * T for c in range(self.n_chunks)]
        self.shape = ops.AttentionShape.from_config(cfg)
        g = torch.Generator(device=device).manual_seed(cfg.seed * 1000 + rank)
        self.qw, self.kw = _randn(g, device, D, scale=0.1, mean=1.0), _randn(g, device, D, scale=0.1, mean=1.0)
        cap = cfg.seq_len
        C = self.n_chunks
        per_set = 2 * C * (B * T * Hq * D * 2 + B * T * Hkv * D * 2 * 2) + 2 * B * Hkv * cap * D * 2
        self.R = max(1, min(16, math.ceil(2 * L2_BYTES / per_set)))
        self.sets = []
        for _ in range(self.R):
            s = dict(q=_randn(g, device, C, B, T, Hq, D), k=_randn(g, device, C, B, T, Hkv, D),
                     v=_randn(g, device, C, B, T, Hkv, D),
                     kc=torch.zeros(B, Hkv, cap, D, dtype=torch.bfloat16, device=device),
                     vc=torch.zeros(B, Hkv, cap, D, dtype=torch.bfloat16, device=device),
                     ws=ops.PrefillWorkspace(self.shape, B, T, device=device),
                     out=torch.empty(C, B, T, Hq, D, dtype=torch.bfloat16, device=device))
            s["cache"] = ops.KvCache(s["kc"], s["vc"])
            self.sets.append(s)
        self.ws = ops.PrefillWorkspace(self.shape, B, T, device=device)
        self.chunk_flops = [prefill_flops(cfg, p0, T) * B for p0 in self.pos0s]
        self.flops = sum(self.chunk_flops)      # this rank's share of the step
        self.units = self.flops
        owns_tokens = self.sharding != "kv-head-shard" or rank == 0
        self.tokens = B * T * C if owns_tokens else 0
        self.launches_per_step = 2 * C
        # head_dim 512 (the global layers): the tcgen05 pair kernel for groups of 1, 2, 4 and 8, else
        # the mma.sync form
        if cfg.head_dim == 512:
            self.kernel_name = "prefill_wide_kernel" if Hq // Hkv in (1, 2, 4, 8) else "prefill_gqa_kernel"
        else:
            self.kernel_name = "prefill_pair_kernel"

    def _chunk(self, s, c, out, ws):
        self.ops.attention_prefill_prep(self.shape, s["q"][c], s["k"][c], s["v"][c], self.qw, self.kw, s["cache"],
                                        self.pos0s[c], ws)
        self.ops.attention_prefill_attend(self.shape, ws, s["cache"], self.B, self.T, self.pos0s[c], out[c])

    def step(self, i):
        s = self.sets[i % self.R]
        for c in range(self.n_chunks):
            self._chunk(s, c, s["out"], s["ws"])

    def dominant_launches(self, i, record):
        """Prep each chunk, then the attention kernel between events; returns algorithmic FLOPs."""
        s = self.sets[i % self.R]
        for c in range(self.n_chunks):
            self.ops.attention_prefill_prep(self.shape, s["q"][c], s["k"][c], s["v"][c], self.qw, self.kw,
                                            s["cache"], self.pos0s[c], s["ws"])
            record(lambda: self.ops.attention_prefill_attend(self.shape, s["ws"], s["cache"], self.B, self.T,
                                                             self.pos0s[c], s["out"][c]))
        return self.flops

    def roofline_work(self):
        return self.flops, "tensor"

    def e2e_inputs(self):
        s = self.sets[0]
        return [s["q"], s["k"], s["v"]], s["out"]

    def e2e_compute(self, ins, out):
        q, k, v = ins
        for c in range(self.n_chunks):
            self.ops.attention_prefill(self.shape, q[c], k[c], v[c], self.qw, self.kw, self.sets[0]["cache"],
                                       self.pos0s[c], out[c], self.ws)

    def parity(self):
        """One step on set 0, then sampled query rows of the first and last sequence of this rank
        against the fp32 restatement (window and chunk edges included)."""
        torch = self.torch
        cfg = self.cfg
        self.step(0)
        torch.cuda.synchronize()
        self.ops.device_status()
        s = self.sets[0]
        S, T, D, G = cfg.seq_len, self.T, cfg.head_dim, cfg.q_heads // cfg.kv_heads
        rows = {0, 1, S - 1, S // 2}
        if cfg.window:
            rows |= {cfg.window - 2, cfg.window - 1, cfg.window, cfg.window + 1, S - cfg.window}
        for p0 in self.pos0s[1:]:
            rows |= {p0 - 1, p0, p0 + 1}
        rows = sorted(r for r in rows if 0 <= r < S)
        worst = (0.0, 0.0)
        for b in sorted({0, self.B - 1}):
            q_raw = s["q"][:, b].reshape(S, cfg.q_heads, D)
            k_raw = s["k"][:, b].reshape(S, cfg.kv_heads, D)
            v_raw = s["v"][:, b].reshape(S, cfg.kv_heads, D)
            pos = torch.arange(S, device=q_raw.device)
            Kf = t_norm_rope(k_raw, self.kw, pos[:, None], cfg.rope_pairs, cfg.rope_theta, cfg.eps)
            Vf = t_norm_rope(v_raw, None, pos[:, None], 0, cfg.rope_theta, cfg.eps, norm=cfg.v_norm)
            rsel = torch.tensor(rows, device=q_raw.device)
            Qf = t_norm_rope(q_raw[rsel], self.qw, rsel[:, None], cfg.rope_pairs, cfg.rope_theta, cfg.eps)
            got = s["out"][:, b].reshape(S, cfg.q_heads, D)[rsel]
            ref = torch.empty_like(Qf)
            for i, p in enumerate(rows):
                first = p + 1 - cfg.window if (cfg.window and p + 1 > cfg.window) else 0
                for h in range(cfg.q_heads):
                    ref[i, h] = t_attend(Qf[i, h], Kf[:, h // G], Vf[:, h // G], first, p, cfg.scale)
            mx, mn = err_of(got, ref)
            worst = (max(worst[0], mx), max(worst[1], mn))
            del Kf, Vf
        return {"max_abs": worst[0], "mean_abs": worst[1], "rows_checked": len(rows) * len(sorted({0, self.B - 1})),
                "ref": "torch fp32 restatement (norm, RoPE, softmax) of sampled rows incl. window / chunk edges",
                "ok": worst[0] <= TOL_MAX and worst[1] <= TOL_MEAN}

    def close(self):
        pass


class DecodeWorkload:
    """One fused decode step per step; sequences sharded (c3) or the KV range split (c5) across
    ranks; c1 runs replicas."""
    kind = "decode"

    def __init__(self, cfg, device, rank=0, world=1):
        import torch
        from apex_b200 import dist as adist
        from apex_b200 import ops
        self.cfg, self.ops, self.torch, self.device = cfg, ops, torch, device
        self.rank, self.world = rank, world
        Hq, Hkv, D = cfg.q_heads, cfg.kv_heads, cfg.head_dim
        self.shape = ops.AttentionShape.from_config(cfg)
        gl = torch.Generator(device="cpu").manual_seed(cfg.seed)
        if cfg.lens_range:
            lo, hi = cfg.lens_range
            lens_all = torch.randint(lo, hi + 1, (cfg.batch,), generator=gl).tolist()
        else:
            lens_all = [cfg.context] * cfg.batch
        self.kv_split = cfg.name.startswith("c5") and world > 1
        batch_shard = not self.kv_split and world > 1 and cfg.batch >= world
        mine = adist.shard_sequences(lens_all, world)[rank] if batch_shard else list(range(cfg.batch))
        self.sharding = "kv-split" if self.kv_split else "batch-shard" if batch_shard else "replica"
        self.lens = [lens_all[i] for i in mine]
        self.all_lens = lens_all
        B = len(self.lens)
        self.B = B
        L = max(self.lens)
        self.L = L
        if self.kv_split:
            self.kv_begin, self.kv_end = adist.kv_ranges(L, world)[rank]
        else:
            self.kv_begin, self.kv_end = 0, L
        cap = self.kv_end - self.kv_begin
        # the same new-token inputs and (for the KV split) the same whole cache on every rank
        g = torch.Generator(device=device).manual_seed(cfg.seed * 1000 + (0 if self.kv_split else rank))
        self.qw, self.kw = _randn(g, device, D, scale=0.1, mean=1.0), _randn(g, device, D, scale=0.1, mean=1.0)
        per_set = 2 * B * Hkv * cap * D * 2
        self.R = max(1, min(64, math.ceil(2 * L2_BYTES / per_set)))
        self.full = None
        if self.kv_split:  # set 0 is this rank's slice of a whole cache every rank draws alike
            kf, vf = _randn(g, device, B, Hkv, L, D), _randn(g, device, B, Hkv, L, D)
            self.full = ops.KvCache(kf, vf)
        self.sets = []
        for r in range(self.R):
            s = dict(q=_randn(g, device, B, Hq, D), k=_randn(g, device, B, Hkv, D), v=_randn(g, device, B, Hkv, D),
                     out=torch.empty(B, Hq, D, dtype=torch.bfloat16, device=device))
            if r == 0 and self.full is not None:
                s["kc"] = self.full.k[:, :, self.kv_begin:self.kv_end].contiguous()
                s["vc"] = self.full.v[:, :, self.kv_begin:self.kv_end].contiguous()
            else:
                s["kc"], s["vc"] = _randn(g, device, B, Hkv, cap, D), _randn(g, device, B, Hkv, cap, D)
            s["cache"] = ops.KvCache(s["kc"], s["vc"])
            self.sets.append(s)
        self.lens_t = torch.tensor(self.lens, dtype=torch.int32, device=device)
        self.ws = ops.DecodeWorkspace(self.shape, B, L, device=device)
        self.peer, self.exchange = None, "none"
        if self.kv_split:
            # fused: partials merged inside the decode kernel through NVLink peer memory; if the
            # peer mapping is unavailable on any rank, every rank uses the NCCL all-gather instead
            self.splitter = adist.KVSplitDecode(B, Hq, D, device)
            self.partial = torch.empty(B, Hq, D + 2, dtype=torch.float32, device=device)
            try:
                self.peer = adist.PeerExchangeBuffers(self.shape, B)
                self.exchange = "fused peer stores over NVLink (in-kernel merge)"
            except RuntimeError as e:
                self.exchange = f"NCCL all-gather + merge kernel (peer mapping unavailable: {e})"
            local = sum(2 * Hkv * max(0, min(Li, self.kv_end) - self.kv_begin) * D * 2 for Li in self.lens)
            self.bytes = local + 2 * B * Hq * D * 2
        else:
            self.bytes = decode_bytes(cfg, self.lens)
        self.units = self.bytes
        owns_tokens = not self.kv_split or rank == 0
        self.tokens = B if owns_tokens else 0
        self.launches_per_step = 2 if self.kv_split and self.peer is None else 1
        # head_dim 512 or a GQA group other than 2 runs the tensor-core decode (decode_gqa.cu)
        gqa_form = cfg.head_dim != 256 or Hq != 2 * Hkv
        self.kernel_name = ("decode_gqa_kernel" if gqa_form else "decode_kernel") + (
            " (partial mode, this rank's key range)" if self.kv_split else "")

    def _call(self, s):
        if self.peer is not None:
            self.ops.attention_decode_kvsplit(self.shape, s["q"], s["k"], s["v"], self.qw, self.kw, s["cache"],
                                              self.lens_t, self.L, self.kv_begin, self.kv_end, self.peer.exchange,
                                              s["out"], self.ws)
        elif self.kv_split:
            ops = self.ops

            def partial(p):
                ops.attention_decode_partial(self.shape, s["q"], s["k"], s["v"], self.qw, self.kw, s["cache"],
                                             self.lens_t, self.L, self.kv_begin, self.kv_end, p, self.ws)

            self.splitter.step(partial, lambda parts, out: ops.merge_partials(parts, out), s["out"])
        else:
            self.ops.attention_decode(self.shape, s["q"], s["k"], s["v"], self.qw, self.kw, s["cache"], self.lens_t,
                                      self.L, s["out"], self.ws)

    def step(self, i):
        self._call(self.sets[i % self.R])

    def dominant_launches(self, i, record):
        """The decode kernel between events (for a KV split: its partial mode over this rank's
        range, without the exchange, so the events do not include waits for other ranks)."""
        s = self.sets[i % self.R]
        if self.kv_split:
            record(lambda: self.ops.attention_decode_partial(
                self.shape, s["q"], s["k"], s["v"], self.qw, self.kw, s["cache"], self.lens_t, self.L,
                self.kv_begin, self.kv_end, self.partial, self.ws))
        else:
            record(lambda: self._call(s))
        return self.bytes

    def roofline_work(self):
        return self.bytes, "hbm"

    def e2e_inputs(self):
        s = self.sets[0]
        return [s["q"], s["k"], s["v"]], s["out"]

    def e2e_compute(self, ins, out):
        s = dict(self.sets[0])
        s["q"], s["k"], s["v"], s["out"] = ins[0], ins[1], ins[2], out
        self._call(s)

    def parity(self):
        """One step on set 0 against the fp32 restatement for sampled sequences; a KV split also
        against the one-GPU decode of the whole cache on this GPU."""
        torch, cfg = self.torch, self.cfg
        s = self.sets[0]
        self._call(s)
        torch.cuda.synchronize()
        self.ops.device_status()
        got = s["out"].clone()
        res = {}
        if self.kv_split:
            one = torch.empty_like(got)
            ws = self.ops.DecodeWorkspace(self.shape, self.B, self.L, device=self.device)
            self.ops.attention_decode(self.shape, s["q"], s["k"], s["v"], self.qw, self.kw, self.full,
                                      self.lens_t, self.L, one, ws)
            torch.cuda.synchronize()
            mx, mn = err_of(got, one)
            res["vs_one_gpu_decode"] = {"max_abs": mx, "mean_abs": mn,
                                        "ok": mx <= TOL_SPLIT_MAX and mn <= TOL_SPLIT_MEAN}
        D, G = cfg.head_dim, cfg.q_heads // cfg.kv_heads
        worst = (0.0, 0.0)
        longest = max(range(self.B), key=lambda b: self.lens[b])
        seqs = sorted({0, longest, self.B - 1})
        for b in seqs:
            L = self.lens[b]
            if self.kv_split:
                Kc, Vc = self.full.k[b, :, :L - 1], self.full.v[b, :, :L - 1]
            else:
                Kc, Vc = s["kc"][b, :, :L - 1], s["vc"][b, :, :L - 1]
            pos = torch.full((1,), L - 1, device=got.device)
            qf = t_norm_rope(s["q"][b], self.qw, pos, cfg.rope_pairs, cfg.rope_theta, cfg.eps)
            kn = t_norm_rope(s["k"][b], self.kw, pos, cfg.rope_pairs, cfg.rope_theta, cfg.eps)
            vn = t_norm_rope(s["v"][b], None, pos, 0, cfg.rope_theta, cfg.eps, norm=cfg.v_norm)
            first = L - cfg.window if (cfg.window and L > cfg.window) else 0
            ref = torch.empty(cfg.q_heads, D, device=got.device)
            for kvh in range(cfg.kv_heads):
                K = torch.cat([Kc[kvh].float(), kn[kvh][None]], 0)
                V = torch.cat([Vc[kvh].float(), vn[kvh][None]], 0)
                for h in range(kvh * G, (kvh + 1) * G):
                    ref[h] = t_attend(qf[h], K, V, first, L - 1, cfg.scale)
                del K, V
            mx, mn = err_of(got[b], ref)
            worst = (max(worst[0], mx), max(worst[1], mn))
        res.update(max_abs=worst[0], mean_abs=worst[1], seqs_checked=len(seqs),
                   ref="torch fp32 restatement (norm, RoPE, softmax) of whole sequences")
        res["ok"] = worst[0] <= TOL_MAX and worst[1] <= TOL_MEAN and res.get("vs_one_gpu_decode", {}).get("ok", True)
        return res

    def close(self):
        self.full = None
        if self.peer is not None:
            self.peer.close()  # unmaps the peers' buffers on every rank before any rank frees its own
            self.peer = None


class ProjWorkload:
    """The projections either side of one attention step of a sliding layer of the reference model
    (docs/B6_3_attention.md:46-60): q (4096 x 2816), k and v (2048 x 2816) from the normed hidden
    state to bf16 raw rows (what the fused attention takes), and o_proj (2816 x 4096) over the bf16
    attention output with the post-attention RMSNorm.  NVFP4 weights (E2M1 codes, E4M3 per-16
    scales).  proj_decode: one token, f32 hidden state (the reference's), q, k and v in one launch
    (apex_matmul_nvfp4_multi: they share the input) and o_proj with the norm fused into its epilogue;
    algorithmic bytes = weight codes + scales + activations.  proj_prefill: one 4096-token chunk of
    bf16 activations on the tensor-core form (each projection one tcgen05 GEMM over exactly
    dequantised weights), the norm a second launch; algorithmic work = 2 x tokens x weights FLOPs.
    N > 1: replicas."""
    kind = "proj"
    SHAPES = (("q", 4096, 2816), ("k", 2048, 2816), ("v", 2048, 2816), ("o", 2816, 4096))

    def __init__(self, cfg, device, rank=0, world=1):
        import torch
        from apex_b200 import ops
        self.ops, self.torch, self.cfg = ops, torch, cfg
        self.sharding = "replica"
        T = self.T = cfg.chunk or 1
        self.prefill = T > 1
        g = torch.Generator(device=device).manual_seed(900 + rank)
        wbytes = sum(r * n // 2 + r * n // 16 for _, r, n in self.SHAPES)
        self.R = max(2, math.ceil(2 * L2_BYTES / wbytes) + 1)

        def matrix(r, n):
            codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (r, n // 8), generator=g, dtype=torch.int32, device=device)
            scales = torch.randint(0x20, 0x40, (r, n // 16), generator=g, dtype=torch.uint8, device=device)
            return ops.Nvfp4Matrix(codes, scales)

        self.sets = [{k: matrix(r, n) for k, r, n in self.SHAPES} for _ in range(self.R)]
        x_dtype = torch.bfloat16 if self.prefill else torch.float32
        self.x = torch.randn(T, 2816, generator=g, device=device).to(x_dtype)
        self.att = torch.randn(T, 4096, generator=g, device=device).to(torch.bfloat16)
        self.nw = (torch.randn(2816, generator=g, device=device) * 0.1 + 1.0).to(torch.bfloat16)
        self.q = torch.empty(T, 4096, dtype=torch.bfloat16, device=device)
        self.k = torch.empty(T, 2048, dtype=torch.bfloat16, device=device)
        self.v = torch.empty(T, 2048, dtype=torch.bfloat16, device=device)
        self.o = torch.empty(T, 2816, device=device)
        self.ws = ops.ProjNormWorkspace(2816, min(T, 16), device=device)
        xb = self.x.element_size()
        self.bytes = wbytes + T * (2816 * xb + 4096 * 2 + (4096 + 2048 * 2) * 2 + 2816 * 4)
        self.flops = 2 * T * sum(r * n for _, r, n in self.SHAPES)
        self.units = self.flops if self.prefill else self.bytes
        self.tokens = T
        if self.prefill:
            self.launches_per_step = 5
            self.kernel_name = "nvfp4_tc_kernel (q, k, v, o_proj: tcgen05 GEMMs) + rms_norm"
        else:
            self.launches_per_step = 2
            self.kernel_name = "nvfp4_stream_kernel (q+k+v in one launch, fused o_proj + rms_norm)"

    def _run(self, W, x, att, q, k, v, o):
        ops = self.ops
        ops.matmul_nvfp4_multi(x, [W["q"], W["k"], W["v"]], [q, k, v], self.T)
        ops.matmul_nvfp4_rms_norm(att, W["o"], self.nw, o, self.T, 1e-6, self.ws)

    def step(self, i):
        self._run(self.sets[i % self.R], self.x, self.att, self.q, self.k, self.v, self.o)

    def dominant_launches(self, i, record):
        record(lambda: self.step(i))
        return self.units

    def roofline_work(self):
        return (self.flops, "tensor") if self.prefill else (self.bytes, "hbm")

    def e2e_inputs(self):
        return [self.x, self.att], self.o

    def e2e_compute(self, ins, out):
        self._run(self.sets[0], ins[0], ins[1], self.q, self.k, self.v, out)

    def parity(self):
        """Against the weights decoded in torch (E2M1 table x E4M3 scale) and fp64 dot products:
        rel-L2 < 1e-5 for the f32 output (the reference's gate), bf16 rounding for the bf16 rows."""
        torch = self.torch
        self.step(0)
        torch.cuda.synchronize()
        self.ops.device_status()
        W = self.sets[0]
        lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=torch.float64,
                           device=self.x.device)

        def dense(M):
            c = M.codes.view(torch.int32)
            nib = torch.stack([(c >> (4 * j)) & 0xF for j in range(8)], -1).reshape(c.shape[0], -1).long()
            b = M.scales.long()
            e, m = (b >> 3) & 0xF, (b & 7).double()
            sc = torch.where(e == 0, m / 512.0, (1 + m / 8) * torch.pow(2.0, (e - 7).double()))
            sc = torch.where((b & 0x80) != 0, -sc, sc)
            return lut[nib] * sc.repeat_interleave(16, 1)

        worst, rel, over = 0.0, 0.0, 0.0
        for name, out in (("q", self.q), ("k", self.k), ("v", self.v)):
            Wd = dense(W[name])
            ref = (Wd @ self.x.double().T).T
            if self.prefill:  # millions of outputs, some near zero: the bf16 rounding as a relative L2
                err = ((out.double() - ref).norm() / ref.norm()).item()
            else:
                # one bf16 rounding of each output (2^-9 of |ref|, doubled) plus the f32 accumulation
                # error, bounded by 1e-6 of sum |w x| (outputs that nearly cancel have a large
                # relative error that is neither rounding nor a fault)
                absdot = (Wd.abs() @ self.x.double().abs().T).T
                diff = (out.double() - ref).abs()
                err = (diff / ref.abs().clamp_min(1e-3)).max().item()
                over = max(over, (diff / (2 ** -8 * ref.abs() + 1e-6 * absdot)).max().item())
            worst = max(worst, err)
        ro = (dense(W["o"]) @ self.att.double().T).T
        ro = ro * torch.rsqrt((ro ** 2).mean(-1, keepdim=True) + 1e-6) * self.nw.double()
        rel = ((self.o.double() - ro).norm() / ro.norm()).item()
        key = "qkv_bf16_rel_l2" if self.prefill else "qkv_bf16_max_rel"
        rep = {"max_abs": worst, "mean_abs": rel, "o_proj_norm_rel_l2": rel, key: worst,
               "ref": "torch fp64: weights decoded from the E2M1 / E4M3 bits"}
        if self.prefill:
            rep["ok"] = rel < 1e-5 and worst <= 2 ** -8
        else:
            rep["qkv_err_over_bound"] = over  # bound: 2^-8 |ref| + 1e-6 sum |w x|
            rep["ok"] = rel < 1e-5 and over <= 1.0
        return rep

    def close(self):
        pass


# ---------------------------------------------------------------------------- reference arm (CPU)

_REF_CACHE = {}


def _ref_decode_setup(cfg, b, L, ref):
    """The cache of sequence b built by the reference's head_norm_rope (untimed: it exists before a
    decode step) and the new token's raw rows."""
    import numpy as np
    import oracle
    from oracle import inputs as I
    key = (cfg.seed, cfg.rope_theta, cfg.window, b, L)   # c5_b1 and c5_b8 share sequence 0
    if key in _REF_CACHE:
        return _REF_CACHE[key]
    Hkv, D = cfg.kv_heads, cfg.head_dim
    qw, kw = I.norm_weights(cfg)
    k = I.f32(I.k_rows(cfg, b, 0, L))
    Kc = np.zeros(Hkv * L * D, np.float32)
    oracle.head_norm_rope_f32(k[:L - 1], kw, Kc, L - 1, Hkv, D, 1, cfg.rope_pairs, cfg.rope_theta, 0, D, L * D,
                              cfg.eps, ref=ref)
    del k
    v = I.f32(I.v_rows(cfg, b, 0, L))
    Vc = np.zeros(Hkv * L * D, np.float32)
    if cfg.v_norm:  # the global layers: weightless RMSNorm of V (docs/B6_3_attention.md:25)
        oracle.head_norm_rope_f32(v[:L - 1], None, Vc, L - 1, Hkv, D, 0, 0, cfg.rope_theta, 0, D, L * D, cfg.eps,
                                  ref=ref)
    else:
        Vc.reshape(Hkv, L, D)[:, :L - 1] = v[:L - 1].transpose(1, 0, 2)
    new = (I.f32(I.q_rows(cfg, b, L - 1, L)), I.f32(I.k_rows(cfg, b, L - 1, L)), v[L - 1:].copy())
    _REF_CACHE[key] = (Kc, Vc, new, qw, kw)
    return _REF_CACHE[key]


def cpu_reference_step(cfg, threads):
    """One step of the reference's CPU path on a bounded sample.  Returns (seconds, algorithmic
    units of the sample, sample description, kind)."""
    import numpy as np
    import oracle
    from oracle import inputs as I
    oracle.set_threads(threads)
    ref = oracle.ref_lib() is not None
    kind = "reference" if ref else "port"
    if cfg.kind == "proj":  # matvecNvfp4Cpu on the four projections, then rmsNormCpu
        key = ("proj",)
        if key not in _REF_CACHE:
            _REF_CACHE[key] = [oracle.nvfp4_matrix(r, n, 900 + i) + (r, n)
                               for i, (_, r, n) in enumerate(ProjWorkload.SHAPES)]
        mats = _REF_CACHE[key]
        nw = oracle.normal_bf16(2816, 900, 4, 0, 1.0, 0.1)
        # prefill: a sample of 4 tokens of the chunk (bf16-valued activations), value = their FLOPs / time
        T = 4 if cfg.chunk else 1
        xs = {n: np.random.default_rng(n).standard_normal((T, n)).astype(np.float32) for _, _, n in ProjWorkload.SHAPES}
        if cfg.chunk:
            xs = {n: oracle.bf16_to_f32(oracle.f32_to_bf16(x.ravel())).reshape(T, n) for n, x in xs.items()}
        t0 = time.perf_counter()
        for codes, scales, r, n in mats:
            y = oracle.matvec_nvfp4(codes, scales, xs[n], T, r, n, ref=ref)
        oracle.rms_norm_rows(y, nw, T, 2816, 1e-6, ref=ref)
        dt = time.perf_counter() - t0
        if cfg.chunk:
            flops = 2 * T * sum(r * n for _, r, n in ProjWorkload.SHAPES)
            return dt, flops, (f"the four projections of {T} of the chunk's {cfg.chunk} tokens (matvecNvfp4Cpu) + "
                               "rmsNormCpu; value = their FLOPs / time"), kind
        nbytes = sum(r * n // 2 + r * n // 16 for _, r, n in ProjWorkload.SHAPES)
        return dt, nbytes, "the four projections of one decode token (matvecNvfp4Cpu) + rmsNormCpu; value = weight bytes / time", kind
    Hq, Hkv, D = cfg.q_heads, cfg.kv_heads, cfg.head_dim
    if cfg.kind == "prefill":
        # c2: the whole prompt; c4 and global_prefill: 16 query rows of the last chunk of sequence 0
        # (the cache of the earlier chunks is built outside the timed region)
        qw, kw = I.norm_weights(cfg)
        S = cfg.seq_len
        last = cfg.name.startswith("c4") or cfg.head_dim == 512
        key = (cfg.name, "prefill")
        if key not in _REF_CACHE:
            _REF_CACHE[key] = (I.f32(I.q_rows(cfg, 0, 0, S)).ravel(), I.f32(I.k_rows(cfg, 0, 0, S)),
                               I.f32(I.v_rows(cfg, 0, 0, S)))
        q_all, k, v = _REF_CACHE[key]
        if last:
            p0 = S - cfg.chunk
            rows = list(range(p0, S, cfg.chunk // 16))[:15] + [S - 1]
            ckey = (cfg.name, "cache")
            if ckey not in _REF_CACHE:
                Kc = np.zeros(Hkv * S * D, np.float32)
                oracle.head_norm_rope_f32(k[:p0], kw, Kc, p0, Hkv, D, 1, cfg.rope_pairs, cfg.rope_theta, 0, D, S * D,
                                          cfg.eps, ref=ref)
                _REF_CACHE[ckey] = Kc
            Kc = _REF_CACHE[ckey].copy()
            t0 = time.perf_counter()
            oracle.head_norm_rope_f32(k[p0:], kw, Kc[p0 * D:], S - p0, Hkv, D, 1, cfg.rope_pairs, cfg.rope_theta, p0, D,
                                      S * D, cfg.eps, ref=ref)
            if cfg.v_norm:
                Vc = np.zeros(Hkv * S * D, np.float32)
                oracle.head_norm_rope_f32(v, None, Vc, S, Hkv, D, 0, 0, cfg.rope_theta, 0, D, S * D, cfg.eps, ref=ref)
            else:
                Vc = np.ascontiguousarray(v.transpose(1, 0, 2)).ravel()
            qs = np.ascontiguousarray(q_all.reshape(S, Hq, D)[rows]).ravel()
            qn = np.zeros_like(qs)
            for i, r in enumerate(rows):
                oracle.head_norm_rope_f32(qs[i * Hq * D:(i + 1) * Hq * D], qw, qn[i * Hq * D:(i + 1) * Hq * D], 1, Hq,
                                          D, 1, cfg.rope_pairs, cfg.rope_theta, r, Hq * D, D, cfg.eps, ref=ref)
            for i, r in enumerate(rows):
                oracle.attention_f32(qn[i * Hq * D:(i + 1) * Hq * D], Kc, Vc, 1, Hq, Hkv, D, S, r, cfg.window,
                                     cfg.scale, ref=ref)
            dt = time.perf_counter() - t0
            flops = 4 * Hq * D * sum(visible_pairs(r, 1, cfg.window) for r in rows)
            desc = (f"{len(rows)} query rows of the last chunk (positions {rows[0]}..{rows[-1]}) x {Hq} heads of "
                    f"sequence 0, with that chunk's K norm + RoPE{' and V norm' if cfg.v_norm else ''} into the "
                    f"cache; value = the sample's FLOPs / time")
            return dt, flops, desc, kind
        t0 = time.perf_counter()
        Kc = np.zeros(Hkv * S * D, np.float32)
        oracle.head_norm_rope_f32(k, kw, Kc, S, Hkv, D, 1, cfg.rope_pairs, cfg.rope_theta, 0, D, S * D, cfg.eps, ref=ref)
        Vc = np.ascontiguousarray(v.transpose(1, 0, 2)).ravel()
        qn = np.zeros_like(q_all)
        oracle.head_norm_rope_f32(q_all, qw, qn, S, Hq, D, 1, cfg.rope_pairs, cfg.rope_theta, 0, Hq * D, D, cfg.eps,
                                  ref=ref)
        oracle.attention_f32(qn, Kc, Vc, S, Hq, Hkv, D, S, 0, cfg.window, cfg.scale, ref=ref)
        dt = time.perf_counter() - t0
        flops = prefill_flops(cfg, 0, S)
        desc = f"the whole prefill of sequence 0 ({S} tokens x {Hq} heads, K/V cache build included)"
        return dt, flops, desc, kind
    # decode: the step of the sampled sequences over caches built beforehand (untimed)
    lens = [int(x) for x in I.decode_lens(cfg)]
    seqs = list(range(min(cfg.batch, 1 if cfg.context >= 65536 else 4)))
    setups = [_ref_decode_setup(cfg, b, lens[b], ref) for b in seqs]
    t0 = time.perf_counter()
    for b, (Kc, Vc, (q, kn, vn), qw, kw) in zip(seqs, setups):
        L = lens[b]
        qn = np.zeros(Hq * D, np.float32)
        oracle.head_norm_rope_f32(q, qw, qn, 1, Hq, D, 1, cfg.rope_pairs, cfg.rope_theta, L - 1, Hq * D, D, cfg.eps,
                                  ref=ref)
        oracle.head_norm_rope_f32(kn, kw, Kc[(L - 1) * D:], 1, Hkv, D, 1, cfg.rope_pairs, cfg.rope_theta, L - 1, D,
                                  L * D, cfg.eps, ref=ref)
        if cfg.v_norm:
            oracle.head_norm_rope_f32(vn, None, Vc[(L - 1) * D:], 1, Hkv, D, 0, 0, cfg.rope_theta, L - 1, D, L * D,
                                      cfg.eps, ref=ref)
        else:
            Vc.reshape(Hkv, L, D)[:, L - 1] = vn[0]
        oracle.attention_f32(qn, Kc, Vc, 1, Hq, Hkv, D, L, L - 1, cfg.window, cfg.scale, ref=ref)
    dt = time.perf_counter() - t0
    nbytes = decode_bytes(cfg, [lens[b] for b in seqs])
    desc = (f"one decode step of {len(seqs)} of {cfg.batch} sequences ({', '.join(str(lens[b]) for b in seqs)} keys; "
            f"new token's norm + RoPE and cache append included, caches built beforehand); value = the sample's "
            f"K/V + q/o bytes / time")
    return dt, nbytes, desc, kind


def metric_of(cfg):
    if cfg.kind == "prefill":
        return "prefill attn TFLOP/s", "TFLOP/s", 1e12
    if cfg.kind == "proj":
        if cfg.chunk:
            return "prefill projections TFLOP/s", "TFLOP/s", 1e12
        return "decode projections GB/s", "GB/s", 1e9
    return "decode attn KV GB/s", "GB/s", 1e9


def cpu_baseline(cfg, threads):
    dt, units, desc, kind = cpu_reference_step(cfg, threads)
    _, unit, scale = metric_of(cfg)
    return {"value": units / dt / scale, "unit": unit, "cores": threads, "kind": kind, "sample": desc,
            "ms_per_sample": dt * 1e3}


def config_of(cfg):
    if cfg.kind == "proj":
        return {"workload": cfg.name, "tokens": cfg.chunk or 1, "matrices": {k: [r, n] for k, r, n in ProjWorkload.SHAPES},
                "weights": "NVFP4 (E2M1 codes, E4M3 per-16 scales)", "activations": "bf16" if cfg.chunk else "f32",
                "fused": "o_proj + post-attention rms_norm"}
    c = {"workload": cfg.name, "batch": cfg.batch, "q_heads": cfg.q_heads, "kv_heads": cfg.kv_heads,
         "head_dim": cfg.head_dim, "window": cfg.window, "rope_theta": cfg.rope_theta,
         "qk_norm": cfg.qk_norm, "scale": "1/sqrt(head_dim)"}
    if cfg.kind == "prefill":
        c.update(seq_len=cfg.seq_len, chunk=cfg.chunk)
    else:
        c.update(context=cfg.context or list(cfg.lens_range))
    return c


def run_reference(args, names):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    primary = CONFIGS[names[0]]
    metric, unit, scale = metric_of(primary)
    secs, units, desc, kind = [], None, None, None
    for i in range(args.warmup + args.steps):
        dt, units, desc, kind = cpu_reference_step(primary, threads)
        if i >= args.warmup:
            secs.append(dt)
    t = statistics.median(secs)
    value = units / t / scale
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64 accumulate / f32", "data": "synthetic (seeded, oracle generator)",
            "impl": "reference", "config": config_of(primary),
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": kind, "sample": desc},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "workloads": {n: dict(cpu_baseline(CONFIGS[n], threads), config=config_of(CONFIGS[n]))
                          for n in names[1:]}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------- our arm

def run_e2e(wl, steps, world, dist):
    """End-to-end steps through the public op (the fused C-ABI call): every step copies its inputs
    host -> device from pinned memory, runs the op and copies its output device -> host.  Steps are
    pipelined the way a serving loop runs them: two device buffer sets, the upload of step i+1 and
    the download of step i-1 on their own streams while step i computes; the `steps` steps are
    captured once into a CUDA graph (copies included) and the replay is timed, so host launch
    overhead does not stand in for the device's work.  Returns (ms for `steps` steps, H2D bytes per
    step, D2H bytes per step, how it ran)."""
    import torch
    dev_in0, dev_out0 = wl.e2e_inputs()
    h_in = [t.cpu().pin_memory() for t in dev_in0]
    bufs = [(list(dev_in0), dev_out0), ([torch.empty_like(t) for t in dev_in0], torch.empty_like(dev_out0))]
    h_out = [torch.empty(dev_out0.shape, dtype=dev_out0.dtype).pin_memory() for _ in range(2)]
    s_up, s_cmp, s_down = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_up = [torch.cuda.Event() for _ in range(2)]
    ev_cmp = [torch.cuda.Event() for _ in range(2)]
    ev_down = [torch.cuda.Event() for _ in range(2)]

    def step(i):
        b = i % 2
        ins, out = bufs[b]
        with torch.cuda.stream(s_up):
            if i >= 2:
                s_up.wait_event(ev_cmp[b])  # step i-2 has finished reading these inputs
            for h, d in zip(h_in, ins):
                d.copy_(h, non_blocking=True)
            ev_up[b].record(s_up)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ev_up[b])
            if i >= 2:
                s_cmp.wait_event(ev_down[b])  # step i-2's output has been read back
            wl.e2e_compute(ins, out)
            ev_cmp[b].record(s_cmp)
        with torch.cuda.stream(s_down):
            s_down.wait_event(ev_cmp[b])
            h_out[b].copy_(out, non_blocking=True)
            ev_down[b].record(s_down)

    def run_steps(n, origin):
        # fork the three streams from `origin`, run n steps, join them back into `origin`
        e0 = torch.cuda.Event()
        e0.record(origin)
        for st in (s_up, s_cmp, s_down):
            st.wait_event(e0)
        for i in range(n):
            step(i)
        for st in (s_up, s_cmp, s_down):
            e = torch.cuda.Event()
            e.record(st)
            origin.wait_event(e)

    origin = torch.cuda.Stream()
    run_steps(3, origin)  # warm-up (also sets kernel attributes before any capture)
    torch.cuda.synchronize()
    graph, mode = None, "graph replay of the pipelined steps"
    try:  # capturing executes nothing (collectives included)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(origin):
            graph.capture_begin()
            run_steps(steps, origin)
            graph.capture_end()
        ok = 1
    except Exception as e:  # capture is an optimisation of the host side only; run eagerly instead
        graph, mode, ok = None, f"eager pipelined steps (graph capture failed: {type(e).__name__})", 0
    torch.cuda.synchronize()
    if world > 1:  # every rank must run the same collectives: graph only if all captured
        flag = torch.tensor([ok], dtype=torch.int32, device=dev_out0.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) == 0 and graph is not None:
            graph, mode = None, "eager pipelined steps (graph capture failed on another rank)"
    if graph is not None:
        with torch.cuda.stream(origin):
            graph.replay()  # warm replay
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        align = torch.zeros(1, device=dev_out0.device)
        with torch.cuda.stream(origin):
            dist.all_reduce(align)
    torch.cuda.synchronize()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(origin)
    if graph is not None:
        with torch.cuda.stream(origin):
            graph.replay()
    else:
        run_steps(steps, origin)
    x1.record(origin)
    torch.cuda.synchronize()
    ms = x0.elapsed_time(x1)
    del graph
    h2d = sum(t.numel() * t.element_size() for t in h_in)
    d2h = dev_out0.numel() * dev_out0.element_size()
    return ms, h2d, d2h, mode


def measure(wl, cfg, K, W, ctx):
    """Warm-up, parity, timed region, dominant kernel and e2e of one workload on every rank; returns
    this workload's report (complete on rank 0)."""
    import torch
    dist, world, rank, local, device, ops = (ctx[k] for k in ("dist", "world", "rank", "local", "device", "ops"))
    stream = torch.cuda.current_stream()
    for i in range(max(W, 3)):  # also sets kernel attributes before any capture
        wl.step(i)
    torch.cuda.synchronize()
    ops.device_status()
    parity = wl.parity()
    if world > 1:
        ok = torch.tensor([1 if parity["ok"] else 0], dtype=torch.int32, device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        parity["ok_all_ranks"] = bool(ok.item())
        worst = torch.tensor([parity["max_abs"], parity["mean_abs"]], dtype=torch.float64, device=device)
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
        parity["max_abs_all_ranks"], parity["mean_abs_all_ranks"] = (float(x) for x in worst.tolist())

    # graphs of G steps (whole rotations of the input sets); K steps = whole replays + a tail graph.
    # Capturing is an optimisation of the host side only: if it fails on any rank, every rank runs
    # the steps eagerly, so that all ranks take the same collectives.
    G = wl.R * max(1, math.ceil(16 / wl.R))
    graphs = {}

    def graph_for(n):
        if n not in graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(n):
                    wl.step(i)
            graphs[n] = g
        return graphs[n]

    full, tail = divmod(K, G)
    try:
        if full:
            graph_for(G)
        if tail:
            graph_for(tail)
        captured = 1
    except Exception:
        graphs.clear()
        captured = 0
    torch.cuda.synchronize()
    if world > 1:
        flag = torch.tensor([captured], dtype=torch.int32, device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        captured = int(flag.item())
    if not captured:
        graphs.clear()
    use_graph = bool(captured)
    if use_graph:  # a warm replay of each graph before the timed region
        for g in graphs.values():
            g.replay()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.sample()
    sampler.start()
    if world > 1:
        # Line the ranks' streams up on the device: a rank whose host reaches this point later
        # would otherwise hold the others' first exchange, and that wait would count as their step.
        align = torch.zeros(1, device=device)
        dist.all_reduce(align)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    if use_graph:
        for _ in range(full):
            graphs[G].replay()
        if tail:
            graphs[tail].replay()
    else:
        for i in range(K):
            wl.step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.finish()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    ms_t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    ops.device_status()
    for g in list(graphs.values()):
        del g
    graphs.clear()
    torch.cuda.synchronize()

    # dominant kernel: events around each of its launches, queued behind a GPU sleep
    M = min(max(K, 8), 30)
    spans, work = [], 0
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e8))

    def record(fn):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        spans.append((a, b))

    for i in range(M):
        work += wl.dominant_launches(i, record)
    torch.cuda.synchronize()
    kern_ms_total = sum(a.elapsed_time(b) for a, b in spans)
    kern_ms = kern_ms_total / len(spans)

    # end to end through the fused C-ABI call, host buffers, copies inside the timed region
    KE = min(K, 50 if wl.kind != "prefill" else 20)
    e2e_ms, h2d_bytes, d2h_bytes, e2e_mode = run_e2e(wl, KE, world, dist)
    e2e_t = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_t.item())

    pk, pk_src = peaks()
    _, bound = wl.roofline_work()
    metric, unit, scale = metric_of(cfg)
    achieved = work / (kern_ms_total * 1e-3) / scale
    peak = pk["bf16_tflops"] if bound == "tensor" else pk["hbm_gbs"]
    tot = torch.tensor([float(wl.units), float(wl.tokens)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(tot)
    total_units, toks = (float(x) for x in tot.tolist())
    value = total_units * K / (ms_max * 1e-3) / scale
    e2e_value = total_units * KE / (e2e_ms * 1e-3) / scale
    rep = {
        "metric": metric, "value": value, "unit": unit, "ms_per_step": ms_max / K, "steps": K,
        "scaling": "weak" if wl.sharding == "replica" else "strong",
        "parallelism": f"{wl.sharding} x{world}", "tokens_per_s": toks * K / (ms_max * 1e-3),
        "l2": f"{wl.R} rotating input sets ({'graph replay' if use_graph else 'stream'}), > 2x L2 between reuses",
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s" if bound == "tensor" else "GB/s", "frac": achieved / peak,
                     "traffic": NCU_TRAFFIC_BYTES.get(cfg.name) if world == 1 else None,
                     "kernel": wl.kernel_name, "kernel_ms": kern_ms, "launches_timed": len(spans),
                     "peak_source": f"{pk_src} ({'bf16_tflops burst' if bound == 'tensor' else 'hbm_gbs'})"},
        "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
                "mode": e2e_mode, "steps": KE, "path": "fused C-ABI call, pinned host buffers"},
        "gpu_launches": K * wl.launches_per_step, "clocks": clocks, "parity": parity,
    }
    if bound == "tensor":
        rep["roofline"]["frac_of_sustained"] = achieved / pk["bf16_tflops_sustained"]
    if wl.kind == "decode" and getattr(wl, "kv_split", False):
        rep["exchange"] = wl.exchange
    if rank == 0 and world == 1:
        rep["cpu_baseline"] = cpu_baseline(cfg, os.cpu_count() or 1)
    return rep


def run_ours(args, names):
    import torch
    import torch.distributed as dist
    from apex_b200 import ops

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py: no CUDA device")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=180))
    ctx = dict(dist=dist, world=world, rank=rank, local=local, device=device, ops=ops)

    reports = {}
    for j, name in enumerate(names):
        cfg = CONFIGS[name]
        K = args.steps if j == 0 else min(args.steps, 50 if cfg.kind != "prefill" else 20)
        wl = {"prefill": PrefillWorkload, "decode": DecodeWorkload, "proj": ProjWorkload}[cfg.kind](cfg, device, rank,
                                                                                                  world)
        try:
            reports[name] = measure(wl, cfg, K, args.warmup, ctx)
        finally:
            torch.cuda.synchronize()
            wl.close()
            if world > 1:
                dist.barrier()
            del wl
            torch.cuda.empty_cache()

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    p = reports[names[0]]
    cfg = CONFIGS[names[0]]
    line = {
        "metric": p["metric"], "value": p["value"], "unit": p["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": p["ms_per_step"], "higher_is_better": True,
        "scaling": p["scaling"], "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded randn on device)",
        "config": config_of(cfg), "parallelism": p["parallelism"], "tokens_per_s": p["tokens_per_s"],
        "l2": p["l2"], "roofline": p["roofline"], "e2e": p["e2e"], "gpu_launches": p["gpu_launches"],
        "clocks": p["clocks"], "cpu_baseline": p.get("cpu_baseline"), "parity": p["parity"],
    }
    if "exchange" in p:
        line["exchange"] = p["exchange"]
    line["workloads"] = {n: dict(r, config=config_of(CONFIGS[n])) for n, r in reports.items() if n != names[0]}
    print(json.dumps(line), flush=True)
    bad = [n for n, r in reports.items() if not r["parity"].get("ok_all_ranks", r["parity"]["ok"])]
    if bad:
        print(f"bench.py: parity check failed for {', '.join(bad)}", file=sys.stderr, flush=True)
        return 1
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=PRIMARY, choices=sorted(CONFIGS))
    ap.add_argument("--also", default=",".join(ALSO),
                    help="comma-separated workloads also measured in this run ('none' for only the primary)")
    args = ap.parse_args(argv)
    also = [] if args.also in ("", "none") else [n for n in args.also.split(",") if n != args.workload]
    for n in also:
        if n not in CONFIGS:
            raise SystemExit(f"unknown workload {n}")
    names = [args.workload] + also
    if args.impl == "reference":
        return run_reference(args, names)
    return run_ours(args, names)


if __name__ == "__main__":
    sys.exit(main())
