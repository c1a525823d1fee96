"""A small synthetic packed checkpoint in the layout the reference's packer writes
(tools/repack.py:1-36): core.bin with every tensor on an `alignment` boundary, layer_NN.bin with
num_experts slots of a fixed page-aligned stride holding the six expert pieces in order, and
manifest.json describing both with a SHA-256 per core tensor and per expert slot.  Test data for
the loader; the real checkpoint is not available here."""
from __future__ import annotations

import hashlib
import json
import pathlib

import numpy as np

PAGE = 16384
EXPERT_PIECES = ("gate_proj.weight", "gate_proj.scales", "up_proj.weight", "up_proj.scales",
                 "down_proj.weight", "down_proj.scales")

TEXT_CONFIG = {
    "hidden_size": 64, "intermediate_size": 48, "moe_intermediate_size": 32, "num_attention_heads": 4,
    "num_key_value_heads": 2, "head_dim": 16, "num_hidden_layers": 2, "num_experts": 4, "top_k_experts": 2,
    "vocab_size": 32, "sliding_window": 8, "rms_norm_eps": 1e-6, "final_logit_softcapping": 30.0,
    "layer_types": ["sliding_attention", "full_attention"], "global_head_dim": 32,
    "num_global_key_value_heads": 1, "attention_k_eq_v": True,
    "rope_parameters": {"sliding_attention": {"rope_theta": 10000.0},
                        "full_attention": {"rope_theta": 1000000.0, "partial_rotary_factor": 0.25}},
}


def _align(n, a=PAGE):
    return (n + a - 1) // a * a


def core_tensors(rng):
    """name -> (dtype, shape, bytes)."""
    H = TEXT_CONFIG["hidden_size"]
    out = {}

    def add(name, dtype, shape, arr):
        out[name] = (dtype, list(shape), np.ascontiguousarray(arr).tobytes())

    add("embed_tokens.weight", "BF16", (32, H), rng.integers(0, 65536, (32, H), dtype=np.uint16))
    add("norm.weight", "BF16", (H,), rng.integers(0, 65536, H, dtype=np.uint16))
    for layer in range(TEXT_CONFIG["num_hidden_layers"]):
        p = f"layers.{layer}."
        add(p + "input_layernorm.weight", "BF16", (H,), rng.integers(0, 65536, H, dtype=np.uint16))
        add(p + "self_attn.q_proj.weight", "U32", (64, H // 8), rng.integers(0, 2**32, (64, H // 8), dtype=np.uint32))
        add(p + "self_attn.q_proj.scales", "U8", (64, H // 16), rng.integers(0, 127, (64, H // 16), dtype=np.uint8))
        add(p + "router.odd", "U8", (3, 7), rng.integers(0, 256, (3, 7), dtype=np.uint8))  # 21 bytes
    # a tensor larger than the loader's 32 MiB staging chunk, spanning chunk boundaries
    add("layers.1.big.weight", "U8", (40 << 20,), rng.integers(0, 256, 40 << 20, dtype=np.uint8))
    return out


def write(dir_: pathlib.Path, seed: int = 0):
    """Writes the checkpoint into dir_; returns (manifest dict, core tensors dict, expert slot bytes)."""
    rng = np.random.default_rng(seed)
    dir_.mkdir(parents=True, exist_ok=True)
    tensors = core_tensors(rng)
    entries, off = [], 0
    with open(dir_ / "core.bin", "wb") as f:
        for name in sorted(tensors):
            dtype, shape, data = tensors[name]
            off = _align(off)
            f.seek(off)
            f.write(data)
            entries.append({"name": name, "dtype": dtype, "shape": shape, "offset": off, "nbytes": len(data),
                            "sha256": hashlib.sha256(data).hexdigest()})
            off += len(data)
        f.truncate(_align(off))
    core_size = (dir_ / "core.bin").stat().st_size
    E = TEXT_CONFIG["num_experts"]
    piece_sizes = {"gate_proj.weight": 2048, "gate_proj.scales": 256, "up_proj.weight": 2048,
                   "up_proj.scales": 256, "down_proj.weight": 1536, "down_proj.scales": 200}
    pieces, po = [], 0
    for name in EXPERT_PIECES:
        n = piece_sizes[name]
        pieces.append({"name": name, "dtype": "U8", "shape": [n], "offset": po, "nbytes": n})
        po += n
    stride = _align(po)
    layers, slots = [], {}
    for layer in range(TEXT_CONFIG["num_hidden_layers"]):
        fname = f"layer_{layer:02d}.bin"
        hashes = []
        with open(dir_ / fname, "wb") as f:
            f.truncate(E * stride)
            for e in range(E):
                blob = rng.integers(0, 256, po, dtype=np.uint8).tobytes()
                f.seek(e * stride)
                f.write(blob)
                hashes.append(hashlib.sha256(blob).hexdigest())
                slots[(layer, e)] = blob
        layers.append({"layer": layer, "file": fname, "size": E * stride, "num_experts": E, "stride": stride,
                       "pieces": pieces, "expert_sha256": hashes})
    manifest = {"version": 1, "alignment": PAGE, "text_config": TEXT_CONFIG,
                "quantization": {"group_size": 16, "bits": 4, "mode": "nvfp4"},
                "core": {"file": "core.bin", "tensors": entries, "size": core_size}, "layers": layers}
    (dir_ / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    return manifest, tensors, slots
