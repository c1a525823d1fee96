"""Packed-weights loader (include/apex_loader.h): the manifest of the reference's checkpoint
layout (src/model_info.h:123-207, tools/repack.py:145-287) parsed and checked against its files,
digests verified, and -- on a GPU -- core.bin and expert slots copied into device memory."""
from __future__ import annotations

import ctypes
import json

import numpy as np
import pytest

import packed_fixture as PF
from apex_b200 import _native


@pytest.fixture()
def packed(tmp_path):
    manifest, tensors, slots = PF.write(tmp_path / "packed")
    return tmp_path / "packed", manifest, tensors, slots


def _open(path):
    lib = _native.load()
    m = ctypes.c_void_p()
    rc = lib.apex_model_open(str(path).encode(), ctypes.byref(m))
    return rc, m, lib


def test_manifest_parsed_like_the_reference(packed):
    path, manifest, tensors, _ = packed
    rc, m, lib = _open(path)
    _native.check(rc)
    try:
        s = _native.ModelSummary()
        _native.check(lib.apex_model_summary_get(m, ctypes.byref(s)))
        tc = PF.TEXT_CONFIG
        assert s.core_size == manifest["core"]["size"] and s.alignment == PF.PAGE
        assert s.core_tensors == len(tensors) and s.layer_files == tc["num_hidden_layers"]
        assert s.expert_slot_size == manifest["layers"][0]["stride"]
        assert (s.hidden_size, s.num_attention_heads, s.num_key_value_heads, s.head_dim) == (64, 4, 2, 16)
        assert (s.global_head_dim, s.num_global_key_value_heads, s.sliding_window) == (32, 1, 8)
        assert (s.quant_group_size, s.quant_bits) == (16, 4)
        assert s.rope_theta_full == 1e6 and abs(s.partial_rotary_factor_full - 0.25) < 1e-7
        for e in manifest["core"]["tensors"]:
            off, n = ctypes.c_uint64(), ctypes.c_uint64()
            _native.check(lib.apex_model_tensor(m, e["name"].encode(), ctypes.byref(off), ctypes.byref(n)))
            assert (off.value, n.value) == (e["offset"], e["nbytes"])
        off, n = ctypes.c_uint64(), ctypes.c_uint64()
        _native.check(lib.apex_model_expert_piece(m, b"down_proj.scales", ctypes.byref(off), ctypes.byref(n)))
        assert (off.value, n.value) == (2048 + 256 + 2048 + 256 + 1536, 200)
        assert lib.apex_model_tensor(m, b"no.such.tensor", ctypes.byref(off), ctypes.byref(n)) == \
            _native.APEX_ERR_INVALID_ARGUMENT
        _native.check(lib.apex_model_verify(m))   # SHA-256 of every tensor and slot (hashlib wrote them)
    finally:
        lib.apex_model_close(m)


def test_verify_names_the_corrupted_tensor_and_slot(packed):
    path, manifest, _, _ = packed
    ent = next(e for e in manifest["core"]["tensors"] if e["name"] == "layers.1.self_attn.q_proj.weight")
    with open(path / "core.bin", "r+b") as f:
        f.seek(ent["offset"] + 5)
        b = f.read(1)
        f.seek(ent["offset"] + 5)
        f.write(bytes([b[0] ^ 1]))
    rc, m, lib = _open(path)
    _native.check(rc)
    try:
        assert lib.apex_model_verify(m) == _native.APEX_ERR_FORMAT
        assert b"layers.1.self_attn.q_proj.weight" in lib.apex_cuda_last_error()
    finally:
        lib.apex_model_close(m)
    with open(path / "core.bin", "r+b") as f:   # restore; break expert 3 of layer 1 instead
        f.seek(ent["offset"] + 5)
        f.write(b)
    stride = manifest["layers"][1]["stride"]
    with open(path / "layer_01.bin", "r+b") as f:
        f.seek(3 * stride + 100)
        c = f.read(1)
        f.seek(3 * stride + 100)
        f.write(bytes([c[0] ^ 0x80]))
    rc, m, lib = _open(path)
    _native.check(rc)
    try:
        assert lib.apex_model_verify(m) == _native.APEX_ERR_FORMAT
        assert b"layer_01.bin expert 3" in lib.apex_cuda_last_error()
    finally:
        lib.apex_model_close(m)


def _rewrite(path, fn):
    man = json.loads((path / "manifest.json").read_text())
    fn(man)
    (path / "manifest.json").write_text(json.dumps(man))


@pytest.mark.parametrize("breakage,needle", [
    (lambda m: m["core"].__setitem__("size", m["core"]["size"] + 1), b"core.bin is"),
    (lambda m: m["core"]["tensors"][0].__setitem__("offset", 8), b"not a multiple of the alignment"),
    (lambda m: m["core"]["tensors"][-1].__setitem__("offset", m["core"]["size"]), b"beyond the end"),
    (lambda m: m["core"]["tensors"][0].__setitem__("nbytes", m["core"]["tensors"][0]["nbytes"] - 2), b"manifest says"),
    (lambda m: m["text_config"].pop("head_dim"), b"missing key 'head_dim'"),
    (lambda m: m["layers"][0].__setitem__("stride", m["layers"][0]["stride"] * 2), b"num_experts x stride"),
    (lambda m: m["layers"][0]["pieces"][5].__setitem__("nbytes", 1 << 20), b"beyond the slot"),
])
def test_inconsistent_manifests_are_rejected(packed, breakage, needle):
    path = packed[0]
    _rewrite(path, breakage)
    rc, m, lib = _open(path)
    assert rc == _native.APEX_ERR_FORMAT and not m.value
    assert needle in lib.apex_cuda_last_error(), lib.apex_cuda_last_error()


def test_missing_or_malformed_manifest(tmp_path):
    rc, m, lib = _open(tmp_path)
    assert rc == _native.APEX_ERR_FORMAT and b"cannot open" in lib.apex_cuda_last_error()
    (tmp_path / "manifest.json").write_text('{"text_config": [1, 2,')
    rc, m, lib = _open(tmp_path)
    assert rc == _native.APEX_ERR_FORMAT and b"json" in lib.apex_cuda_last_error()


@pytest.mark.gpu
def test_upload_core_and_expert_slots_to_device(packed):
    import torch
    path, manifest, tensors, slots = packed
    rc, m, lib = _open(path)
    _native.check(rc)
    try:
        size = manifest["core"]["size"]
        dev = torch.zeros(size, dtype=torch.uint8, device="cuda")
        secs = ctypes.c_double()
        _native.check(lib.apex_model_upload_core(m, dev.data_ptr(), size, 1, torch.cuda.current_stream().cuda_stream,
                                                 ctypes.byref(secs)))
        host = dev.cpu().numpy()
        want = np.fromfile(path / "core.bin", dtype=np.uint8)
        assert np.array_equal(host, want)
        for e in manifest["core"]["tensors"]:   # device base + manifest offset addresses the tensor
            assert host[e["offset"]:e["offset"] + e["nbytes"]].tobytes() == tensors[e["name"]][2]
        assert lib.apex_model_upload_core(m, dev.data_ptr(), size - 1, 0, None, None) == _native.APEX_ERR_FORMAT
        stride = manifest["layers"][0]["stride"]
        slot = torch.zeros(stride, dtype=torch.uint8, device="cuda")
        for (layer, e) in ((0, 0), (1, 3)):
            _native.check(lib.apex_model_load_expert(m, layer, e, slot.data_ptr(), stride, 1, None))
            got = slot.cpu().numpy().tobytes()
            assert got[:len(slots[(layer, e)])] == slots[(layer, e)]
        assert lib.apex_model_load_expert(m, 2, 0, slot.data_ptr(), stride, 0, None) == _native.APEX_ERR_FORMAT
    finally:
        lib.apex_model_close(m)
    # a corrupted tensor is caught while it streams to the device
    ent = next(e for e in manifest["core"]["tensors"] if e["name"] == "layers.1.big.weight")
    with open(path / "core.bin", "r+b") as f:
        f.seek(ent["offset"] + (33 << 20))   # in the second staging chunk of the tensor
        f.write(b"\x00\x01\x02")
    rc, m, lib = _open(path)
    _native.check(rc)
    try:
        dev = torch.zeros(manifest["core"]["size"], dtype=torch.uint8, device="cuda")
        rc = lib.apex_model_upload_core(m, dev.data_ptr(), dev.numel(), 1, None, None)
        assert rc == _native.APEX_ERR_FORMAT and b"layers.1.big.weight" in lib.apex_cuda_last_error()
    finally:
        lib.apex_model_close(m)
