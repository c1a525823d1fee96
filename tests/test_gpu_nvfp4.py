"""NVFP4 projections and RMSNorm on the GPU (the calls either side of the attention path):
matmul_nvfp4 (shaders/matmul.metal:4-53) and rms_norm_f32 (shaders/norm.metal:36-81) against the
reference's own CPU code (matvecNvfp4Cpu, rmsNormCpu) with the reference's gate, rel-L2 < 1e-5
(src/tests/test_norm.cpp:92, src/tests/dense_mlp.cpp:101), and o_proj with the post-attention norm
fused into its epilogue against the reference's composition of the two."""
from __future__ import annotations

import importlib.util
import pathlib

import numpy as np
import pytest
import torch

import oracle
from apex_b200 import ops
from helpers import golden

pytestmark = pytest.mark.gpu
REL_L2 = 1e-5

_spec = importlib.util.spec_from_file_location("make_goldens", pathlib.Path(__file__).parent / "golden" / "make_goldens.py")
MG = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(MG)


def rel_l2(got, ref):
    _, r = oracle.diff(got, ref)
    return r


def dev_matrix(codes, scales):
    return ops.Nvfp4Matrix(torch.from_numpy(codes.view(np.int32)).cuda(), torch.from_numpy(scales).cuda())


def dev_bf16(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).cuda().view(torch.bfloat16)


def test_matmul_nvfp4_f32_vs_reference_golden():
    codes, scales, x, _ = MG.proj_inputs("nvfp4_matvec")
    c = MG.PROJ_CASES["nvfp4_matvec"]
    W = dev_matrix(codes, scales)
    out = torch.empty(c["tokens"], c["rows"], device="cuda")
    ops.matmul_nvfp4(torch.from_numpy(x).cuda(), W, out, c["tokens"])
    assert rel_l2(out.cpu().numpy(), golden("nvfp4_matvec")) < REL_L2


@pytest.mark.parametrize("rows,n,tokens", [(37, 256, 1), (64, 2816, 1), (100, 2816, 4), (48, 4096, 5), (16, 8192, 9),
                                           (2816, 4096, 1)])
def test_matmul_nvfp4_f32_shapes_vs_oracle(rows, n, tokens):
    codes, scales = oracle.nvfp4_matrix(rows, n, 310 + rows)
    x = np.random.default_rng(rows + n).standard_normal((tokens, n)).astype(np.float32)
    ref = oracle.matvec_nvfp4(codes, scales, x, tokens, rows, n, ref=True)
    out = torch.empty(tokens, rows, device="cuda")
    ops.matmul_nvfp4(torch.from_numpy(x).cuda(), dev_matrix(codes, scales), out, tokens)
    assert rel_l2(out.cpu().numpy(), ref) < REL_L2


def test_matmul_nvfp4_bf16_input_and_output():
    rows, n, tokens = 200, 2816, 3
    codes, scales = oracle.nvfp4_matrix(rows, n, 320)
    xb = oracle.normal_bf16(tokens * n, 320, 1)
    x = oracle.bf16_to_f32(xb).reshape(tokens, n)
    ref = oracle.matvec_nvfp4(codes, scales, x, tokens, rows, n, ref=True)
    W = dev_matrix(codes, scales)
    out32 = torch.empty(tokens, rows, device="cuda")
    ops.matmul_nvfp4(dev_bf16(xb).view(tokens, n), W, out32, tokens)
    assert rel_l2(out32.cpu().numpy(), ref) < REL_L2          # bf16 input is exact: same sums
    out16 = torch.empty(tokens, rows, dtype=torch.bfloat16, device="cuda")
    ops.matmul_nvfp4(dev_bf16(xb).view(tokens, n), W, out16, tokens)
    got = out16.float().cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=2 ** -8, atol=1e-6)  # one bf16 rounding of each output


def test_rms_norm_f32_vs_reference_golden():
    x, w = MG.proj_inputs("rms_norm_rows")
    c = MG.PROJ_CASES["rms_norm_rows"]
    out = torch.empty(c["rows"], c["n"], device="cuda")
    ops.rms_norm(torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda(), dev_bf16(w), out, c["rows"], c["n"], 1e-6)
    assert rel_l2(out.cpu().numpy(), golden("rms_norm_rows")) < REL_L2


def test_oproj_post_norm_fused_vs_reference_golden_and_repeatable():
    codes, scales, x, w = MG.proj_inputs("oproj_post_norm")
    c = MG.PROJ_CASES["oproj_post_norm"]
    W = dev_matrix(codes, scales)
    ws = ops.ProjNormWorkspace(c["rows"], c["tokens"])
    resid = torch.randn(c["tokens"], c["rows"], device="cuda")
    outs = []
    for _ in range(2):  # the workspace counter must be back to zero after every call
        out = torch.empty(c["tokens"], c["rows"], device="cuda")
        h = torch.empty_like(out)
        ops.matmul_nvfp4_rms_norm(torch.from_numpy(x).cuda(), W, dev_bf16(w), out, c["tokens"], 1e-6, ws, resid, h)
        ops.device_status()
        outs.append(out.cpu().numpy())
        assert rel_l2(outs[-1], golden("oproj_post_norm")) < REL_L2
        np.testing.assert_allclose(h.cpu().numpy(), resid.cpu().numpy() + outs[-1], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.parametrize("tokens", [1, 7, 16, 20])
def test_oproj_post_norm_token_counts(tokens):
    """Up to 16 tokens: one launch (the last CTA normalises); more: projection + norm launches."""
    rows, n = 2816, 4096
    codes, scales = oracle.nvfp4_matrix(rows, n, 330)
    xb = oracle.normal_bf16(tokens * n, 330 + tokens, 1)
    x = oracle.bf16_to_f32(xb).reshape(tokens, n)
    w = oracle.normal_bf16(rows, 330, 4, 0, 1.0, 0.1)
    ref = oracle.rms_norm_rows(oracle.matvec_nvfp4(codes, scales, x, tokens, rows, n, ref=True), w, tokens, rows, 1e-6,
                               ref=True)
    out = torch.empty(tokens, rows, device="cuda")
    ws = ops.ProjNormWorkspace(rows, tokens)
    ops.matmul_nvfp4_rms_norm(dev_bf16(xb).view(tokens, n), dev_matrix(codes, scales), dev_bf16(w), out, tokens, 1e-6, ws)
    ops.device_status()
    assert rel_l2(out.cpu().numpy(), ref) < REL_L2


@pytest.mark.parametrize("shapes,n,tokens,bf16", [
    (((4096, 1), (2048, 1), (2048, 1)), 2816, 1, True),     # q, k, v of a sliding layer (bf16 in and out)
    (((64, 1), (48, 1), (37, 1)), 256, 1, False),           # ragged last tiles, one stage per matrix
    (((100, 1), (64, 1)), 2816, 4, False),                  # several tokens
    (((40, 1), (24, 1), (16, 1), (8, 1)), 96, 3, False),   # rows not filling tiles at n % 256 != 0: one launch each
])
def test_matmul_nvfp4_multi_equals_single_calls(shapes, n, tokens, bf16):
    """One launch over several matrices of the same input writes what one apex_matmul_nvfp4 per
    matrix writes (same per-row sums in the same order: bit-identical), and the f32 outputs meet the
    oracle."""
    mats = [oracle.nvfp4_matrix(r, n, 500 + i) for i, (r, _) in enumerate(shapes)]
    x = np.random.default_rng(n + tokens).standard_normal((tokens, n)).astype(np.float32)
    dt = torch.bfloat16 if bf16 else torch.float32
    xd = torch.from_numpy(x).cuda().to(dt)
    Ws = [dev_matrix(c, s) for c, s in mats]
    multi = [torch.full((tokens, r), float("nan"), dtype=dt, device="cuda") for r, _ in shapes]
    single = [torch.empty((tokens, r), dtype=dt, device="cuda") for r, _ in shapes]
    ops.matmul_nvfp4_multi(xd, Ws, multi, tokens)
    for W, o in zip(Ws, single):
        ops.matmul_nvfp4(xd, W, o, tokens)
    torch.cuda.synchronize()
    ops.device_status()
    for (r, _), (c, s), a, b in zip(shapes, mats, multi, single):
        assert torch.equal(a.view(torch.int16) if bf16 else a, b.view(torch.int16) if bf16 else b)
        if not bf16:
            ref = oracle.matvec_nvfp4(c, s, x, tokens, r, n, ref=True)
            assert rel_l2(a.cpu().numpy(), ref) < REL_L2


@pytest.mark.parametrize("rows,n,tokens", [(128, 256, 32), (200, 2816, 100), (1024, 4096, 256), (512, 2816, 300),
                                           (64, 512, 513)])
def test_matmul_nvfp4_tensor_core_form_vs_oracle(rows, n, tokens):
    """bf16 input from 32 tokens runs on tcgen05 (weights dequantised exactly to bf16 in shared memory,
    f32 accumulation in TMEM): the reference's gate against the oracle on the same bf16 values, for
    full and ragged row / token tiles, f32 and bf16 output."""
    codes, scales = oracle.nvfp4_matrix(rows, n, 700 + rows)
    xb = oracle.normal_bf16(tokens * n, 700 + tokens, 1)
    x = oracle.bf16_to_f32(xb).reshape(tokens, n)
    ref = oracle.matvec_nvfp4(codes, scales, x, tokens, rows, n, ref=True)
    W = dev_matrix(codes, scales)
    xd = dev_bf16(xb).view(tokens, n)
    out32 = torch.full((tokens, rows), float("nan"), device="cuda")
    ops.matmul_nvfp4(xd, W, out32, tokens)
    torch.cuda.synchronize()
    ops.device_status()
    assert rel_l2(out32.cpu().numpy(), ref) < REL_L2
    out16 = torch.empty(tokens, rows, dtype=torch.bfloat16, device="cuda")
    ops.matmul_nvfp4(xd, W, out16, tokens)
    # one bf16 rounding of each output; the absolute term covers f32 sums that cancel to near zero
    np.testing.assert_allclose(out16.float().cpu().numpy(), ref, rtol=2 ** -8, atol=4e-6 * np.abs(ref).max())
