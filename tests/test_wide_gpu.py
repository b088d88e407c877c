"""GPU parity at c_z = c = 256, the pair width of ESMFold2's released trunk (mlx_trunk.py:4).

The wide kernels (the CTA-pair K1P and K3P; K2 is width-agnostic) against the CPU oracle, with the same bounds
as the c_z = 128 tests: kernel outputs within 2 fp16 ulps of the oracle's intermediates (a few %
of elements may differ), whole updates with e_cuda <= 2 e_ref + 1e-3 against the exact float64
update and within 4 ulps of the fp16 oracle.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from esmfold2_mlx_b200 import _lib, ops
from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_mask, pair_tensor, trimul_biases
from oracle import trimul_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"
CZ = 256


def _ulp16(x: float) -> float:
    import math
    x = max(abs(x), 2.0**-14)
    return 2.0 ** (math.floor(math.log2(x)) - 10)


def _setup(L, B=1, seed=0, n_pad=0, biases=False):
    trunk = FoldingTrunk(1, CZ, CZ, hidden=512, seed=seed + 7, ln_noise=0.1)
    z = pair_tensor(B, L, CZ, seed).half().float()
    mask = pair_mask(B, L, n_pad) if n_pad else None
    bias = {d: trimul_biases(CZ, CZ, seed + 31 + i) for i, d in enumerate(("out", "in"))} if biases else None
    return trunk, z, mask, bias


def _w(trunk, direction, bias, fp16=True):
    tri = getattr(trunk.blocks[0], "tri_mul_" + direction)
    b = None if bias is None else bias[direction]
    return ops.TrimulWeights.from_module(tri, DEV, b), orc.trimul_params(tri, fp16, b)


# K1P takes K1's 128-position tile shapes (the least padding below 512 x 512 positions): these
# sizes reach the wide (1 x 128, 2 x 64), square-ish (8 x 16, 16 x 8) and sub-tile (L = 12) cases
@pytest.mark.parametrize("L,B,n_pad,biases", [(64, 1, 0, False), (100, 1, 9, True), (146, 2, 0, False),
                                              (37, 3, 5, True), (12, 2, 3, False), (96, 1, 0, True)])
def test_wide_project_gate_matches_oracle(L, B, n_pad, biases):
    trunk, z, mask, bias = _setup(L, B, seed=L, n_pad=n_pad, biases=biases)
    w, p = _w(trunk, "out", bias)
    _, a_ref, b_ref = orc.project_gate_fp16(p, z, mask)
    a, b = ops.project_gate(z.half().to(DEV), None if mask is None else mask.half().to(DEV), w)
    torch.cuda.synchronize()
    for name, got, ref in (("a", a, a_ref), ("b", b, b_ref)):
        got = got[:, :, :L].float().cpu().reshape(B, CZ, L, L)
        diff = (got - ref).abs()
        assert float(diff.max()) <= 2 * _ulp16(float(ref.abs().max())), f"{name}: {float(diff.max()):.3g}"
        assert float((diff > 0).float().mean()) < 0.05, name
        if mask is not None:
            assert float(got.permute(0, 2, 3, 1)[~mask.bool()].abs().max()) == 0.0


@pytest.mark.parametrize("L,B,biases", [(64, 1, True), (130, 1, False), (90, 2, True)])
def test_wide_emit_residual_matches_oracle(L, B, biases):
    trunk, z, _, bias = _setup(L, B, seed=L + 1, biases=biases)
    w, p = _w(trunk, "in", bias)
    g = torch.Generator().manual_seed(L)
    xg = (torch.randn(B, CZ, L, L, generator=g) * 3).half().float()
    ref, _ = orc.emit_residual_fp16(p, z, xg, ops.MIX_EPS_FP16)
    x = torch.zeros(B * CZ, L, ops.row_pitch(L), dtype=torch.float16)
    x[:, :, :L] = xg.reshape(B * CZ, L, L).half()
    out = ops.emit_residual(x.to(DEV), z.half().to(DEV), w)
    torch.cuda.synchronize()
    diff = (out.float().cpu() - ref).abs()
    assert float(diff.max()) <= 4 * _ulp16(float(ref.abs().max()))


@pytest.mark.parametrize("L,B,n_pad,biases", [(48, 1, 0, False), (130, 1, 11, True), (200, 1, 0, False),
                                              (77, 2, 6, False)])
@pytest.mark.parametrize("outgoing", [True, False])
def test_wide_trimul_matches_oracle(L, B, n_pad, biases, outgoing):
    trunk, z, mask, bias = _setup(L, B, seed=L + 2, n_pad=n_pad, biases=biases)
    direction = "out" if outgoing else "in"
    w, p = _w(trunk, direction, bias)
    _, p32 = _w(trunk, direction, bias, fp16=False)
    ref16 = orc.trimul_fp16(p, z, mask, outgoing)
    exact = orc.trimul_fp32(p32, z.double(), mask, outgoing, dtype=torch.float64)
    zd = z.half().to(DEV)
    out = ops.trimul(zd, None if mask is None else mask.half().to(DEV), w, outgoing)
    torch.cuda.synchronize()
    got = out.float().cpu()
    e_ref, e_got = orc.error_stats(exact, ref16), orc.error_stats(exact, got)
    assert e_got["finite"]
    assert e_got["max_abs"] <= 2 * e_ref["max_abs"] + 1e-3, (e_got, e_ref)
    assert e_got["rel_l2"] <= 2 * e_ref["rel_l2"] + 1e-3, (e_got, e_ref)
    assert float((got - ref16).abs().max()) <= 4 * _ulp16(float(ref16.abs().max()))


def test_wide_in_place_goes_through_second_buffer_and_abi_rejects_alias():
    trunk, z, mask, bias = _setup(70, 1, seed=3, n_pad=4)
    w, _ = _w(trunk, "out", bias)
    zd = z.half().to(DEV)
    m = mask.half().to(DEV)
    ws = ops.Workspace()
    ref = ops.trimul(zd, m, w, True, workspace=ws).clone()
    zz = zd.clone()
    ops.trimul(zz, m, w, True, out=zz, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(zz, ref)
    lib = _lib.load()
    buf = ws.get(1, 70, CZ, CZ, zd.device)
    rc = lib.tmu_trimul(ops._ptr(zz), ops._ptr(zz), ops._ptr(m), ctypes.byref(w.struct), 1, 70, CZ, CZ, 1,
                        ops.MIX_EPS_FP16, ops._ptr(buf), buf.numel(), ops._stream_ptr(zd.device))
    assert _lib.STATUS_NAMES.get(rc) == "TMU_ERR_INVALID_ARGUMENT"
    assert b"overlap" in lib.tmu_last_error()


def test_wide_trunk_module_matches_oracle():
    from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk

    trunk = FoldingTrunk(2, CZ, CZ, hidden=512, seed=3, ln_noise=0.1)
    L = 60
    z = pair_tensor(1, L, CZ, 9)
    mask = pair_mask(1, L, 5)
    ref = orc.trunk_fp16(orc.trunk_params(trunk, True), z, mask)
    out = CUDAFoldingTrunk(trunk)(z.to(DEV), pair_attention_mask=mask.to(DEV))
    st = orc.error_stats(ref, out.cpu())
    assert st["finite"] and st["rel_l2"] < 2e-3, st
