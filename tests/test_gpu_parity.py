"""GPU parity: the sm_100a kernels (through the C ABI) against the CPU oracle.

Tolerance (fp16 path).  Let e_ref be the error of the fp16-emulating oracle against the exact
(float64) update on the same inputs, and e_cuda the CUDA result's error against the same exact
update.  Each test requires  e_cuda.max_abs <= 2 * e_ref.max_abs + 1e-3  and the same for the
relative L2 error, and also bounds the direct CUDA-vs-oracle difference by a few fp16 ulps at the
tensor's scale.  Kernel-level tests (K1, K2, K3 alone) compare with the oracle's intermediates.
"""

from __future__ import annotations

import pytest
import torch

from esmfold2_mlx_b200 import ops
from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_mask, pair_tensor, trimul_biases
from oracle import trimul_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ulp16(x: float) -> float:
    import math
    x = max(abs(x), 2.0**-14)
    return 2.0 ** (math.floor(math.log2(x)) - 10)


def _setup(L, B=1, seed=0, n_pad=0, biases=False, ln_noise=0.1):
    trunk = FoldingTrunk(1, 128, 128, hidden=256, seed=seed + 7, ln_noise=ln_noise)
    z = pair_tensor(B, L, 128, seed).to(torch.float16).float()
    mask = pair_mask(B, L, n_pad) if n_pad else None
    bias = {d: trimul_biases(128, 128, seed + 31 + i) for i, d in enumerate(("out", "in"))} if biases else None
    return trunk, z, mask, bias


def _cuda_w(trunk, direction, bias):
    return ops.TrimulWeights.from_module(getattr(trunk.blocks[0], "tri_mul_" + direction), DEV,
                                         None if bias is None else bias[direction])


def _oracle_p(trunk, direction, bias, fp16=True):
    return orc.trimul_params(getattr(trunk.blocks[0], "tri_mul_" + direction), fp16,
                             None if bias is None else bias[direction])


def _unpad(t, B, c, L):
    return t[:, :, :L].reshape(B, c, L, L).float().cpu()


def test_library_loads_on_b200():
    lib = ops._lib.load()
    ops._lib.check(lib.tmu_device_check(), "tmu_device_check")


def test_bounded_wait_reports_timeout():
    """A device wait on a barrier nothing arrives at gives up and reports, without a fault."""
    lib = ops._lib.load()
    st = ops.new_status(DEV)
    ops._lib.check(lib.tmu_selftest_wait_timeout(ops._ptr(st), 1_000_000, ops._stream_ptr(torch.device(DEV))),
                   "selftest")
    code, site = ops.read_status(st)
    assert code == 6 and site == 0x901
    # the context is still healthy afterwards
    x = torch.ones(16, device=DEV)
    assert float(x.sum()) == 16.0


@pytest.mark.parametrize("L", [64, 76, 130, 146, 238, 256, 300, 384])  # tile widths 128, 192, 256
@pytest.mark.parametrize("outgoing", [True, False])
def test_contract_matches_fp32_bmm(L, outgoing):
    g = torch.Generator().manual_seed(L)
    Bc = 6
    Lp = ops.row_pitch(L)
    a = torch.zeros(Bc, L, Lp, dtype=torch.float16)
    b = torch.zeros(Bc, L, Lp, dtype=torch.float16)
    a[:, :, :L] = torch.randn(Bc, L, L, generator=g).half()
    b[:, :, :L] = torch.randn(Bc, L, L, generator=g).half()
    if Lp > L:  # garbage in the pad columns must never be read
        a[:, :, L:] = 1e4
        b[:, :, L:] = -1e4
    x = ops.contract(a.to(DEV), b.to(DEV), L, outgoing)
    torch.cuda.synchronize()
    A, Bm = a[:, :, :L].double(), b[:, :, :L].double()
    ref = A @ Bm.transpose(1, 2) if outgoing else A.transpose(1, 2) @ Bm
    got = x[:, :, :L].double().cpu()
    err = (got - ref).abs()
    tol = 2 * ref.abs().clamp_min(1.0) * 2.0**-11 + 1e-2
    assert bool((err <= tol).all()), f"max err {float(err.max()):.4g}"
    assert float((got - ref).norm() / ref.norm()) < 1e-3


@pytest.mark.parametrize("L,B,n_pad,biases", [(76, 1, 0, False), (238, 1, 24, True), (146, 2, 10, False)])
def test_project_gate_matches_oracle(L, B, n_pad, biases):
    trunk, z, mask, bias = _setup(L, B, seed=L, n_pad=n_pad, biases=biases)
    p = _oracle_p(trunk, "out", bias)
    _, it = orc.trimul_fp16(p, z, mask, True, return_intermediates=True)
    w = _cuda_w(trunk, "out", bias)
    a, b = ops.project_gate(z.half().to(DEV), None if mask is None else mask.half().to(DEV), w)
    torch.cuda.synchronize()
    for name, got in (("a", a), ("b", b)):
        got = _unpad(got, B, 128, L)
        ref = it[name]
        diff = (got - ref).abs()
        scale = _ulp16(float(ref.abs().max()))
        assert float(diff.max()) <= 2 * scale, f"{name}: max diff {float(diff.max()):.3g}"
        assert float((diff > 0).float().mean()) < 0.05, f"{name}: {float((diff > 0).float().mean()):.3f} differ"
        if mask is not None:  # masked rows/columns are exactly zero
            m = mask.bool()
            assert float(got.permute(0, 2, 3, 1)[~m].abs().max()) == 0.0


# tile shapes: 76, 238 -> 8 x 16; 146 -> 4 x 32; 120 -> 1 x 128 (ragged columns); 59 -> 2 x 64
# (ragged rows and columns); 128 -> 1 x 128 (jw >= 64 loads x as two swizzled halves)
@pytest.mark.parametrize("L,B", [(76, 1), (238, 1), (146, 2), (120, 1), (59, 2), (128, 1)])
@pytest.mark.parametrize("outgoing", [True, False])
def test_emit_residual_matches_oracle(L, B, outgoing):
    trunk, z, mask, bias = _setup(L, B, seed=L + 1, biases=True)
    direction = "out" if outgoing else "in"
    p = _oracle_p(trunk, direction, bias)
    ref_z, it = orc.trimul_fp16(p, z, None, outgoing, return_intermediates=True)
    w = _cuda_w(trunk, direction, bias)
    Lp = ops.row_pitch(L)
    x = torch.zeros(B * 128, L, Lp, dtype=torch.float16)
    x[:, :, :L] = it["x"].reshape(B * 128, L, L).half()
    zin = z.half().to(DEV)
    out = ops.emit_residual(x.to(DEV), zin, w)
    torch.cuda.synchronize()
    got = out.float().cpu()
    diff = (got - ref_z).abs()
    scale = _ulp16(float(ref_z.abs().max()))
    assert float(diff.max()) <= 2 * scale, f"max diff {float(diff.max()):.3g} (ulp {scale:.3g})"
    assert float((diff > 0).float().mean()) < 0.05


def _exact_update(trunk, direction, bias, z, mask, outgoing):
    p = _oracle_p(trunk, direction, bias, fp16=False)
    return orc.trimul_fp32(p, z.double(), mask, outgoing, dtype=torch.float64)


@pytest.mark.parametrize("L,B,n_pad,biases", [(76, 1, 0, False), (238, 1, 24, True), (146, 2, 0, False),
                                              (33, 3, 5, True), (200, 1, 0, False), (120, 1, 8, True),
                                              (59, 2, 3, False), (12, 2, 3, True)])
@pytest.mark.parametrize("outgoing", [True, False])
def test_trimul_matches_oracle(L, B, n_pad, biases, outgoing):
    trunk, z, mask, bias = _setup(L, B, seed=L + 2, n_pad=n_pad, biases=biases)
    direction = "out" if outgoing else "in"
    ref16 = orc.trimul_fp16(_oracle_p(trunk, direction, bias), z, mask, outgoing)
    exact = _exact_update(trunk, direction, bias, z, mask, outgoing)
    w = _cuda_w(trunk, direction, bias)
    out = ops.trimul(z.half().to(DEV), None if mask is None else mask.half().to(DEV), w, outgoing)
    torch.cuda.synchronize()
    got = out.float().cpu()
    e_ref = orc.error_stats(exact, ref16)
    e_cuda = orc.error_stats(exact, got)
    assert e_cuda["finite"]
    assert e_cuda["max_abs"] <= 2 * e_ref["max_abs"] + 1e-3, (e_cuda, e_ref)
    assert e_cuda["rel_l2"] <= 2 * e_ref["rel_l2"] + 1e-3, (e_cuda, e_ref)
    diff = (got - ref16).abs()
    assert float(diff.max()) <= 4 * _ulp16(float(ref16.abs().max()))


def test_trimul_in_place_and_workspace_reuse():
    trunk, z, mask, bias = _setup(96, 1, seed=5, n_pad=7)
    w = _cuda_w(trunk, "out", bias)
    ws = ops.Workspace()
    zd = z.half().to(DEV)
    m = mask.half().to(DEV)
    ref = ops.trimul(zd, m, w, True, workspace=ws).clone()
    zz = zd.clone()
    ops.trimul(zz, m, w, True, out=zz, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(zz, ref)
    code, _ = ops.read_status(ws.status)
    assert code == 0


def test_trunk_module_matches_oracle():
    from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk

    trunk = FoldingTrunk(2, 128, 128, hidden=256, seed=3, ln_noise=0.1)
    L = 70
    z = pair_tensor(1, L, 128, 9)
    mask = pair_mask(1, L, 6)
    ref = orc.trunk_fp16(orc.trunk_params(trunk, True), z, mask)
    mod = CUDAFoldingTrunk(trunk)
    out = mod(z.to(DEV), pair_attention_mask=mask.to(DEV))
    assert out.dtype == torch.float32 and out.device.type == "cuda"
    got = out.cpu()
    st = orc.error_stats(ref, got)
    assert st["finite"] and st["rel_l2"] < 2e-3, st
    # an all-ones mask is skipped, as the reference does
    out1 = mod(z.to(DEV), pair_attention_mask=torch.ones(1, L, L, device=DEV))
    out2 = mod(z.to(DEV))
    assert torch.equal(out1, out2)


def test_invalid_arguments_raise():
    trunk, z, _, _ = _setup(40)
    w = _cuda_w(trunk, "out", None)
    with pytest.raises((TypeError, ValueError)):
        ops.trimul(z.to(DEV), None, w, True)  # fp32 input
    lib = ops._lib.load()
    code = lib.tmu_trimul(None, None, None, None, 1, 40, 128, 128, 1, 1e-5, None, 0, None)
    assert ops._lib.STATUS_NAMES[code] == "TMU_ERR_INVALID_ARGUMENT"
    code = lib.tmu_contract(None, None, None, 1, 40, 1, None, None)
    assert code == 1


def test_trunk_graph_replay_equals_eager_and_is_cached():
    from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk

    trunk = FoldingTrunk(2, 128, 128, hidden=256, seed=4, ln_noise=0.1)
    eager = CUDAFoldingTrunk(trunk, graphs=False)
    graphed = CUDAFoldingTrunk(trunk, graphs=True, max_graphs=2)
    for L, n_pad in ((40, 0), (57, 5), (40, 0), (57, 5)):
        z = pair_tensor(1, L, 128, L).to(DEV)
        mask = pair_mask(1, L, n_pad).to(DEV) if n_pad else None
        a = eager(z, pair_attention_mask=mask)
        b = graphed(z, pair_attention_mask=mask)
        assert torch.equal(a, b)
    assert len(graphed._graph_cache) == 2  # one graph per (shape, mask) seen, reused on repeat
    # a third shape evicts the least recently used one
    z = pair_tensor(1, 33, 128, 1).to(DEV)
    assert torch.equal(eager(z), graphed(z))
    assert len(graphed._graph_cache) == 2


def test_trunk_graph_survives_a_later_capture_and_cache_release():
    """A cached graph's kernels address the workspace of the trunk function it was captured
    with; the cache entry owns that function, so a later capture (which runs gc.collect() and
    empty_cache()) or an explicit empty_cache() cannot hand the workspace back to the driver."""
    from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk

    first = CUDAFoldingTrunk(FoldingTrunk(1, 128, 128, hidden=256, seed=5, ln_noise=0.1))
    second = CUDAFoldingTrunk(FoldingTrunk(2, 128, 128, hidden=256, seed=6, ln_noise=0.1))
    z = pair_tensor(1, 40, 128, 7).to(DEV)
    a = first(z)
    second(z)  # a second capture
    torch.cuda.empty_cache()
    assert torch.equal(first(z), a)
