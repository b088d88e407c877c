"""GPU parity on the exact inputs the benchmark times (``synthetic.workload``, the configurations
``bench.py`` runs), against the CPU oracle.

Tolerance (as in ``test_gpu_parity.py``): with e_ref the fp16 oracle's error against the exact
float64 update and e_cuda the CUDA error against the same, e_cuda <= 2 e_ref + 1e-3 in max-abs
and in relative L2, and |cuda - oracle| <= 4 fp16 ulps at the tensor's scale.  Each direction is
checked on the same input for both sides (the incoming update takes the CUDA outgoing result),
so errors do not compound across the two updates.

Lengths whose whole update is too slow for the CPU oracle (L = 2048 and config 5's L = 3072,
which a single B200 holds in full) are checked on slabs of rows (``oracle.trimul_rows``):
outgoing rows need a's rows and all of b, incoming rows a's columns and all of b.  The slabs
straddle a 128-position tile edge and include the last row.  At c_z = 256 the L = 2048 case
runs the wide kernels' tile choice for grids of 512 x 512 positions and up.
"""

from __future__ import annotations

import pytest
import torch

from esmfold2_mlx_b200 import ops
from esmfold2_mlx_b200.synthetic import workload
from oracle import trimul_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"
ULPS = 4.0


def _params(wl, d, fp16=True):
    return orc.trimul_params(getattr(wl.trunk.blocks[0], "tri_mul_" + d), fp16, wl.biases[d])


def _weights(wl, d):
    return ops.TrimulWeights.from_module(getattr(wl.trunk.blocks[0], "tri_mul_" + d), DEV, wl.biases[d])


def _assert_parity(exact, ref16, got, what):
    par = orc.parity(exact, ref16, got)
    assert par["within_tolerance"], (what, par)
    assert par["max_ulps"] <= ULPS, (what, par)
    return par


def _gpu_pair(wl, dtype=torch.float32):
    """The benchmark's step on the GPU: out then in, returning both results on the CPU."""
    z = wl.z.to(DEV)
    m = None if wl.mask is None else wl.mask.to(DEV)
    ws = ops.Workspace()
    z1 = ops.trimul(z, m, _weights(wl, "out"), True, workspace=ws)
    z2 = ops.trimul(z1, m, _weights(wl, "in"), False, workspace=ws) if "in" in wl.cfg.directions else None
    torch.cuda.synchronize()
    assert ops.read_status(ws.status) == (0, 0)
    return z1.cpu().to(dtype), None if z2 is None else z2.cpu().to(dtype)


def _full_check(wl, folds=slice(None)):
    z = wl.z.float()
    m = None if wl.mask is None else wl.mask.float()
    z1, z2 = _gpu_pair(wl)
    steps = [("out", True, z, z1)] + ([("in", False, z1, z2)] if z2 is not None else [])
    for d, outgoing, zin, got in steps:
        zin_f, m_f = zin[folds], None if m is None else m[folds]
        ref16 = orc.trimul_fp16(_params(wl, d), zin_f, m_f, outgoing)
        exact = orc.trimul_fp32(_params(wl, d, False), zin_f.double(), m_f, outgoing, dtype=torch.float64)
        _assert_parity(exact, ref16, got[folds], f"{wl.cfg.name} {d}")


def test_config1_L76_outgoing():
    _full_check(workload("c1"))


def test_config2_L238_out_in_mask_bias():
    _full_check(workload("c2"))


def test_config2_wide_cz256():
    _full_check(workload("c2w"))


def test_config4_64_folds_L146():
    """All 64 folds against the fp16 oracle in ulps; the exact-error rule on 16 of them."""
    wl = workload("c4")
    z = wl.z.float()
    z1, z2 = _gpu_pair(wl)
    for d, outgoing, zin, got in (("out", True, z, z1), ("in", False, z1, z2)):
        p16 = _params(wl, d)
        for f0 in range(0, wl.cfg.B, 16):
            ref16 = orc.trimul_fp16(p16, zin[f0:f0 + 16], None, outgoing)
            assert orc.ulps16(ref16, got[f0:f0 + 16]) <= ULPS, (d, f0)
        sel = list(range(8)) + list(range(wl.cfg.B - 8, wl.cfg.B))
        ref16 = orc.trimul_fp16(p16, zin[sel], None, outgoing)
        exact = orc.trimul_fp32(_params(wl, d, False), zin[sel].double(), None, outgoing, dtype=torch.float64)
        _assert_parity(exact, ref16, got[sel], f"c4 {d}")


def _slab_check(name, slabs):
    wl = workload(name)
    z1, z2 = _gpu_pair(wl, torch.float16)  # fp16 on the host: config 5's tensors are 2.4 GB each
    ranges = [range(r0, r1) for r0, r1 in slabs(wl.cfg.L)]
    for d, outgoing, zin, got in (("out", True, wl.z, z1), ("in", False, z1, z2)):
        ref16 = orc.trimul_rows(_params(wl, d), zin, None, outgoing, ranges)
        exact = orc.trimul_rows(_params(wl, d, False), zin, None, outgoing, ranges, exact=True)
        for rows, r, e in zip(ranges, ref16, exact):
            _assert_parity(e, r, got[:, rows.start:rows.stop].float(), f"{name} {d} rows {rows.start}:{rows.stop}")


def _edge_slabs(L):
    return [(124, 132), (L - 3, L)]


def test_L2048_row_slabs():
    _slab_check("L2048", _edge_slabs)


def test_L2048_wide_cz256_row_slabs():
    _slab_check("L2048w", lambda L: [(60, 68), (L - 2, L)])


def test_config5_L3072_on_one_gpu_row_slabs():
    """Config 5's fold on one B200 (the 1-GPU point of its row-sharded runs)."""
    _slab_check("c5", lambda L: [(1532, 1540), (L - 2, L)])


def test_config3_one_recycle_of_the_16_block_trunk():
    """One pass of config 3's 16-block stack (ReLU transition) through the public module,
    against the oracle trunk: relative L2 within 2e-3 and distogram agreement p95 < 0.1 Å."""
    from esmfold2_mlx_b200.synthetic import recycle_workload
    from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk

    cfg, trunk, z0 = recycle_workload("c3")
    mod = CUDAFoldingTrunk(trunk, check_status="sync")
    got = mod(z0.to(DEV)).cpu()
    ref = orc.trunk_fp16(orc.trunk_params(trunk, True), z0, None, activation="relu")
    st = orc.error_stats(ref, got)
    assert st["finite"] and st["rel_l2"] < 2e-3, st
    g = torch.Generator().manual_seed(12)
    head_w = torch.randn(128, cfg.c_z, generator=g) / cfg.c_z**0.5
    head_b = 0.1 * torch.randn(128, generator=g)
    assert orc.disto_p95(ref, got, head_w, head_b) < 0.1
