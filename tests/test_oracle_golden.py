"""The CPU oracle against fixtures produced by the reference's own trunk code.

``tests/golden/trimul_golden.npz`` was made by ``tests/golden/make_golden.py`` running
``esmfold2_mlx.mlx_trunk`` / ``mlx_trunk_kernels`` unmodified (MLX primitives restated over
numpy).  Both sides compute in fp32 with the same fp16 rounding points, so they differ only
where a different fp32 summation order flips an fp16 rounding: the tolerances below allow a
couple of fp16 ulps at the tensor's scale, on a few percent of the elements (one flipped
rounding of a contraction output spreads through the channel LayerNorm that follows it).
"""

from __future__ import annotations

import ast
import os

import numpy as np
import pytest
import torch

from esmfold2_mlx_b200.synthetic import FoldingTrunk
from oracle import trimul_oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
# c_z = c = 128 (the BASELINE configurations) and 256 (the released trunk, mlx_trunk.py:4)
FILES = {128: ("trimul_golden.npz", ("B1L20", "B2L13")), 256: ("trimul_golden_cz256.npz", ("B1L12", "B2L7"))}


@pytest.fixture(scope="module", params=sorted(FILES), ids=lambda w: f"cz{w}")
def gold(request):
    name, tags = FILES[request.param]
    d = np.load(os.path.join(GOLDEN, name))
    meta = ast.literal_eval(bytes(d["meta"]).decode())
    assert meta["c_z"] == request.param
    trunk = FoldingTrunk(1, meta["c_z"], meta["c"], hidden=meta["hidden"], seed=0)
    sd = {k[2:]: torch.from_numpy(d[k].astype(np.float32)) for k in d.files if k.startswith("w/")}
    trunk.load_state_dict(sd)
    return d, trunk, {**meta, "tags": tags}


def _ulp16(x: torch.Tensor) -> torch.Tensor:
    """Spacing of fp16 numbers at |x| (>= the subnormal spacing)."""
    ax = x.abs().clamp_min(2.0**-14)
    return 2.0 ** (torch.floor(torch.log2(ax)) - 10)


def _close16(ref: np.ndarray, test: torch.Tensor, max_ulps: float, frac_off: float = 1.0,
             rel_l2: float = 1e-3):
    """``|test - ref| <= max_ulps`` fp16 ulps at the tensor's scale (the spacing of fp16
    numbers at max|ref|), at most ``frac_off`` of the elements differ at all, and the
    relative L2 error is below ``rel_l2``.  Chained steps (a whole block) re-round inputs that
    already differ by an ulp, so only the single-step tests bound ``frac_off``."""
    ref_t = torch.from_numpy(ref.astype(np.float32))
    diff = (test.float() - ref_t).abs()
    scale = float(_ulp16(ref_t.abs().max()))
    assert torch.isfinite(test).all()
    assert float(diff.max()) <= max_ulps * scale, f"max diff {float(diff.max()):.3g} > {max_ulps} x {scale:.3g}"
    off = float((diff > 0).float().mean())
    assert off <= frac_off, f"{off:.4f} of elements differ"
    err = float(diff.norm() / ref_t.norm())
    assert err <= rel_l2, f"rel L2 {err:.3g}"


@pytest.mark.parametrize("case", [0, 1])
@pytest.mark.parametrize("direction", ["out", "in"])
@pytest.mark.parametrize("mname", ["nomask", "mask"])
def test_trimul_matches_reference_code(gold, case, direction, mname):
    d, trunk, meta = gold
    tag = meta["tags"][case]
    blk = trunk.blocks[0]
    p = orc.trimul_params(getattr(blk, "tri_mul_" + direction), fp16=True)
    z = torch.from_numpy(d[f"z/{tag}"].astype(np.float32))
    mask = torch.from_numpy(d[f"mask/{tag}"].astype(np.float32)) if mname == "mask" else None
    z2 = orc.trimul_fp16(p, z, mask, direction == "out", meta["mix_eps16"])
    _close16(d[f"tm_{direction}_{mname}/{tag}/z"], z2, max_ulps=2, frac_off=0.05)
    # the fused kernel's second output: LayerNorm of the rounded residual for the next op
    nxt = blk.tri_mul_in._engine.norm_start if direction == "out" else blk.pair_transition.norm
    n2 = orc.r16(orc.layer_norm(z2, orc.r16(nxt.weight.detach()), orc.r16(nxt.bias.detach()), orc.EPS))
    _close16(d[f"tm_{direction}_{mname}/{tag}/n_next"], n2, max_ulps=2, frac_off=0.05)


@pytest.mark.parametrize("mname", ["nomask", "mask"])
def test_trunk16_matches_reference_code(gold, mname):
    d, trunk, meta = gold
    params = orc.trunk_params(trunk, fp16=True)
    z = torch.from_numpy(d[f"z/{meta['tags'][0]}"].astype(np.float32))
    mask = torch.from_numpy(d[f"mask/{meta['tags'][0]}"].astype(np.float32)) if mname == "mask" else None
    out = orc.trunk_fp16(params, z, mask, meta["mix_eps16"])
    _close16(d[f"trunk16_{mname}/{meta['tags'][0]}"], out, max_ulps=4, rel_l2=1e-3)


def test_unfused_trunk_is_close_to_fused(gold):
    """The reference's unfused fp16 path (plain MLX ops) rounds more often than the fused
    one; the oracle follows the fused path and stays within fp16 noise of the unfused one."""
    d, trunk, meta = gold
    params = orc.trunk_params(trunk, fp16=True)
    z = torch.from_numpy(d[f"z/{meta['tags'][0]}"].astype(np.float32))
    mask = torch.from_numpy(d[f"mask/{meta['tags'][0]}"].astype(np.float32))
    out = orc.trunk_fp16(params, z, mask, meta["mix_eps16"])
    ref = torch.from_numpy(d[f"trunk16_unfused_mask/{meta['tags'][0]}"])
    st = orc.error_stats(ref, out)
    assert st["rel_l2"] < 5e-3 and st["max_abs"] < 0.1, st


def test_trunk32_matches_reference_code(gold):
    d, trunk, meta = gold
    blk = trunk.blocks[0]
    z = torch.from_numpy(d[f"z/{meta['tags'][0]}"].astype(np.float32))
    mask = torch.from_numpy(d[f"mask/{meta['tags'][0]}"].astype(np.float32))
    p32o = orc.trimul_params(blk.tri_mul_out, fp16=False)
    p32i = orc.trimul_params(blk.tri_mul_in, fp16=False)
    zz = orc.trimul_fp32(p32o, z, mask, True)
    zz = orc.trimul_fp32(p32i, zz, mask, False)
    tp = orc.transition_params(blk.pair_transition, fp16=False)
    h = orc.layer_norm(zz, tp["ln_w"], tp["ln_b"], orc.EPS)
    x = h @ tp["w12"]
    x1, x2 = x.chunk(2, -1)
    zz = zz + (x1 * torch.sigmoid(x1) * x2) @ tp["w3"]
    st = orc.error_stats(torch.from_numpy(d[f"trunk32_mask/{meta['tags'][0]}"]), zz)
    assert st["rel_l2"] < 1e-5, st


def test_fp16_scheme_tracks_fp32(gold):
    """The 1/256 pre-scale keeps the fp16 path within fp16 noise of the exact fp32 trunk."""
    d, trunk, meta = gold
    z = torch.from_numpy(d[f"z/{meta['tags'][0]}"].astype(np.float32))
    ref32 = torch.from_numpy(d[f"trunk32_mask/{meta['tags'][0]}"])
    ref16 = torch.from_numpy(d[f"trunk16_mask/{meta['tags'][0]}"])
    st = orc.error_stats(ref32, ref16)
    assert st["rel_l2"] < 5e-3, st
    assert z.shape == ref32.shape
