"""The pair-conditioning and parcae oracles against fixtures produced by the reference's own code.

``tests/golden/conditioning_golden.npz`` was made by ``tests/golden/make_golden_conditioning.py``
running ``esmfold2_mlx.mlx_diffusion16.pair_biases`` and ``esmfold2_mlx.var_6b_mlx_loop._step``
unmodified (MLX primitives restated over numpy).  The pair conditioning runs in fp16 with the
same rounding points on both sides, so outputs differ only where a different fp32 summation
order flips an fp16 rounding; the tolerance is a couple of fp16 ulps at the tensor's scale and a
relative L2 error of 1e-3.  Four LayerNorms are chained (input, two transitions, bias), and each
re-rounds inputs that already differ by an ulp, so a few percent of the outputs differ at all:
the oracle with float64 accumulation differs from itself with float32 accumulation by as much.  The
parcae step is fp32 throughout: the bound is a few fp32 ulps of the output's scale.
"""

from __future__ import annotations

import ast
import os

import numpy as np
import pytest
import torch

from esmfold2_mlx_b200.synthetic import DiffusionHead
from oracle import pair_cond_oracle as pco
from oracle import parcae_oracle as pao

GOLD = os.path.join(os.path.dirname(__file__), "golden", "conditioning_golden.npz")


@pytest.fixture(scope="module")
def gold():
    d = np.load(GOLD)
    meta = ast.literal_eval(bytes(d["meta"]).decode())
    return d, meta


def _ulp16(x: torch.Tensor) -> torch.Tensor:
    ax = x.abs().clamp_min(2.0**-14)
    return 2.0 ** (torch.floor(torch.log2(ax)) - 10)


@pytest.mark.parametrize("name,tag", [("pc", "B1L12"), ("pc", "B2L7"), ("pc2", "B1L64")])
def test_pair_cond_matches_reference_code(gold, name, tag):
    d, meta = gold
    head = DiffusionHead(**meta[name])
    pre = f"{name}_w/"
    head.load_state_dict({k[len(pre):]: torch.from_numpy(d[k]) for k in d.files if k.startswith(pre)})
    p = pco.pair_cond_params(head)
    zt = torch.from_numpy(d[f"{name}/{tag}/z_trunk"]).float()
    rp = torch.from_numpy(d[f"{name}/{tag}/rel_pos"]).float()
    got = pco.pair_biases_fp16(p, zt, rp)
    ref = torch.from_numpy(d[f"{name}/{tag}/bias"].astype(np.float32))
    B, L = zt.shape[:2]
    assert got.shape == ref.shape == (meta[name]["n_blocks"], B, meta[name]["heads"], L, L)
    diff = (got - ref).abs()
    scale = float(_ulp16(ref.abs().max()))
    assert float(diff.max()) <= 2 * scale, f"max diff {float(diff.max()):.3g} > 2 x {scale:.3g}"
    assert float(diff.norm() / ref.norm()) <= 1e-3


@pytest.mark.parametrize("tag", ["B1L9", "B2L5", "B1L20c128"])
def test_parcae_step_matches_reference_code(gold, tag):
    d, _ = gold
    t = {k: torch.from_numpy(d[f"parcae/{tag}/{k}"]) for k in
         ("z", "z_init", "refined", "ln_w", "ln_b", "a", "b_mat", "z_next")}
    got = pao.parcae_step(t["z"], t["z_init"], t["refined"], t["ln_w"], t["ln_b"], t["a"], t["b_mat"])
    ref = t["z_next"]
    assert got.dtype == torch.float32 and got.shape == ref.shape
    tol = 8 * float(torch.finfo(torch.float32).eps) * float(ref.abs().max())
    assert float((got - ref).abs().max()) <= tol
    exact = pao.parcae_step(t["z"], t["z_init"], t["refined"], t["ln_w"], t["ln_b"], t["a"], t["b_mat"],
                            dtype=torch.float64)
    assert float((exact - ref.double()).abs().max()) <= tol


def test_planted_mistakes_are_caught(gold):
    """The tolerances above reject small semantic slips in the oracle: the two halves of the
    SwiGLU swapped in one transition, and ``B`` used untransposed in the parcae step."""
    d, meta = gold
    head = DiffusionHead(**meta["pc"])
    head.load_state_dict({k[5:]: torch.from_numpy(d[k]) for k in d.files if k.startswith("pc_w/")})
    p = pco.pair_cond_params(head)
    t0 = p["transitions"][1]
    p["transitions"][1] = {**t0, "a": t0["b"], "b": t0["a"]}
    got = pco.pair_biases_fp16(p, torch.from_numpy(d["pc/B1L12/z_trunk"]), torch.from_numpy(d["pc/B1L12/rel_pos"]))
    ref = torch.from_numpy(d["pc/B1L12/bias"].astype(np.float32))
    assert float((got - ref).norm() / ref.norm()) > 1e-2

    t = {k: torch.from_numpy(d[f"parcae/B1L9/{k}"]) for k in
         ("z", "z_init", "refined", "ln_w", "ln_b", "a", "b_mat", "z_next")}
    wrong = pao.parcae_step(t["z"], t["z_init"], t["refined"], t["ln_w"], t["ln_b"], t["a"], t["b_mat"].T)
    assert float((wrong - t["z_next"]).abs().max()) > 1e-2 * float(t["z_next"].abs().max())
