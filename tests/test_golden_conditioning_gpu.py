"""GPU: ``tmu_pair_cond`` and ``tmu_parcae_step`` (through the C ABI) against the outputs of the
reference's own ``mlx_diffusion16.pair_biases`` and ``var_6b_mlx_loop._step``
(``tests/golden/conditioning_golden.npz``, cases ``pc2/B1L64`` and ``parcae/B1L20c128``).

Tolerances follow from the two bounds already established, by the triangle inequality:
* pair conditioning: the oracle is within 2 fp16 ulps (at the tensor's scale) of the fixture and
  the CUDA path within 2 of the oracle (``tests/test_pair_cond_gpu.py``), so 4 ulps; rel-L2 2e-3;
* parcae step (fp32): |cuda - fixture| <= |cuda - exact| + |fixture - exact|, with the CUDA bound
  of ``tests/test_parcae_gpu.py`` (4 x the fp32 oracle's own error + 2^-20 of the scale) and the
  fixture's measured distance from the float64 step.
"""

from __future__ import annotations

import ast
import math
import os

import numpy as np
import pytest
import torch
from torch import nn

from esmfold2_mlx_b200 import pair_cond, parcae
from esmfold2_mlx_b200.ops import new_status, read_status
from esmfold2_mlx_b200.synthetic import DiffusionHead
from oracle import parcae_oracle as pao

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLD = os.path.join(os.path.dirname(__file__), "golden", "conditioning_golden.npz")


@pytest.fixture(scope="module")
def gold():
    d = np.load(GOLD)
    return d, ast.literal_eval(bytes(d["meta"]).decode())


def test_pair_cond_matches_reference_outputs(gold):
    d, meta = gold
    head = DiffusionHead(**meta["pc2"])
    head.load_state_dict({k[6:]: torch.from_numpy(d[k]) for k in d.files if k.startswith("pc2_w/")})
    w = pair_cond.PairCondWeights.from_head(head, DEV)
    zt = torch.from_numpy(d["pc2/B1L64/z_trunk"]).float().to(DEV)
    rp = torch.from_numpy(d["pc2/B1L64/rel_pos"]).float().to(DEV)
    st = new_status(DEV)
    out = pair_cond.pair_biases(w, zt, rp, status=st)
    torch.cuda.synchronize()
    assert read_status(st)[0] == 0
    got = out.float().cpu()
    ref = torch.from_numpy(d["pc2/B1L64/bias"].astype(np.float32))
    assert got.shape == ref.shape
    diff = (got - ref).abs()
    scale = 2.0 ** (math.floor(math.log2(max(float(ref.abs().max()), 2.0**-14))) - 10)
    assert float(diff.max()) <= 4 * scale, f"max diff {float(diff.max()):.3g} > 4 x {scale:.3g}"
    assert float(diff.norm() / ref.norm()) <= 2e-3


def test_parcae_step_matches_reference_outputs(gold):
    d, _ = gold
    t = {k: torch.from_numpy(d[f"parcae/B1L20c128/{k}"]) for k in
         ("z", "z_init", "refined", "ln_w", "ln_b", "a", "b_mat", "z_next")}
    c = t["z"].shape[-1]
    model = nn.Module()
    model.parcae_input_norm = nn.LayerNorm(c)
    with torch.no_grad():
        model.parcae_input_norm.weight.copy_(t["ln_w"])
        model.parcae_input_norm.bias.copy_(t["ln_b"])
    w = parcae.ParcaeWeights.from_model(model, t["a"], t["b_mat"], DEV)
    st = new_status(DEV)
    out = parcae.parcae_step(t["z"].to(DEV), t["z_init"].to(DEV), t["refined"].to(DEV), w, status=st)
    torch.cuda.synchronize()
    assert read_status(st)[0] == 0
    got = out.double().cpu()
    args = (t["z"], t["z_init"], t["refined"], t["ln_w"], t["ln_b"], t["a"], t["b_mat"])
    exact = pao.parcae_step(*args, dtype=torch.float64)
    e32 = float((pao.parcae_step(*args, dtype=torch.float32).double() - exact).abs().max())
    scale = float(exact.abs().max())
    e_fix = float((t["z_next"].double() - exact).abs().max())
    bound = 4 * e32 + scale * 2.0**-20 + e_fix
    assert float((got - t["z_next"].double()).abs().max()) <= bound
