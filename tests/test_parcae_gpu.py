"""GPU parity of the parcae step (``tmu_parcae_step``: LayerNorm pass with a three-way bf16
split + K6 over the six partial products) against the fp32 restatement of
var_6b_mlx_loop.py:67-71 (``oracle/parcae_oracle.py``).

Bound: the CUDA result's distance to the exact (float64) step is at most 4x the fp32
oracle's own distance to it, plus 2^-20 of the output's scale: the bf16x3 product keeps 24
significant bits, so only the summation order differs from an fp32 GEMM.
"""

from __future__ import annotations

import pytest
import torch
from torch import nn

from esmfold2_mlx_b200 import parcae
from esmfold2_mlx_b200.ops import new_status, read_status
from oracle import parcae_oracle as po

pytestmark = pytest.mark.gpu

DEV = "cuda"


class _Model(nn.Module):
    def __init__(self, c, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.parcae_input_norm = nn.LayerNorm(c)
        with torch.no_grad():
            self.parcae_input_norm.weight.copy_(1 + 0.1 * torch.randn(c, generator=g))
            self.parcae_input_norm.bias.copy_(0.1 * torch.randn(c, generator=g))


def _inputs(B, L, c, seed):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(B, L, L, c, generator=g) * 30.0
    z_init = torch.randn(B, L, L, c, generator=g) * 3.0
    refined = torch.randn(B, L, L, c, generator=g) * 10.0
    a = torch.rand(c, generator=g) * 0.9
    b_mat = torch.randn(c, c, generator=g) / c**0.5
    return z, z_init, refined, a, b_mat


@pytest.mark.parametrize("B,L,c", [(1, 37, 256), (2, 50, 128), (1, 130, 256)])
@pytest.mark.parametrize("in_place", [False, True])
def test_parcae_step_matches_fp32_oracle(B, L, c, in_place):
    m = _Model(c, seed=L + c)
    z, zi, rf, a, b_mat = _inputs(B, L, c, seed=L * c)
    w = parcae.ParcaeWeights.from_model(m, a, b_mat, DEV)
    zd = z.to(DEV)
    st = new_status(DEV)
    out = parcae.parcae_step(zd, zi.to(DEV), rf.to(DEV), w, out=zd if in_place else None, status=st)
    torch.cuda.synchronize()
    assert read_status(st)[0] == 0
    got = out.double().cpu()
    nw, nb = m.parcae_input_norm.weight.detach(), m.parcae_input_norm.bias.detach()
    ref64 = po.parcae_step(z, zi, rf, nw, nb, a, b_mat, torch.float64)
    ref32 = po.parcae_step(z, zi, rf, nw, nb, a, b_mat, torch.float32).double()
    e32 = float((ref32 - ref64).abs().max())
    e = float((got - ref64).abs().max())
    scale = float(ref64.abs().max())
    assert e <= 4 * e32 + scale * 2.0**-20, (e, e32, scale)


def test_parcae_scalar_a_broadcasts():
    c, L = 128, 24
    m = _Model(c, seed=1)
    z, zi, rf, _, b_mat = _inputs(1, L, c, seed=2)
    w = parcae.ParcaeWeights.from_model(m, torch.tensor(0.5), b_mat, DEV)
    out = parcae.parcae_step(z.to(DEV), zi.to(DEV), rf.to(DEV), w).double().cpu()
    nw, nb = m.parcae_input_norm.weight.detach(), m.parcae_input_norm.bias.detach()
    ref = po.parcae_step(z, zi, rf, nw, nb, 0.5, b_mat, torch.float64)
    assert float((out - ref).abs().max()) <= float(ref.abs().max()) * 2.0**-19


def test_loop_step_composes_lm_encoder_parcae_and_trunk():
    """loop_step == folding_trunk(parcae(z, z_init, lm_encoder(lz))) (var_6b_mlx_loop.py:67-71)."""
    from esmfold2_mlx_b200.synthetic import FoldingTrunk
    from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk

    c, L = 128, 40
    lm = CUDAFoldingTrunk(FoldingTrunk(1, c, c, hidden=256, seed=1, ln_noise=0.1), device=DEV)
    tr = CUDAFoldingTrunk(FoldingTrunk(2, c, c, hidden=256, seed=2, ln_noise=0.1), device=DEV)
    m = _Model(c, seed=3)
    z, zi, rf, a, b_mat = _inputs(1, L, c, seed=4)
    w = parcae.ParcaeWeights.from_model(m, a, b_mat, DEV)
    lz, zd, zid = rf.to(DEV), (z / 10).to(DEV), zi.to(DEV)
    got = parcae.loop_step(lm, tr, w, lz, zd, zid)
    ref = tr(parcae.parcae_step(zd, zid, lm(lz).float().contiguous(), w))
    torch.cuda.synchronize()
    assert got.shape == (1, L, L, c) and torch.equal(got, ref)
