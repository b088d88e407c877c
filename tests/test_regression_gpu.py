"""Two trunk-level checks from the reference, carried over to the CUDA path.

* ``tools/regression_check.py:121-137``: the trunk's input of a 238-residue fold, tiled 2 x 2 to
  L = 476 and run with an all-ones mask, must give a finite output.  The fold's real trunk input
  needs the checkpoint; a seeded pair tensor with large entries stands in for it.
* Distogram agreement: the expected distance per pair (the distogram head on ``z + z^T``, softmax,
  bin centres; ``var_adaptive_loops.py:39-46``) of the CUDA trunk's output and of the oracle's
  must agree to a 95th-percentile difference well below 0.1 A; the reference treats 0.6 A as "the
  structure does not move" (``var_adaptive_loops.py:31-32``).
"""

from __future__ import annotations

import pytest
import torch
from torch import nn

from esmfold2_mlx_b200.adaptive import CENTRES
from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_mask, pair_tensor
from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk
from oracle import trimul_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("cz", [128, 256])
def test_trunk_is_finite_on_a_2x2_tiled_input(cz):
    trunk = FoldingTrunk(4, cz, cz, hidden=2 * cz, seed=cz, ln_noise=0.1)
    z = 8.0 * pair_tensor(1, 238, cz, 5)
    big = z.repeat(1, 2, 2, 1).to(DEV)
    assert big.shape == (1, 476, 476, cz)
    out = CUDAFoldingTrunk(trunk)(big, pair_attention_mask=torch.ones(big.shape[:-1], device=DEV))
    torch.cuda.synchronize()
    assert out.shape == big.shape and out.dtype == torch.float32
    assert bool(torch.isfinite(out).all()), "non-finite trunk output at L = 476"
    print(f"c_z={cz} at L=476 (2 x 2 tiled): finite, max |z| {float(out.abs().max()):.1f}")
    assert float(out.abs().max()) < 6e4  # inside fp16 range: nothing saturated


@torch.no_grad()
def _expected_distance(z: torch.Tensor, head: nn.Linear) -> torch.Tensor:
    logits = head(z + z.transpose(-2, -3))
    return logits.softmax(-1) @ CENTRES


@pytest.mark.parametrize("cz,L,n_pad", [(128, 76, 6), (256, 60, 0)])
def test_distogram_agrees_with_the_oracle_trunk(cz, L, n_pad):
    trunk = FoldingTrunk(2, cz, cz, hidden=2 * cz, seed=11 + cz, ln_noise=0.1)
    z = pair_tensor(1, L, cz, 12)
    mask = pair_mask(1, L, n_pad) if n_pad else None
    ref = orc.trunk_fp16(orc.trunk_params(trunk, True), z, mask)
    got = CUDAFoldingTrunk(trunk)(z.to(DEV), pair_attention_mask=None if mask is None else mask.to(DEV)).cpu()
    head = nn.Linear(cz, 128)
    g = torch.Generator().manual_seed(cz)
    with torch.no_grad():
        head.weight.copy_(torch.randn(128, cz, generator=g) / cz**0.5)
        head.bias.copy_(0.1 * torch.randn(128, generator=g))
    e_ref, e_got = _expected_distance(ref, head), _expected_distance(got, head)
    spread = float(e_ref.std())
    assert spread > 0.5  # the head resolves distances on these inputs, so agreement means something
    d = (e_got - e_ref).abs().flatten()
    p95 = float(d.quantile(0.95))
    print(f"distogram agreement c_z={cz} L={L}: p95 |dE| = {p95:.4f} A, max {float(d.max()):.4f} A")
    assert p95 < 0.1, f"p95 |dE| = {p95:.4f} A"
    assert float(d.max()) < 0.6, f"max |dE| = {float(d.max()):.4f} A"
