"""GPU: ``tmu_pair_block`` (one PairUpdateBlock in one C-ABI call) against ``trunk.block_forward``,
which composes the same kernels through three calls (tri-mul out, tri-mul in, transition).
Both run the same deterministic kernels on the same inputs, so the results must be identical
bit for bit, in place and out of place, at c_z = 128 and 256."""

from __future__ import annotations

import pytest
import torch

from esmfold2_mlx_b200 import ops
from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_mask, pair_tensor
from esmfold2_mlx_b200.trunk import block_forward, trunk_params

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("cz,L,B,n_pad", [(128, 76, 1, 5), (128, 33, 2, 0), (256, 64, 1, 4), (256, 48, 2, 0)])
@pytest.mark.parametrize("in_place", [False, True])
def test_pair_block_equals_block_forward(cz, L, B, n_pad, in_place):
    trunk = FoldingTrunk(1, cz, cz, hidden=2 * cz, seed=L + cz, ln_noise=0.1)
    p = trunk_params(trunk, device=DEV)[0]
    assert p["tw"].fused
    z = pair_tensor(B, L, cz, L + 1).half().to(DEV)
    mask = pair_mask(B, L, n_pad).half().to(DEV) if n_pad else None
    ref = z.clone()
    block_forward(p, ref, mask)
    ws = ops.Workspace()
    if in_place:
        got = z.clone()
        assert ops.pair_block(got, mask, p["out"], p["in"], p["tw"], out=got, workspace=ws) is got
    else:
        zin = z.clone()
        got = ops.pair_block(zin, mask, p["out"], p["in"], p["tw"], workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(zin, z)  # the input is left as it was
    code, site = ops.read_status(ws.status)
    assert code == 0, (code, hex(site))
    assert torch.equal(got, ref)


def test_pair_block_twice_reuses_its_workspace():
    """Two blocks in a row through one workspace: the second call's first kernel re-zeroes the
    shared status word and the pair buffer is rewritten before it is read."""
    cz, L = 256, 64
    trunk = FoldingTrunk(2, cz, cz, hidden=512, seed=2, ln_noise=0.1)
    params = trunk_params(trunk, device=DEV)
    z = pair_tensor(1, L, cz, 3).half().to(DEV)
    ref = z.clone()
    for p in params:
        block_forward(p, ref, None)
    ws = ops.Workspace()
    got = z.clone()
    for p in params:
        ops.pair_block(got, None, p["out"], p["in"], p["tw"], out=got, workspace=ws)
    assert ops.read_status(ws.status)[0] == 0
    assert torch.equal(got, ref)
