"""GPU parity of K4, the fused pair transition (``tmu_transition``), against the CPU oracle.

The oracle (``transition_fp16``) follows the reference's fused path's rounding points
(mlx_trunk_kernels.py:236-239).  Bounds as for the tri-mul kernels: within 4 fp16 ulps of the
oracle at the tensor's scale, with only a small fraction of elements differing at all (fp32
summation order and the hardware sigmoid flip rare roundings).
"""

from __future__ import annotations

import pytest
import torch

from esmfold2_mlx_b200 import _lib, ops
from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_tensor
from oracle import trimul_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ulp16(x: float) -> float:
    import math
    x = max(abs(x), 2.0**-14)
    return 2.0 ** (math.floor(math.log2(x)) - 10)


def _case(L, B, hidden, activation, seed, cz=128):
    trunk = FoldingTrunk(1, cz, cz, hidden=hidden, seed=seed, activation=activation, ln_noise=0.1)
    tr = trunk.blocks[0].pair_transition
    z = (pair_tensor(B, L, cz, seed + 1) * 2).half().float()
    p = orc.trunk_params(trunk, True)[0]
    ref = orc.transition_fp16(p, z, activation)
    return tr, z, ref


@pytest.mark.parametrize("activation", ["swiglu", "relu"])
@pytest.mark.parametrize("L,B,hidden,cz", [(37, 1, 512, 128), (76, 2, 512, 128), (130, 1, 256, 128), (64, 1, 64, 128),
                                           (37, 1, 512, 256), (76, 2, 1024, 256), (130, 1, 256, 256),
                                           (64, 1, 64, 256)])
def test_transition_matches_oracle(activation, L, B, hidden, cz):
    tr, z, ref = _case(L, B, hidden, activation, seed=L + hidden, cz=cz)
    w = ops.TransitionWeights.from_module(tr, DEV)
    assert w.fused
    st = ops.new_status(DEV)
    out = ops.transition(z.half().to(DEV), w, status=st)
    torch.cuda.synchronize()
    assert ops.read_status(st)[0] == 0
    got = out.float().cpu()
    diff = (got - ref).abs()
    assert bool(torch.isfinite(got).all())
    assert float(diff.max()) <= 4 * _ulp16(float(ref.abs().max())), float(diff.max())
    assert float((diff > 0).float().mean()) < 0.05


@pytest.mark.parametrize("cz", [128, 256])
def test_transition_in_place_equals_out_of_place(cz):
    tr, z, _ = _case(96, 1, 512, "swiglu", seed=5, cz=cz)
    w = ops.TransitionWeights.from_module(tr, DEV)
    zd = z.half().to(DEV)
    ref = ops.transition(zd, w).clone()
    zz = zd.clone()
    ops.transition(zz, w, out=zz)
    torch.cuda.synchronize()
    assert torch.equal(zz, ref)


def test_transition_rejects_unsupported_shapes():
    tr, z, _ = _case(16, 1, 512, "swiglu", seed=2)
    w = ops.TransitionWeights.from_module(tr, DEV)
    w.hidden = 100  # not a multiple of 64
    with pytest.raises(_lib.TmuError):
        ops.transition(z.half().to(DEV), w)
