"""K5 (distogram expected distance) against the oracle, the reference-signature hook
``expected_distance(z, disto_head)``, and the adaptive-recycling wrapper (behaviour of
var_adaptive_loops.py:76-142) with K5 as its settle signal."""

from __future__ import annotations

import types

import pytest
import torch
from torch import nn

from esmfold2_mlx_b200 import adaptive, ops
from esmfold2_mlx_b200.synthetic import pair_tensor
from oracle import trimul_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _head(c_z, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    h = nn.Linear(c_z, 128, bias=bias)
    with torch.no_grad():
        h.weight.copy_(torch.randn(128, c_z, generator=g) / c_z ** 0.5)
        if bias:
            h.bias.copy_(torch.randn(128, generator=g) * 0.1)
    return h


@pytest.mark.parametrize("c_z,L,B,bias", [(128, 70, 2, True), (128, 130, 1, False), (256, 40, 1, True)])
def test_expected_distance_matches_oracle(c_z, L, B, bias):
    head = _head(c_z, seed=L, bias=bias)
    z = (pair_tensor(B, L, c_z, L + 1) * 0.5).half()
    dh = adaptive.ExpectedDistance(head, DEV)
    got = dh(z.to(DEV)).cpu()
    torch.cuda.synchronize()
    assert ops.read_status(dh.status)[0] == 0
    # the kernel uses the head's weight rounded to fp16; compare with the oracle on that weight
    w16 = head.weight.detach().half().float()
    b = head.bias.detach() if bias else torch.zeros(128)
    ref16 = orc.expected_distance(z.float(), w16, b)
    ref32 = orc.expected_distance(z.float(), head.weight.detach(), b)
    assert got.shape == (B, L, L)
    assert float((got - ref16).abs().max()) < 2e-3, float((got - ref16).abs().max())
    assert float((got - ref32).abs().max()) < 5e-2  # the fp16 weight's own effect, far below 0.6 Å
    # symmetric by construction (z + z^T)
    assert float((got - got.transpose(1, 2)).abs().max()) < 1e-4


def test_reference_signature_hook_takes_fp32_output_and_head_module():
    """``expected_distance(z, disto_head)`` as the reference's wrapper calls it: the trunk's fp32
    output and the model's head module; equal to K5 on the fp16 values, one device copy per head."""
    head = _head(128, seed=9).to(DEV)
    z32 = pair_tensor(1, 40, 128, 8).half().float().to(DEV)
    e1 = adaptive.expected_distance(z32, head)
    e2 = adaptive.expected_distance(z32, head)
    ref = adaptive.ExpectedDistance(head, DEV)(z32.half())
    torch.cuda.synchronize()
    assert torch.equal(e1, ref) and torch.equal(e2, ref)
    assert len(adaptive._evaluators[head]) == 1


class _Trunk(nn.Module):
    """Stand-in trunk: returns the input plus fresh noise of size `step` (0 = a fixed point)."""

    def __init__(self, step):
        super().__init__()
        self.step, self.calls = step, 0

    def set_chunk_size(self, n):
        pass

    def set_kernel_backend(self, b):
        pass

    def forward(self, pair, pair_attention_mask=None):
        self.calls += 1
        g = torch.Generator(device=pair.device).manual_seed(self.calls)
        return (pair + self.step * torch.randn(pair.shape, generator=g, device=pair.device)).half().float()


@pytest.mark.parametrize("step,expect_converged", [(0.0, True), (3.0, False)])
def test_adaptive_wrapper_stops_when_converged(step, expect_converged):
    L = 48
    model = types.SimpleNamespace(distogram_head=_head(128, 3).to(DEV), pair_loop_proj=None,
                                  config=types.SimpleNamespace(num_loops=3))
    inner = _Trunk(step)
    model.folding_trunk = inner
    trunk = adaptive.CUDAAdaptiveTrunk(inner, model)
    trunk.start_fold(4)
    z = pair_tensor(1, L, 128, 5).half().float().to(DEV)
    outs = [trunk(z) for _ in range(4)]  # the model's recycling loop: 4 trunk calls
    if expect_converged:
        assert trunk.converged and inner.calls == 2 and trunk.passes == 2
        assert trunk.fold.changes[0] < adaptive.SETTLE_A
        assert outs[3] is outs[1]  # the converged output is returned without running the trunk
    else:
        assert not trunk.converged and inner.calls == 4
        assert all(ch >= adaptive.SETTLE_A for ch in trunk.fold.changes)
