"""Host logic of the parcae step: the exact three-way bf16 split of B, the weight copy, and
the entry point's argument checks (no GPU)."""

from __future__ import annotations

import ctypes

import torch
from torch import nn

from esmfold2_mlx_b200 import _lib
from esmfold2_mlx_b200.parcae import ParcaeWeights, split_bf16x3


def test_bf16x3_split_is_exact():
    """Exact while the third part stays a normal bf16, |m| >= 2^-110 (weights are far above)."""
    g = torch.Generator().manual_seed(0)
    m = torch.cat([torch.randn(64, 256, generator=g) * s for s in (1e-20, 1e-3, 1.0, 1e3, 1e30)], 0)
    parts = split_bf16x3(m)
    assert parts.dtype == torch.bfloat16 and parts.shape == (320, 768)
    m0, m1, m2 = parts.double().split(256, -1)
    assert torch.equal(m0 + m1 + m2, m.double())


def test_weights_from_model_expand_a_and_split_b():
    c = 128
    model = nn.Module()
    model.parcae_input_norm = nn.LayerNorm(c)
    b = torch.randn(c, c)
    w = ParcaeWeights.from_model(model, torch.tensor(0.25), b, "cpu")
    assert w.a.shape == (c,) and bool((w.a == 0.25).all())
    assert torch.equal(w.b_split.double().split(c, -1)[0] + w.b_split.double().split(c, -1)[1]
                       + w.b_split.double().split(c, -1)[2], b.double())


def test_parcae_argument_checks_need_no_gpu():
    lib = _lib.load()
    PW = ctypes.POINTER(_lib.TmuParcaeWeights)
    pw = _lib.TmuParcaeWeights()
    assert lib.tmu_parcae_step(None, None, None, PW(), None, 1, 16, 192, None, 0, None, None) == 4  # c_z 192
    assert lib.tmu_parcae_step(None, None, None, PW(), None, 1, 16, 256, None, 0, None, None) == 1  # no weights
    assert lib.tmu_parcae_step(None, None, None, ctypes.byref(pw), None, 1, 16, 256, None, 0, None, None) == 1
    assert lib.tmu_parcae_workspace_bytes(1, 16, 256) == 16 * 16 * 768 * 2
