"""The drop-in through the reference's own code, on the CPU.

The reference's registry ``apply_variants`` (``src/esmfold2_mlx/variants.py:74-86``) imports
``esmfold2_mlx.var_<name>`` and calls its ``apply(model)``.  Here the reference's modules are
imported unmodified from a checkout (``ESMFOLD2_MLX_REFERENCE``, default: a ``reference``
directory beside this repository; the tests skip without one), with:

* the two Biohub ``esm`` classes its modules import (``fast_trunk.py:16``, ``variants.py:10``)
  registered as this repository's stand-in module tree (``synthetic.py``), since ``esm`` is not
  installed;
* the shim files a maintainer of the reference adds to its package (``var_cuda_trunk16.py`` and the
  others, one ``import`` line each) written to a temporary directory that is appended to the
  ``esmfold2_mlx`` package's search path.

The trunk's weights are placed on the CPU (there is no GPU here).  Its forward therefore raises
(no CPU fallback); for the recycling-loop test its compute function ``_fn`` is replaced by the
oracle trunk, so the reference's ``AdaptiveTrunk`` (``var_adaptive_loops.py:79-142``) and the
forward-hook capture of ``tools/regression_check.py:73-77`` run over the real module chain.
"""

from __future__ import annotations

import os
import sys
import types

import pytest
import torch
from torch import nn

from esmfold2_mlx_b200 import adaptive, synthetic
from esmfold2_mlx_b200 import var_6b_cuda_trunks16 as v6
from esmfold2_mlx_b200 import var_cuda_trunk16 as v16
from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk
from oracle import trimul_oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("ESMFOLD2_MLX_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))
REF_SRC = os.path.join(REF, "src")

pytestmark = pytest.mark.skipif(not os.path.exists(os.path.join(REF_SRC, "esmfold2_mlx", "variants.py")),
                                reason="no checkout of the reference (set ESMFOLD2_MLX_REFERENCE)")

# The shims a maintainer adds beside the reference's variants, one import line each.
SHIMS = {
    "var_cuda_trunk16.py": "from esmfold2_mlx_b200.var_cuda_trunk16 import apply  # noqa: F401\n",
    "var_6b_cuda_trunks16.py": "from esmfold2_mlx_b200.var_6b_cuda_trunks16 import apply  # noqa: F401\n",
    "var_cuda_adaptive_loops.py": "from esmfold2_mlx_b200.var_cuda_adaptive_loops import apply  # noqa: F401\n",
}


@pytest.fixture
def ref(monkeypatch, tmp_path):
    """The reference's ``variants`` and ``var_adaptive_loops`` modules, imported unmodified."""
    before = set(sys.modules)
    layers = types.ModuleType("esm.models.esmfold2.layers")
    layers.TriangleMultiplicativeBlock = synthetic.TriangleMultiplicativeBlock
    layers.Transition = synthetic.Transition
    esmfold2 = types.ModuleType("esm.models.esmfold2")
    esmfold2.EsmFold2ExperimentalModel = type("EsmFold2ExperimentalModel", (nn.Module,), {})
    esmfold2.layers = layers
    for name, mod in (("esm", types.ModuleType("esm")), ("esm.models", types.ModuleType("esm.models")),
                      ("esm.models.esmfold2", esmfold2), ("esm.models.esmfold2.layers", layers)):
        monkeypatch.setitem(sys.modules, name, mod)
    monkeypatch.syspath_prepend(REF_SRC)
    for fname, text in SHIMS.items():
        (tmp_path / fname).write_text(text)
    import esmfold2_mlx

    monkeypatch.setattr(esmfold2_mlx, "__path__", list(esmfold2_mlx.__path__) + [str(tmp_path)])
    from esmfold2_mlx import var_adaptive_loops, variants

    assert variants.__file__.startswith(REF_SRC) and var_adaptive_loops.__file__.startswith(REF_SRC)
    # weights on the CPU: the variants' apply() takes no device argument from the registry
    monkeypatch.setattr(v16, "DEVICE", "cpu")
    monkeypatch.setattr(v6, "DEVICE", "cpu")
    yield types.SimpleNamespace(variants=variants, adaptive_loops=var_adaptive_loops)
    for name in set(sys.modules) - before:
        if name.split(".")[0] in ("esmfold2_mlx", "esm"):
            del sys.modules[name]


C_Z, L = 128, 10


class _Model(nn.Module):
    """The parts of Biohub's model the variants and the recycling loop touch: the trunk, the
    distogram head, ``pair_loop_proj``, ``config.num_loops``, ``set_chunk_size`` and a forward
    that runs the recycling recurrence ``z = trunk(z_init + pair_loop_proj(z))`` num_loops + 1
    times."""

    def __init__(self, seed=5):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.folding_trunk = synthetic.FoldingTrunk(2, C_Z, C_Z, hidden=256, seed=seed)
        self.distogram_head = nn.Linear(C_Z, 128)
        self.pair_loop_proj = nn.Linear(C_Z, C_Z)
        with torch.no_grad():
            self.distogram_head.weight.copy_(torch.randn(128, C_Z, generator=g) / C_Z**0.5)
            self.pair_loop_proj.weight.copy_(0.1 * torch.randn(C_Z, C_Z, generator=g) / C_Z**0.5)
        self.config = types.SimpleNamespace(num_loops=3)

    def set_chunk_size(self, n):
        self.folding_trunk.set_chunk_size(n)

    def forward(self, z_init, mask=None, num_loops=None):
        n = self.config.num_loops if num_loops is None else num_loops
        z = torch.zeros_like(z_init)
        for _ in range(n + 1):
            z = self.folding_trunk(z_init + self.pair_loop_proj(z), pair_attention_mask=mask)
        return z


def test_reference_registry_swaps_in_the_cuda_trunk_under_its_adaptive_wrapper(ref):
    model = _Model()
    ref.variants.apply_variants(model, ["fast_trunk", "cuda_trunk16", "adaptive_loops"])
    wrapper = model.folding_trunk
    assert isinstance(wrapper, ref.adaptive_loops.AdaptiveTrunk)  # the reference's own class
    assert isinstance(wrapper.trunk, CUDAFoldingTrunk)
    wrapper.set_chunk_size(64)  # forwarded to the CUDA trunk, which ignores it
    wrapper.set_kernel_backend("cuda")
    assert len(wrapper.trunk.params) == 2
    # the default stack string form of the registry
    with pytest.raises(ValueError, match="unknown speed variant"):
        ref.variants.apply_variants(_Model(), ["cuda_trunk_no_such"])


def test_cuda_trunk_under_the_reference_wrapper_has_no_cpu_fallback(ref):
    model = _Model()
    ref.variants.apply_variants(model, ["cuda_trunk16", "adaptive_loops"])
    with pytest.raises(TypeError, match="CUDA"):
        model(torch.zeros(1, L, L, C_Z))


def test_reference_adaptive_loop_and_forward_hook_drive_the_cuda_trunk_module(ref):
    """The reference's AdaptiveTrunk runs its own convergence logic around CUDAFoldingTrunk's
    forward (cast, mask skip, fp32 result); the compute function is the oracle trunk here."""
    model = _Model()
    oracle_params = orc.trunk_params(model.folding_trunk, True)
    ref.variants.apply_variants(model, ["fast_trunk", "cuda_trunk16", "adaptive_loops"])
    wrapper = model.folding_trunk
    calls = []

    def oracle_fn(params, z, mask):
        calls.append(z.dtype)
        return orc.trunk_fp16(oracle_params, z.to(torch.float16).float(), mask)

    wrapper.trunk._fn = oracle_fn
    captured = {}
    trunk = model.folding_trunk
    while hasattr(trunk, "trunk"):  # regression_check.py:73-77: unwrap to the trunk doing the maths
        trunk = trunk.trunk
    trunk.register_forward_pre_hook(
        lambda m, a, k: captured.__setitem__("z", (a[0] if a else k["pair"]).detach()), with_kwargs=True)
    z_init = synthetic.pair_tensor(1, L, C_Z, 6)
    mask = torch.ones(1, L, L)
    with torch.no_grad():
        out = model(z_init, mask)
        # the same recurrence with the oracle trunk directly (an all-ones mask is skipped)
        z = torch.zeros_like(z_init)
        expect = []
        for _ in range(4):
            z = orc.trunk_fp16(oracle_params, (z_init + model.pair_loop_proj(z)).half().float(), None)
            expect.append(z)
    assert out.dtype == torch.float32 and out.shape == z_init.shape
    assert wrapper.passes == len(calls) and 2 <= wrapper.passes <= 4
    assert torch.equal(out, expect[wrapper.passes - 1])
    assert "z" in captured and captured["z"].shape == z_init.shape
    assert len(wrapper.history) == wrapper.passes - 1


def test_cuda_adaptive_variant_through_the_reference_registry(ref, monkeypatch):
    monkeypatch.setattr(adaptive, "ExpectedDistance",
                        lambda head, device: (lambda z: head(z.float() + z.float().transpose(-2, -3)).softmax(-1)
                                              @ adaptive.CENTRES))
    model = _Model()
    ref.variants.apply_variants(model, ["cuda_trunk16", "cuda_adaptive_loops"])
    assert isinstance(model.folding_trunk, adaptive.CUDAAdaptiveTrunk)
    assert isinstance(model.folding_trunk.trunk, CUDAFoldingTrunk)
    # the state dict keeps the model's own keys (the head and projection are not re-registered)
    keys = set(model.state_dict())
    assert "distogram_head.weight" in keys and not any(k.startswith("folding_trunk._") for k in keys)


def test_6b_variant_through_the_reference_registry(ref):
    m = nn.Module()
    m.folding_trunk = synthetic.FoldingTrunk(1, C_Z, C_Z, hidden=256, seed=1)
    m.lm_encoder = synthetic.FoldingTrunk(1, C_Z, C_Z, hidden=256, seed=2)
    m.parcae_coda = synthetic.FoldingTrunk(1, C_Z, C_Z, hidden=256, seed=3)
    m.confidence_head = nn.Module()
    m.confidence_head.folding_trunk = synthetic.FoldingTrunk(1, C_Z, C_Z, hidden=256, seed=4)
    ref.variants.apply_variants(m, ["6b_cuda_trunks16"])
    stacks = [m.folding_trunk, m.lm_encoder, m.parcae_coda, m.confidence_head.folding_trunk]
    assert all(isinstance(s, CUDAFoldingTrunk) for s in stacks)
