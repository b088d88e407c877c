"""Host logic with no GPU: the variant registry (``src/esmfold2_mlx/variants.py:74-86``) and the
adaptive-recycling state machine (``src/esmfold2_mlx/var_adaptive_loops.py:79-156``).

The adaptive tests replace the K5 distogram kernel with the reference's formula on the CPU
(``var_adaptive_loops.py:43-46``: ``softmax(head(z + z^T)) @ centres``) and the trunk with a
scripted module, so only the pass / settle / extra-pass bookkeeping is under test.
"""

from __future__ import annotations

import sys
import types

import pytest
import torch
from torch import nn

from esmfold2_mlx_b200 import adaptive, variants


# ---------------------------------------------------------------- registry

def test_unknown_variant_raises_value_error():
    with pytest.raises(ValueError, match="unknown speed variant 'no_such_stack'"):
        variants.apply_variants(object(), ["no_such_stack"])


def test_variants_apply_in_order_from_a_comma_string(monkeypatch):
    calls = []
    for name in ("fake_a", "fake_b"):
        mod = types.ModuleType(f"esmfold2_mlx_b200.var_{name}")
        mod.apply = lambda model, _n=name: calls.append((_n, model))
        monkeypatch.setitem(sys.modules, mod.__name__, mod)
    model = object()
    assert variants.apply_variants(model, "fake_b,,fake_a") is model
    assert calls == [("fake_b", model), ("fake_a", model)]
    calls.clear()
    variants.apply_variants(model, [])
    variants.apply_variants(model, "")
    assert calls == []


def test_a_broken_import_inside_a_variant_is_not_reported_as_unknown(monkeypatch):
    """Only a missing ``var_<name>`` module means "unknown"; an import error inside it surfaces."""
    import importlib

    real = importlib.import_module

    def fake_import(name, *a, **k):
        if name.endswith("var_broken"):
            raise ModuleNotFoundError("No module named 'dependency_x'", name="dependency_x")
        return real(name, *a, **k)

    monkeypatch.setattr(importlib, "import_module", fake_import)
    with pytest.raises(ModuleNotFoundError, match="dependency_x"):
        variants.apply_variants(object(), "broken")


# ---------------------------------------------------------------- adaptive recycling

C_Z, L = 8, 6


class _ScriptedTrunk(nn.Module):
    """Returns ``base * s`` for the next scale ``s`` of its script; records every call."""

    def __init__(self, scales):
        super().__init__()
        self.scales = list(scales)
        self.inputs = []
        self.base = torch.randn(1, L, L, C_Z, generator=torch.Generator().manual_seed(0))

    def forward(self, pair, pair_attention_mask=None):
        self.inputs.append(pair.clone())
        return self.base * self.scales[len(self.inputs) - 1]

    def set_chunk_size(self, n):
        self.chunk = n

    def set_kernel_backend(self, b):
        self.backend = b


@torch.no_grad()
def _formula_expected_distance(z, head):
    """The reference's formula on the CPU (var_adaptive_loops.py:43-46)."""
    logits = head(z.float() + z.float().transpose(-2, -3))
    return logits.softmax(-1) @ adaptive.CENTRES


def _model(proj=None):
    m = nn.Module()
    m.distogram_head = nn.Linear(C_Z, 128)
    torch.nn.init.normal_(m.distogram_head.weight, std=2.0, generator=torch.Generator().manual_seed(1))
    if proj is not None:
        m.pair_loop_proj = proj
    return m


@pytest.fixture
def cpu_head(monkeypatch):
    """K5 replaced by the formula on the CPU: the wrapper's evaluator calls the head module."""
    monkeypatch.setattr(adaptive, "ExpectedDistance", lambda head, device: (lambda z: _formula_expected_distance(z, head)))


def _p95(trunk_a, trunk_b, head):
    ea = _formula_expected_distance(trunk_a.to(torch.float16), head)
    eb = _formula_expected_distance(trunk_b.to(torch.float16), head)
    return float((eb - ea).abs().flatten().quantile(0.95))


def test_bin_centres_follow_the_reference_edges():
    """128 centres: 127 edges evenly over 2-52 A, open-ended bins 0.2 A outside (var_adaptive_loops.py:38-40)."""
    c = adaptive.CENTRES
    step = 50.0 / 126
    assert c.shape == (128,)
    assert abs(float(c[0]) - 1.8) < 1e-6 and abs(float(c[-1]) - 52.2) < 1e-5
    assert torch.allclose(c[1:-1], 2.0 + step * (torch.arange(126) + 0.5), atol=1e-5)


def test_converges_then_returns_the_converged_output_without_running_the_trunk(cpu_head):
    scripted = _ScriptedTrunk([1.0, -1.0, -1.0, 9.0, 9.0])
    model = _model()
    t = adaptive.CUDAAdaptiveTrunk(scripted, model)
    t.start_fold(5)
    pair = torch.zeros(1, L, L, C_Z)
    outs = [t(pair) for _ in range(5)]
    # pass 2 (the sign flipped) moves the distogram (p95 well above 0.6 A), pass 3 repeats it
    assert _p95(scripted.base, -scripted.base, model.distogram_head) > adaptive.SETTLE_A
    assert t.converged and t.passes == 3 and len(scripted.inputs) == 3
    assert t.fold.changes[1] == 0.0
    assert outs[3] is outs[2] and outs[4] is outs[2]


def test_min_passes_holds_back_an_early_convergence(cpu_head):
    scripted = _ScriptedTrunk([2.0, 2.0, 2.0, 2.0])
    t = adaptive.CUDAAdaptiveTrunk(scripted, _model(), min_passes=3)
    t.start_fold(4)
    pair = torch.zeros(1, L, L, C_Z)
    t(pair)
    t(pair)
    assert not t.converged and t.passes == 2  # converged by the metric, but only two passes ran
    t(pair)
    assert t.converged and t.passes == 3
    t(pair)
    assert len(scripted.inputs) == 3


def test_start_fold_begins_a_new_fold(cpu_head):
    scripted = _ScriptedTrunk([1.0, 1.0, 1.0, -1.0])
    t = adaptive.CUDAAdaptiveTrunk(scripted, _model())
    pair = torch.zeros(1, L, L, C_Z)
    t.start_fold(2)
    t(pair)
    t(pair)
    assert t.converged
    t.start_fold(2)
    assert not t.converged and t.passes == 0 and t.fold.changes == [] and t.fold.latest is None
    t(pair)
    t(pair)
    # the first pass of the new fold has nothing to compare with (no carry-over from the last
    # fold), and the second (sign flip) moves the distogram
    assert t.passes == 2 and not t.converged and len(t.fold.changes) == 1
    assert len(scripted.inputs) == 4


def test_extra_passes_after_the_scheduled_ones(cpu_head):
    """With ``max_extra``, the last scheduled call runs up to ``max_extra`` more passes on
    ``z_init + proj(out)`` (``var_adaptive_loops.py:127-142``), stopping at the extra threshold."""
    proj = nn.Linear(C_Z, C_Z)
    scripted = _ScriptedTrunk([1.0, -1.0, 1.0, -1.0, -1.0, 1.0])
    t = adaptive.CUDAAdaptiveTrunk(scripted, _model(proj), max_extra=3)
    t.start_fold(3)
    pair = torch.randn(1, L, L, C_Z, generator=torch.Generator().manual_seed(2))
    z_init = pair - proj(torch.zeros_like(pair))
    t(pair)
    t(pair)
    out = t(pair)  # scheduled call 3: pass 3, then extra passes 4 (moves) and 5 (repeats: stop)
    assert t.passes == 5 and not t.converged
    assert torch.equal(out, -scripted.base)
    # extra pass inputs are z_init + proj(previous output)
    assert torch.allclose(scripted.inputs[3], z_init + proj(scripted.base))
    assert torch.allclose(scripted.inputs[4], z_init + proj(-scripted.base))
    assert t.fold.changes[-1] == 0.0


def test_wrapper_forwards_chunk_and_backend_setters(cpu_head):
    scripted = _ScriptedTrunk([1.0])
    t = adaptive.CUDAAdaptiveTrunk(scripted, _model())
    t.set_chunk_size(64)
    t.set_kernel_backend("cuda")
    assert scripted.chunk == 64 and scripted.backend == "cuda"


def test_apply_starts_a_fold_per_forward_with_num_loops_plus_one(cpu_head):
    model = _model()
    model.folding_trunk = _ScriptedTrunk([1.0] * 8)
    model.config = types.SimpleNamespace(num_loops=3)
    seen = []
    model.forward = lambda *a, num_loops=None, **k: seen.append(model.folding_trunk.fold.scheduled)
    trunk = adaptive.apply(model)
    assert model.folding_trunk is trunk
    model.forward()
    model.forward(num_loops=5)
    assert seen == [4, 6]


def test_wrapper_keeps_the_model_state_dict_unchanged(cpu_head):
    proj = nn.Linear(C_Z, C_Z)
    model = _model(proj)
    model.folding_trunk = _ScriptedTrunk([1.0])
    before = set(model.state_dict())
    adaptive.apply(model)
    after = {k for k in model.state_dict() if not k.startswith("folding_trunk.")}
    assert after == before - {k for k in before if k.startswith("folding_trunk.")}


# ---------------------------------------------------------------- weight copies (mlx_trunk.py:40-69)

@pytest.mark.parametrize("c_z", [128, 256])
def test_trunk_weight_copy_matches_the_reference_orientation(c_z):
    """``trunk_params`` (the kernels' layouts, built on the CPU here) holds exactly the oracle's
    reference-orientation fp16 weights: the packed projection is ``w_in^T`` with rows in the
    order [signal a | gate a | signal b | gate b] and the 1/256 pre-scale on signal a
    (``mlx_trunk.py:44-48``); emit / gate / transition matrices are the ``nn.Linear`` layouts,
    i.e. the transposes of ``w_emit`` / ``w_out_gate`` / ``w12`` / ``w3`` (``:49-66``)."""
    from esmfold2_mlx_b200 import ops
    from esmfold2_mlx_b200.synthetic import FoldingTrunk, trimul_biases
    from esmfold2_mlx_b200.trunk import trunk_params
    from oracle import trimul_oracle as orc

    ft = FoldingTrunk(2, c_z, c_z, hidden=2 * c_z, seed=3)
    biases = [{"out": trimul_biases(c_z, c_z, seed=10 + i), "in": trimul_biases(c_z, c_z, seed=20 + i)} for i in range(2)]
    got = trunk_params(ft, device="cpu", biases=biases)
    ref = orc.trunk_params(ft)
    order = torch.tensor(ops.proj_row_order_py(c_z))
    for g, r, blk, bb in zip(got, ref, ft.blocks, biases):
        for d in ("out", "in"):
            w, p = g[d], r[d]
            assert (w.c, w.c_z) == (c_z, c_z)
            assert torch.equal(w.w_proj.float(), p["w_in"].T[order])
            assert torch.equal(w.w_emit.float(), p["w_emit"].T)
            assert torch.equal(w.w_gate.float(), p["w_out_gate"].T)
            for k in ("ln_in_w", "ln_in_b", "ln_mix_w", "ln_mix_b"):
                assert torch.equal(getattr(w, k).float(), p[k])
            b_in = bb[d]["b_in"].detach().float().clone()
            b_in[:c_z] /= ops.CONTRACT_SCALE
            assert torch.equal(w.b_proj, b_in[order])
            assert torch.equal(w.b_emit, bb[d]["b_emit"].float())
            assert w.w_proj.dtype == torch.float16 and w.b_proj.dtype == torch.float32
        tw = g["tw"]
        assert tw.fused and tw.activation == "swiglu" and tw.hidden == 2 * c_z
        assert torch.equal(tw.w12.float(), r["w12"].T) and torch.equal(tw.w3.float(), r["w3"].T)
        assert torch.equal(tw.ln_w.float(), r["ln_w"]) and torch.equal(tw.ln_b.float(), r["ln_b"])


def test_trunk_params_refuses_other_dtypes():
    from esmfold2_mlx_b200.synthetic import FoldingTrunk
    from esmfold2_mlx_b200.trunk import trunk_params

    with pytest.raises(ValueError, match="fp16"):
        trunk_params(FoldingTrunk(1, 128, 128, hidden=256, seed=0), dtype=torch.bfloat16, device="cpu")


# ---------------------------------------------------------------- drop-in module surface (var_mlx_trunk.py:24-46)

def _tiny_trunk(seed):
    from esmfold2_mlx_b200.synthetic import FoldingTrunk

    return FoldingTrunk(1, 128, 128, hidden=256, seed=seed)


def test_trunk_module_surface_and_no_cpu_fallback():
    """``CUDAFoldingTrunk`` keeps the reference module's surface (``params``, ``_fn``, no-op
    ``set_chunk_size`` / ``set_kernel_backend``, an ``nn.Module`` whose forward hooks see the pair
    tensor, as ``tools/regression_check.py:73-77`` reads it), and its compute path refuses tensors
    that are not on a CUDA device instead of falling back to another implementation."""
    from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk, make_trunk

    t = CUDAFoldingTrunk(_tiny_trunk(1), device="cpu")
    assert isinstance(t, nn.Module) and callable(t._fn) and len(t.params) == 1
    assert set(t.params[0]) >= {"out", "in", "tw"}
    assert t.set_chunk_size(64) is None and t.set_kernel_backend("triton") is None
    seen = []
    t.register_forward_pre_hook(lambda mod, args, kwargs: seen.append(args[0] if args else kwargs["pair"]),
                                with_kwargs=True)
    pair = torch.zeros(1, 8, 8, 128)
    with pytest.raises(TypeError, match="CUDA"):
        t(pair)
    assert len(seen) == 1 and seen[0] is pair
    with pytest.raises(ValueError, match="fp16"):
        make_trunk(torch.float32)


def test_6b_variant_wraps_all_four_trunk_stacks():
    """``var_6b_mlx_trunks16k.py:19-32``: folding trunk, lm_encoder (when present), parcae coda and
    the confidence head's trunk each become the B200 module; applying twice keeps them."""
    from esmfold2_mlx_b200 import var_6b_cuda_trunks16 as v6
    from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk

    def model(with_lm):
        m = nn.Module()
        m.folding_trunk, m.parcae_coda = _tiny_trunk(1), _tiny_trunk(2)
        m.lm_encoder = _tiny_trunk(3) if with_lm else None
        m.confidence_head = nn.Module()
        m.confidence_head.folding_trunk = _tiny_trunk(4)
        return m

    m = model(True)
    v6.apply(m, device="cpu")
    stacks = (m.folding_trunk, m.lm_encoder, m.parcae_coda, m.confidence_head.folding_trunk)
    assert all(isinstance(s, CUDAFoldingTrunk) for s in stacks)
    v6.apply(m, device="cpu")
    assert all(a is b for a, b in zip(stacks, (m.folding_trunk, m.lm_encoder, m.parcae_coda,
                                                 m.confidence_head.folding_trunk)))
    m = model(False)
    v6.apply(m, device="cpu")
    assert m.lm_encoder is None and isinstance(m.parcae_coda, CUDAFoldingTrunk)
