"""CPU oracle for the triangle multiplicative update (TEST INFRASTRUCTURE ONLY).

This module is the checker the parity tests, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` compare against.  Nothing in
the product package imports it; the CUDA path never routes through it.

It restates, in plain PyTorch on the CPU, the arithmetic of the reference's trunk
(abhi0raj/esmfold2-mlx, paths relative to ``src/esmfold2_mlx/``):

* ``mlx_trunk.py:40-55``   ``_trimul_params``: ``w_in = proj_bundle.weight.T`` with columns
  ``[signal_a | signal_b | gate_a | gate_b]``; in fp16 the left operand's columns are divided
  by ``CONTRACT_SCALE = 256`` (``:33,47-48``).
* ``mlx_trunk.py:72-90``   ``_gated_cf`` / ``_trimul``: ``n = LN(z)``, ``proj = n @ w_in``,
  ``a = proj[:, :c]*sigmoid(proj[:, 2c:3c])*mask``, ``b = proj[:, c:2c]*sigmoid(proj[:, 3c:])*mask``
  (channels first), outgoing ``x[d,i,j] = sum_k a[d,i,k] b[d,j,k]``, incoming
  ``x[d,i,j] = sum_k a[d,k,i] b[d,k,j]``, ``mixed = LN_mix(x^T) @ w_emit``,
  ``update = mixed * sigmoid(n @ w_out_gate)``.
* ``mlx_trunk.py:93-99``   ``block_forward``: out, in, then the SwiGLU transition.
* ``mlx_trunk.py:114``     ``mix_eps = 1e-5 / 256**2`` in fp16 (``LN(x/s, eps/s^2) == LN(x, eps)``).
* ``mlx_trunk_kernels.py:16-19,47-80,107-147,165-190,232-239``: the fused fp16 path the
  default stack runs -- fp32 arithmetic inside each fused step with ONE rounding to fp16 per
  output; ``resgate_ln`` normalises the *rounded* residual (``:179``); the transition residual
  is ``mx.addmm(z, s, w3)`` (one rounding of ``z + s @ w3``).

Rounding points of the fp16 path (each ``r16`` below is one fp16 rounding, as the reference's
fp16 arrays are):  ``n = r16(LN(z))``; ``proj = r16(n @ w_in)`` (MLX fp16 GEMM: fp32 accumulate,
fp16 out); ``a, b = r16(sig * sigmoid(gate) * mask)`` (gate_cf); ``x = r16(contraction)``;
``m = r16(LN_mix(x))`` (ln_cf_to_cl); ``mixed = r16(m @ w_emit)``; ``g = r16(n @ w_gate)``;
``z' = r16(z + mixed * sigmoid(g))`` (resgate_ln).  Optional biases (not in the reference,
which asserts they are absent: ``fast_trunk.py:53,59``) are added in fp32 before the rounding
of the GEMM they belong to.

Parity anchoring: ``tests/golden/make_golden.py`` executes the reference's own
``mlx_trunk.py`` / ``mlx_trunk_kernels.py`` over a numpy stand-in for MLX 0.32.3 (absent from
this image) and commits the outputs; ``tests/test_oracle_golden.py`` checks this module
against them.  The stand-in restates MLX's primitives, so the pin covers the reference's
orchestration (weight extraction, orientation, eps, rounding points) and not MLX's own
kernels or Apple-GPU arithmetic.
"""

from __future__ import annotations

import math

import torch

EPS = 1e-5  # mlx_trunk.py:31
CONTRACT_SCALE = 256.0  # mlx_trunk.py:33
MIX_EPS_FP16 = EPS / CONTRACT_SCALE**2  # mlx_trunk.py:114


def r16(x: torch.Tensor) -> torch.Tensor:
    """One rounding to fp16, returned as fp32 (the value an fp16 array holds)."""
    return x.to(torch.float16).to(torch.float32)


def layer_norm(x: torch.Tensor, w, b, eps: float) -> torch.Tensor:
    """LayerNorm over the last dim with fp32 statistics, two-pass (mean, then centred
    variance) as the reference's Metal kernels compute it (mlx_trunk_kernels.py:140-145)."""
    x = x.to(torch.float32)
    mean = x.mean(-1, keepdim=True)
    v = x - mean
    var = (v * v).mean(-1, keepdim=True)
    y = v * torch.rsqrt(var + eps)
    return y * w.to(torch.float32) + b.to(torch.float32)


def sigmoid(x: torch.Tensor) -> torch.Tensor:
    return 1.0 / (1.0 + torch.exp(-x))


# --------------------------------------------------------------------------------------
# weights (mlx_trunk.py:40-69)
# --------------------------------------------------------------------------------------


def trimul_params(tri, fp16: bool = True, biases: dict | None = None) -> dict:
    """Weights of one tri-mul in the reference's orientation (``x @ W``), fp32 tensors.

    ``tri`` is a module with ``_engine.{latent_channels, norm_start, proj_bundle, norm_mix,
    proj_emit, proj_gate}`` (mlx_trunk.py:41-55).  In fp16 mode the signal-a columns are
    divided by 256 and every weight is rounded to fp16 (``_mx(t, float16)``)."""
    eng = tri._engine
    c = eng.latent_channels
    assert eng.proj_bundle.weight.shape[0] == 4 * c
    w_in = eng.proj_bundle.weight.detach().float().T.clone()
    b_in = None
    if biases is not None and biases.get("b_in") is not None:
        b_in = biases["b_in"].detach().float().clone()
    if fp16:
        w_in[:, :c] /= CONTRACT_SCALE
        if b_in is not None:
            b_in[:c] /= CONTRACT_SCALE
    rnd = r16 if fp16 else (lambda t: t.float())
    p = {
        "c": c,
        "ln_in_w": rnd(eng.norm_start.weight.detach().float()),
        "ln_in_b": rnd(eng.norm_start.bias.detach().float()),
        "w_in": rnd(w_in),
        "ln_mix_w": rnd(eng.norm_mix.weight.detach().float()),
        "ln_mix_b": rnd(eng.norm_mix.bias.detach().float()),
        "w_emit": rnd(eng.proj_emit.weight.detach().float().T),
        "w_out_gate": rnd(eng.proj_gate.weight.detach().float().T),
        "b_in": None if b_in is None else b_in,
        "b_emit": None,
        "b_gate": None,
    }
    if biases is not None:
        for k in ("b_emit", "b_gate"):
            if biases.get(k) is not None:
                p[k] = biases[k].detach().float().clone()
    return p


def transition_params(tr, fp16: bool = True) -> dict:
    rnd = r16 if fp16 else (lambda t: t.float())
    return {
        "ln_w": rnd(tr.norm.weight.detach().float()),
        "ln_b": rnd(tr.norm.bias.detach().float()),
        "w12": rnd(tr.ffn.w12.weight.detach().float().T),
        "w3": rnd(tr.ffn.w3.weight.detach().float().T),
    }


def trunk_params(folding_trunk, fp16: bool = True) -> list:
    """mlx_trunk.py:58-69 for every block."""
    return [
        {
            "out": trimul_params(blk.tri_mul_out, fp16),
            "in": trimul_params(blk.tri_mul_in, fp16),
            **transition_params(blk.pair_transition, fp16),
        }
        for blk in folding_trunk.blocks
    ]


# --------------------------------------------------------------------------------------
# tri-mul
# --------------------------------------------------------------------------------------


def _contract(a: torch.Tensor, b: torch.Tensor, outgoing: bool) -> torch.Tensor:
    """a, b: [B, c, L, L] -> x [B, c, L, L] (mlx_trunk.py:84-88)."""
    B, c, L, _ = a.shape
    a3 = a.reshape(B * c, L, L)
    b3 = b.reshape(B * c, L, L)
    if outgoing:
        x = torch.bmm(a3, b3.transpose(1, 2))
    else:
        x = torch.bmm(a3.transpose(1, 2), b3)
    return x.reshape(B, c, L, L)


def project_gate_fp16(p: dict, z: torch.Tensor, mask):
    """The first fused step (mlx_trunk_kernels.py:214-216, gate_cf :47-80) on a [B, rows, cols,
    c_z] grid: returns n and channel-major a, b [B, c, rows, cols] (fp16 values as fp32)."""
    c = p["c"]
    z = r16(z.float())
    n = r16(layer_norm(z, p["ln_in_w"], p["ln_in_b"], EPS))
    proj = n @ p["w_in"]
    if p.get("b_in") is not None:
        proj = proj + p["b_in"]
    proj = r16(proj)
    m = None if mask is None else r16(mask.float())

    def gated(lo):
        v = proj[..., lo:lo + c] / (1.0 + torch.exp(-proj[..., 2 * c + lo:3 * c + lo]))  # gate_cf :62
        if m is not None:
            v = v * m[..., None]
        return r16(v).permute(0, 3, 1, 2).contiguous()

    return n, gated(0), gated(c)


def emit_residual_fp16(p: dict, z: torch.Tensor, x: torch.Tensor, mix_eps: float = MIX_EPS_FP16):
    """The last fused step (ln_cf_to_cl, @ w_emit, n @ w_out_gate, resgate_ln:
    mlx_trunk_kernels.py:221-227) on a [B, rows, cols, c_z] grid with x [B, c, rows, cols]."""
    z = r16(z.float())
    n = r16(layer_norm(z, p["ln_in_w"], p["ln_in_b"], EPS))
    mixn = r16(layer_norm(r16(x.float()).permute(0, 2, 3, 1), p["ln_mix_w"], p["ln_mix_b"], mix_eps))
    mixed = mixn @ p["w_emit"]
    if p.get("b_emit") is not None:
        mixed = mixed + p["b_emit"]
    mixed = r16(mixed)
    g = n @ p["w_out_gate"]
    if p.get("b_gate") is not None:
        g = g + p["b_gate"]
    g = r16(g)
    return r16(z + mixed / (1.0 + torch.exp(-g))), {"mixn": mixn, "mixed": mixed, "g": g}  # resgate_ln :176-177


def trimul_fp16(p: dict, z: torch.Tensor, mask, outgoing: bool, mix_eps: float = MIX_EPS_FP16,
                return_intermediates: bool = False):
    """One fused fp16 triangle update, returning ``z + update`` rounded to fp16 (as fp32).

    z: [B, L, L, c_z] (values representable in fp16); mask: [B, L, L] or None.
    Follows mlx_trunk_kernels.py:210-229 with ``use=ALL`` (the default stack's path)."""
    n, a, b = project_gate_fp16(p, z, mask)
    x = r16(_contract(a, b, outgoing))
    z_new, it = emit_residual_fp16(p, z, x, mix_eps)
    if return_intermediates:
        return z_new, {"n": n, "a": a, "b": b, "x": x, **it}
    return z_new


def trimul_fp32(p: dict, z: torch.Tensor, mask, outgoing: bool, eps_mix: float = EPS,
                dtype=torch.float32) -> torch.Tensor:
    """The unrounded update ``z + trimul(z)`` computed in ``dtype`` (mlx_trunk.py:79-90 with
    fp32 params).  ``p`` must come from ``trimul_params(..., fp16=False)`` (no pre-scale)."""
    cast = lambda t: None if t is None else t.to(dtype)  # noqa: E731
    z = z.to(dtype)
    c = p["c"]
    n = _ln(z, p["ln_in_w"], p["ln_in_b"], EPS, dtype)
    proj = n @ cast(p["w_in"])
    if p.get("b_in") is not None:
        proj = proj + cast(p["b_in"])
    mk = None if mask is None else mask.to(dtype)

    def gated(lo):
        v = proj[..., lo:lo + c] * torch.sigmoid(proj[..., 2 * c + lo:3 * c + lo])
        if mk is not None:
            v = v * mk[..., None]
        return v.permute(0, 3, 1, 2).contiguous()

    a, b = gated(0), gated(c)
    x = _contract(a, b, outgoing)
    mixn = _ln(x.permute(0, 2, 3, 1), p["ln_mix_w"], p["ln_mix_b"], eps_mix, dtype)
    mixed = mixn @ cast(p["w_emit"])
    if p.get("b_emit") is not None:
        mixed = mixed + cast(p["b_emit"])
    g = n @ cast(p["w_out_gate"])
    if p.get("b_gate") is not None:
        g = g + cast(p["b_gate"])
    return z + mixed * torch.sigmoid(g)


def _ln(x, w, b, eps, dtype):
    x = x.to(dtype)
    mean = x.mean(-1, keepdim=True)
    v = x - mean
    var = (v * v).mean(-1, keepdim=True)
    return v / torch.sqrt(var + eps) * w.to(dtype) + b.to(dtype)


# --------------------------------------------------------------------------------------
# a slab of rows of one update, for lengths whose full update is too slow on the CPU
# --------------------------------------------------------------------------------------


def _gated_half(p: dict, z: torch.Tensor, mask, half: int, exact: bool, exact_dtype=torch.float64) -> torch.Tensor:
    """One gated operand (half 0: a, half 1: b) on a [B, rows, cols, c_z] grid, channel-major
    [B, c, rows, cols]: only the projection columns of that operand (its signal and gate
    columns), with the same arithmetic as :func:`project_gate_fp16` (``exact``: float64 and no
    rounding, as :func:`trimul_fp32`)."""
    c = p["c"]
    cols = list(range(half * c, half * c + c)) + list(range(2 * c + half * c, 3 * c + half * c))
    if exact:
        dt = exact_dtype
        n = _ln(z, p["ln_in_w"], p["ln_in_b"], EPS, dt)
        proj = n @ p["w_in"][:, cols].to(dt)
        if p.get("b_in") is not None:
            proj = proj + p["b_in"][cols].to(dt)
        v = proj[..., :c] * torch.sigmoid(proj[..., c:])
        if mask is not None:
            v = v * mask.to(dt)[..., None]
        return v.permute(0, 3, 1, 2).contiguous()
    z = r16(z.float())
    n = r16(layer_norm(z, p["ln_in_w"], p["ln_in_b"], EPS))
    proj = n @ p["w_in"][:, cols]
    if p.get("b_in") is not None:
        proj = proj + p["b_in"][cols]
    proj = r16(proj)
    v = proj[..., :c] / (1.0 + torch.exp(-proj[..., c:]))
    if mask is not None:
        v = v * r16(mask.float())[..., None]
    return r16(v).permute(0, 3, 1, 2).contiguous()


def trimul_rows(p: dict, z: torch.Tensor, mask, outgoing: bool, rows, exact: bool = False,
                mix_eps: float | None = None, chunk: int = 64, exact_dtype=torch.float64):
    """Rows of ``z + trimul(z)`` without forming the whole update: ``rows`` is a range of i, or a
    list of ranges (slabs) that share one projection of b.

    Outgoing, row i needs a[:, i, :] (the projection of z's row i) and all of b; incoming,
    ``x[d, i, j] = sum_k a[d, k, i] b[d, k, j]`` needs a[:, :, i] (the projection of z's column
    i) and all of b.  b is projected in chunks of ``chunk`` rows and kept in fp16 (exact: its
    values are fp16 roundings) or, with ``exact``, in fp32 (float64 arithmetic otherwise; the
    fp32 storage of b is 2^13 times finer than the fp16 errors this reference measures).
    ``z`` may be fp16 or fp32.  With ``exact``, ``p`` comes from ``trimul_params(..., fp16=False)``
    and the arithmetic is ``exact_dtype`` (float64 by default; float32 is 2^13 times finer than
    the fp16 errors it measures, and much faster for L in the thousands).
    Returns [B, len(rows), L, c_z] per slab, fp32 holding fp16 values, or ``exact_dtype``."""
    single = isinstance(rows, range)
    slabs = [rows] if single else list(rows)
    B, L = z.shape[0], z.shape[1]
    c = p["c"]
    store = torch.float32 if exact else torch.float16
    b_all = torch.empty(B, c, L, L, dtype=store)
    for s in range(0, L, chunk):
        e = min(L, s + chunk)
        b_all[:, :, s:e] = _gated_half(p, z[:, s:e], None if mask is None else mask[:, s:e], 1, exact,
                                       exact_dtype).to(store)
    dt = exact_dtype if exact else torch.float32
    outs = []
    for sl in slabs:
        r0, r1 = sl[0], sl[-1] + 1
        if outgoing:
            a_r = _gated_half(p, z[:, r0:r1], None if mask is None else mask[:, r0:r1], 0, exact,
                              exact_dtype)  # [B, c, R, L]
        else:
            a_r = _gated_half(p, z[:, :, r0:r1], None if mask is None else mask[:, :, r0:r1], 0, exact,
                              exact_dtype)
            a_r = a_r.transpose(2, 3)  # [B, c, R, L]: a[d, k, i] as rows i
        x = torch.empty(B, c, r1 - r0, L, dtype=dt)
        for d0 in range(0, c, 16):
            d1 = min(c, d0 + 16)
            bb = b_all[:, d0:d1].to(dt).reshape(B * (d1 - d0), L, L)
            ar = a_r[:, d0:d1].to(dt).reshape(B * (d1 - d0), r1 - r0, L)
            xr = torch.bmm(ar, bb.transpose(1, 2)) if outgoing else torch.bmm(ar, bb)
            x[:, d0:d1] = xr.reshape(B, d1 - d0, r1 - r0, L)
        zr = z[:, r0:r1]
        if exact:
            n = _ln(zr, p["ln_in_w"], p["ln_in_b"], EPS, dt)
            mixn = _ln(x.permute(0, 2, 3, 1), p["ln_mix_w"], p["ln_mix_b"], EPS if mix_eps is None else mix_eps, dt)
            mixed = mixn @ p["w_emit"].to(dt)
            if p.get("b_emit") is not None:
                mixed = mixed + p["b_emit"].to(dt)
            g = n @ p["w_out_gate"].to(dt)
            if p.get("b_gate") is not None:
                g = g + p["b_gate"].to(dt)
            outs.append(zr.to(dt) + mixed * torch.sigmoid(g))
        else:
            out, _ = emit_residual_fp16(p, zr, r16(x), MIX_EPS_FP16 if mix_eps is None else mix_eps)
            outs.append(out)
    return outs[0] if single else outs


def ulps16(ref: torch.Tensor, test: torch.Tensor) -> float:
    """Largest |test - ref| in fp16 ulps at the reference tensor's scale (the ulp of max |ref|)."""
    scale = max(float(ref.abs().max()), 2.0**-14)
    ulp = 2.0 ** (math.floor(math.log2(scale)) - 10)
    return float((test.double() - ref.double()).abs().max()) / ulp


def parity(exact: torch.Tensor, ref16: torch.Tensor, test: torch.Tensor) -> dict:
    """The parity figures of a CUDA result ``test``: its error against the exact (float64)
    update, the fp16 oracle's own error against the same (e_ref), and its distance from the
    oracle in fp16 ulps.  The acceptance rule is e_cuda <= 2 * e_ref + 1e-3 (max-abs and rel-L2)."""
    e = error_stats(exact, test)
    er = error_stats(exact, ref16)
    ok = (e["finite"] and e["max_abs"] <= 2 * er["max_abs"] + 1e-3 and e["rel_l2"] <= 2 * er["rel_l2"] + 1e-3)
    return {"max_abs": e["max_abs"], "rel_l2": e["rel_l2"], "e_ref_max_abs": er["max_abs"],
            "e_ref_rel_l2": er["rel_l2"], "max_ulps": ulps16(ref16, test), "within_tolerance": bool(ok)}


# --------------------------------------------------------------------------------------
# transition, block, trunk (mlx_trunk.py:93-109, mlx_trunk_kernels.py:232-249)
# --------------------------------------------------------------------------------------


def transition_fp16(p: dict, z: torch.Tensor, activation: str = "swiglu") -> torch.Tensor:
    """``z + ffn(LN(z))`` with the fused path's rounding points (mlx_trunk_kernels.py:236-239).

    swiglu: ``x = r16(h @ w12)``; ``s = r16(r16(x1 * r16(sigmoid(x1))) * x2)`` (three fp16
    element-wise ops); ``z' = r16(z + s @ w3)`` (``mx.addmm``).  relu (synthetic configs
    only): ``s = r16(relu(h @ w1))``."""
    z = r16(z.float())
    h = r16(layer_norm(z, p["ln_w"], p["ln_b"], EPS))
    x = r16(h @ p["w12"])
    if activation == "swiglu":
        x1, x2 = x.chunk(2, dim=-1)
        s = r16(r16(x1 * r16(sigmoid(x1))) * x2)
    elif activation == "relu":
        s = torch.relu(x)
    else:
        raise ValueError(activation)
    return r16(z + s @ p["w3"])


def block_fp16(p: dict, z, mask, mix_eps: float = MIX_EPS_FP16, activation: str = "swiglu"):
    z = trimul_fp16(p["out"], z, mask, True, mix_eps)
    z = trimul_fp16(p["in"], z, mask, False, mix_eps)
    return transition_fp16(p, z, activation)


def trunk_fp16(params: list, z, mask=None, mix_eps: float = MIX_EPS_FP16, activation: str = "swiglu"):
    """trunk_forward (mlx_trunk_kernels.py:242-249): cast in, blocks, fp32 out."""
    z = r16(z.float())
    for p in params:
        z = block_fp16(p, z, mask, mix_eps, activation)
    return z.float()


# --------------------------------------------------------------------------------------
# downstream agreement (var_adaptive_loops.py:38-46)
# --------------------------------------------------------------------------------------

_EDGES = torch.linspace(2.0, 52.0, 127)
DISTO_CENTERS = torch.cat([_EDGES[:1] - 0.2, (_EDGES[1:] + _EDGES[:-1]) / 2, _EDGES[-1:] + 0.2])


def expected_distance(z: torch.Tensor, head_w: torch.Tensor, head_b: torch.Tensor) -> torch.Tensor:
    """Distogram head expected distance per pair (Å) on ``z + z^T`` (var_adaptive_loops.py:43-46)."""
    z = z.float()
    logits = (z + z.transpose(-2, -3)) @ head_w.float().T + head_b.float()
    return logits.softmax(-1) @ DISTO_CENTERS


def disto_p95(z_ref: torch.Tensor, z_test: torch.Tensor, head_w, head_b) -> float:
    """95th percentile of |Δ expected distance| between two pair tensors (Å)."""
    d = (expected_distance(z_test, head_w, head_b) - expected_distance(z_ref, head_w, head_b)).abs()
    return float(d.flatten().quantile(0.95)) if d.numel() < 16_000_000 else float(
        d.flatten()[:: max(1, d.numel() // 8_000_000)].quantile(0.95))


def error_stats(ref: torch.Tensor, test: torch.Tensor) -> dict:
    ref = ref.double()
    test = test.double()
    diff = (test - ref)
    return {
        "max_abs": float(diff.abs().max()),
        "rel_l2": float(diff.norm() / ref.norm().clamp_min(1e-30)),
        "finite": bool(torch.isfinite(test).all()),
    }


def flops_per_cell(L: int, c_z: int = 128, c: int = 128) -> int:
    """Algorithmic FLOPs per pair-cell of one tri-mul: projections (4c + c_z outputs over
    c_z inputs), emit (c -> c_z) and the contraction (2*c*L)."""
    return 2 * c_z * (4 * c + c_z) + 2 * c * c_z + 2 * c * L


def _selfcheck():  # pragma: no cover - manual
    torch.manual_seed(0)
    print(math.isfinite(MIX_EPS_FP16))


if __name__ == "__main__":  # pragma: no cover
    _selfcheck()
