"""CPU oracle for the diffusion head's per-fold pair conditioning (TEST INFRASTRUCTURE ONLY).

The parity tests compare ``tmu_pair_cond`` (K6 + K4 row mode) against this module; nothing in
the product package imports it.

It restates, in plain PyTorch on the CPU, ``pair_biases`` of the reference's diffusion sampler
(abhi0raj/esmfold2-mlx, paths relative to ``src/esmfold2_mlx/``) in the precision of its adopted
stack ``var_mlx_diffusion16`` (``tok16 + cond16 + pair16``):

* ``mlx_diffusion.py:51-52,85-92``  weights: ``z_input_norm`` (LN), ``z_proj``, the
  ``z_transitions`` (LN -> silu(h @ a) * (h @ b) -> @ out), and every token block's pair bias
  folded into one matrix: ``bias_w = cat_i(pair_norm_i.weight[:, None] * pair_bias_proj_i.weight^T)``,
  ``bias_b = cat_i(pair_bias_proj_i(pair_norm_i.bias))`` (computed in fp32 torch).
* ``mlx_diffusion16.py:224-227``  pair16 casts ``proj``, ``bias_w``, ``bias_b`` and the
  transitions' ``a``, ``b``, ``out`` to fp16; LayerNorm parameters stay fp32.
* ``mlx_diffusion16.py:50-57,64-67,81-87``  ``_mm(x, w) = x.astype(w.dtype) @ w`` (fp16 GEMM,
  fp32 accumulation, fp16 result); ``_transition``; ``pair_biases``; the output layout
  ``bias.reshape(B, L, L, nb, H).transpose(3, 0, 4, 1, 2)`` (``mlx_diffusion.py:259``).

Rounding points (``r16`` = one fp16 rounding): ``h = r16(LN(cat(z_trunk, rel_pos)))``,
``z = r16(h @ proj)`` then fp32; per transition ``hh = r16(LN(z))``, ``xa = r16(hh @ a)``,
``xb = r16(hh @ b)``, ``s = r16(r16(xa * r16(sigmoid(xa))) * xb)``, ``z = z + r16(s @ out)``
(fp32 residual); ``bias = r16(r16(r16(LN(z)) @ bias_w) + bias_b)`` with an affine-free LN.

Parity pin: ``tests/golden/conditioning_golden.npz``, made by
``tests/golden/make_golden_conditioning.py`` running the reference's ``pair_biases``
(``mlx_diffusion16.py:81-87``) unmodified over a numpy stand-in for MLX 0.32.3; checked by
``tests/test_oracle_golden_conditioning.py`` (<= 2 fp16 ulps at the tensor's scale, rel-L2 <= 1e-3).
The reference's own tests cover this path only through end-to-end atom coordinates that need the
esm package, the checkpoint and MLX (all absent).
"""

from __future__ import annotations

import torch

from .trimul_oracle import layer_norm, r16, sigmoid

LN_EPS = 1e-5  # mlx_diffusion.py:30


def pair_cond_params(head, pair16: bool = True) -> dict:
    """The ``pair`` weights of ``diffusion_params`` (``mlx_diffusion.py:85-92``), fp16 per pair16."""
    dm = head.diffusion_module
    cond, blocks = dm.conditioning, dm.token_transformer.attn_blocks
    rnd = r16 if pair16 else (lambda t: t.float())
    f = lambda t: t.detach().float()  # noqa: E731
    with torch.no_grad():
        bias_w = torch.cat([f(b.pair_norm.weight)[:, None] * f(b.pair_bias_proj.weight).T for b in blocks], -1)
        bias_b = torch.cat([b.pair_bias_proj(b.pair_norm.bias).detach().float() for b in blocks], -1)
    return {
        "ln_w": f(cond.z_input_norm.weight), "ln_b": f(cond.z_input_norm.bias),
        "proj": rnd(f(cond.z_proj.weight).T),
        "transitions": [{"ln_w": f(t.norm.weight), "ln_b": f(t.norm.bias), "a": rnd(f(t.a_proj.weight).T),
                         "b": rnd(f(t.b_proj.weight).T), "out": rnd(f(t.out_proj.weight).T)}
                        for t in cond.z_transitions],
        "bias_w": rnd(bias_w), "bias_b": rnd(bias_b),
        "heads": int(blocks[0].num_heads),
    }


def _mm(x: torch.Tensor, w: torch.Tensor, acc: torch.dtype) -> torch.Tensor:
    """GEMM of fp16-valued operands accumulated in ``acc`` (fp32 as MLX; fp64 to measure how much
    the pipeline's roundings depend on summation order)."""
    return (x.to(acc) @ w.to(acc)).float()


def stage_project(p: dict, z_trunk, rel_pos, acc=torch.float32) -> torch.Tensor:
    """z0 = r16(r16(LN(cat(z_trunk, rel_pos))) @ proj), fp16 values as fp32 (mlx_diffusion16.py:82)."""
    x = torch.cat([z_trunk.float(), rel_pos.float()], -1)
    return r16(_mm(r16(layer_norm(x, p["ln_w"], p["ln_b"], LN_EPS)), p["proj"], acc))


def stage_transition_delta(t: dict, z: torch.Tensor, acc=torch.float32) -> torch.Tensor:
    """r16(s @ out), s the fp16 SwiGLU of r16(LN(z)) (mlx_diffusion16.py:64-67)."""
    hh = r16(layer_norm(z, t["ln_w"], t["ln_b"], LN_EPS))
    xa, xb = r16(_mm(hh, t["a"], acc)), r16(_mm(hh, t["b"], acc))
    s = r16(r16(xa * r16(sigmoid(xa))) * xb)
    return r16(_mm(s, t["out"], acc))


def stage_transition(t: dict, z: torch.Tensor, acc=torch.float32) -> torch.Tensor:
    """z + r16(s @ out): the fp32 residual update (mlx_diffusion16.py:83-84)."""
    return z + stage_transition_delta(t, z, acc)


def stage_bias(p: dict, z: torch.Tensor, acc=torch.float32) -> torch.Tensor:
    """r16(r16(r16(LN(z)) @ bias_w) + bias_b) as [nb, B, H, L, L] (mlx_diffusion16.py:86-87)."""
    c = z.shape[-1]
    hb = r16(layer_norm(z, torch.ones(c), torch.zeros(c), LN_EPS))
    bias = r16(r16(_mm(hb, p["bias_w"], acc)) + p["bias_b"])
    B, L = z.shape[0], z.shape[1]
    return bias.reshape(B, L, L, -1, p["heads"]).permute(3, 0, 4, 1, 2).contiguous()


def pair_biases_fp16(p: dict, z_trunk: torch.Tensor, rel_pos: torch.Tensor, acc=torch.float32) -> torch.Tensor:
    """[nb, B, H, L, L] pair biases (fp16 values as fp32) for fp32 ``z_trunk`` / ``rel_pos``."""
    z = stage_project(p, z_trunk, rel_pos, acc)
    for t in p["transitions"]:
        z = stage_transition(t, z, acc)
    return stage_bias(p, z, acc)
