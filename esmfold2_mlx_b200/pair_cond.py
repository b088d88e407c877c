"""Per-fold pair conditioning of the diffusion head on B200: ``pair_biases`` as one call of
``tmu_pair_cond`` (LayerNorm pass + K6 projection, LayerNorm pass + K4 for each transition,
LayerNorm pass + K6 for the folded pair-bias GEMM).

Each GEMM kernel reads its LayerNorm output from a row LayerNorm pass (many warps per SM,
coalesced), and the fp32 residual stream between the transitions is kept as its fp16 terms.

Reference (``src/esmfold2_mlx/``): ``mlx_diffusion16.pair_biases`` (``mlx_diffusion16.py:81-87``)
in the pair16 precision of the adopted ``var_mlx_diffusion16`` stack, weights as
``diffusion_params`` copies them (``mlx_diffusion.py:85-92``), call site ``MlxDiffusion._context``
(``mlx_diffusion.py:322-324``).  The result is the ``[nb, B, H, L, L]`` fp16 tensor the token
transformer's attention takes as its mask (``mlx_diffusion.py:259,369``).  The diffusion sampler
itself (atom transformer, token transformer, Kabsch, Euler steps) is not part of this package.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib
from .ops import _ptr, _stream_ptr, new_status
from .ops import check_status as check_status_fn


@dataclass
class PairCondWeights:
    """Device-resident weights of the pair conditioning in the layouts of ``tmu_pair_cond``:
    LayerNorm parameters fp32; ``proj`` [c_pair, c_in], each transition's ``w12`` = [a; b] rows
    [2h, c_pair] and ``w3`` [c_pair, h], ``bias_w`` [nb*H, c_pair] fp16 (nn.Linear layouts, the
    reference keeps the same matrices transposed); ``bias_b`` fp16 [nb*H]."""

    c_in: int
    c_pair: int
    hidden: int
    heads: int
    n_bias: int
    tensors: dict
    _struct: _lib.TmuPairCondWeights | None = field(default=None, repr=False)
    _trans: ctypes.Array | None = field(default=None, repr=False)

    @classmethod
    def from_head(cls, head, device="cuda") -> "PairCondWeights":
        """Copy the weights out of a diffusion head (``head.diffusion_module``), folding every
        token block's ``pair_norm`` affine into its ``pair_bias_proj`` in fp32 first
        (``mlx_diffusion.py:85-89``), then rounding the matrices to fp16 (pair16)."""
        dm = head.diffusion_module
        cond, blocks = dm.conditioning, dm.token_transformer.attn_blocks
        f32 = lambda t: t.detach().float().cpu()  # noqa: E731
        dev32 = lambda t: f32(t).to(device).contiguous()  # noqa: E731
        dev16 = lambda t: f32(t).to(torch.float16).to(device).contiguous()  # noqa: E731
        with torch.no_grad():
            bias_w = torch.cat([f32(b.pair_norm.weight)[:, None] * f32(b.pair_bias_proj.weight).T for b in blocks], -1)
            bias_b = torch.cat([b.pair_bias_proj(b.pair_norm.bias).detach().float().cpu() for b in blocks], -1)
        trans = [{"ln_w": dev32(t.norm.weight), "ln_b": dev32(t.norm.bias),
                  "w12": dev16(torch.cat([f32(t.a_proj.weight), f32(t.b_proj.weight)], 0)),
                  "w3": dev16(t.out_proj.weight)} for t in cond.z_transitions]
        hidden = int(cond.z_transitions[0].a_proj.weight.shape[0]) if len(trans) else 64
        tensors = {"ln_w": dev32(cond.z_input_norm.weight), "ln_b": dev32(cond.z_input_norm.bias),
                   "proj": dev16(cond.z_proj.weight), "bias_w": dev16(bias_w.T), "bias_b": dev16(bias_b),
                   "transitions": trans}
        return cls(c_in=int(cond.z_proj.weight.shape[1]), c_pair=int(cond.z_proj.weight.shape[0]), hidden=hidden,
                   heads=int(blocks[0].num_heads), n_bias=int(bias_b.numel()), tensors=tensors)

    @property
    def struct(self) -> _lib.TmuPairCondWeights:
        if self._struct is None:
            t = self.tensors
            arr = (_lib.TmuCondTransitionWeights * max(1, len(t["transitions"])))()
            for i, tr in enumerate(t["transitions"]):
                arr[i] = _lib.TmuCondTransitionWeights(_ptr(tr["ln_w"]), _ptr(tr["ln_b"]), _ptr(tr["w12"]),
                                                        _ptr(tr["w3"]))
            self._trans = arr
            self._struct = _lib.TmuPairCondWeights(_ptr(t["ln_w"]), _ptr(t["ln_b"]), _ptr(t["proj"]),
                                                   len(t["transitions"]), arr, _ptr(t["bias_w"]), _ptr(t["bias_b"]))
        return self._struct


def workspace_bytes(B: int, L: int, c_in: int, c_pair: int, n_transitions: int) -> int:
    """Scratch for z0 and each transition's fp16 output (the fp32 residual stream's terms) and
    the LayerNorm output buffer."""
    return int(_lib.load().tmu_pair_cond_workspace_bytes(B, L, c_in, c_pair, n_transitions))


def pair_biases(w: PairCondWeights, z_trunk: torch.Tensor, rel_pos: torch.Tensor, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None, status: torch.Tensor | None = None,
                check_status: bool = False) -> torch.Tensor:
    """The token transformer's pair biases ``[nb, B, H, L, L]`` fp16 from fp32 ``z_trunk``
    [B, L, L, c_trunk] and ``rel_pos`` [B, L, L, c_rel] (``mlx_diffusion16.py:81-87``).

    A device-side error (a bounded wait that gave up) lands in ``status``; with ``check_status``
    the call synchronises and raises ``TmuError`` if one was recorded."""
    for name, t in (("z_trunk", z_trunk), ("rel_pos", rel_pos)):
        if not t.is_cuda or t.dtype != torch.float32 or t.dim() != 4 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous CUDA fp32 [B, L, L, C] tensor")
    B, L = z_trunk.shape[0], z_trunk.shape[1]
    if rel_pos.shape[:3] != z_trunk.shape[:3] or z_trunk.shape[2] != L:
        raise ValueError("z_trunk and rel_pos must share [B, L, L]")
    if z_trunk.shape[3] + rel_pos.shape[3] != w.c_in:
        raise ValueError(f"c_trunk + c_rel must be {w.c_in}")
    lib = _lib.load()
    dev = z_trunk.device
    nb = w.n_bias // w.heads
    out = torch.empty(nb, B, w.heads, L, L, dtype=torch.float16, device=dev) if out is None else out
    need = workspace_bytes(B, L, w.c_in, w.c_pair, len(w.tensors["transitions"]))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    status = new_status(dev) if status is None else status
    _lib.check(lib.tmu_pair_cond(_ptr(z_trunk), _ptr(rel_pos), ctypes.byref(w.struct), B, L, z_trunk.shape[3],
                                 rel_pos.shape[3], w.c_pair, w.hidden, w.n_bias, w.heads, _ptr(out), _ptr(workspace),
                                 workspace.numel(), _ptr(status), _stream_ptr(dev)), "tmu_pair_cond")
    if check_status:
        check_status_fn(status, "tmu_pair_cond")
    return out
