"""The parcae step of the 6B release model's recycling loop on B200 (``tmu_parcae_step``):
``z' = a * z + LN(z_init + refined) @ B^T`` in fp32, ``refined`` being the lm_encoder trunk's
output for this step.

Reference (``src/esmfold2_mlx/var_6b_mlx_loop.py``): ``_step`` (``:67-71``), which runs it in fp32
MLX between the lm_encoder and the folding trunk; ``MLXLoop.run`` passes ``a`` and ``b_mat``
(``:157,169``) and the LayerNorm is ``model.parcae_input_norm`` (eps 1e-5, ``:129-130``).  The GEMM
runs on the tensor cores at fp32 accuracy: ``B`` is split once into three bf16 parts, the
LayerNorm output likewise inside the kernel, and the six partial products that carry 24
significant bits accumulate in fp32.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib
from .ops import _ptr, _stream_ptr, check_status as _check_status, new_status


def split_bf16x3(m: torch.Tensor) -> torch.Tensor:
    """[m0 | m1 | m2] bf16 along the last dim with m = m0 + m1 + m2 exactly (fp32 ``m``):
    m0 = bf16(m), m1 = bf16(m - m0), m2 = bf16(m - m0 - m1); each remainder is exact in fp32, and
    the split is exact while m2 stays a normal bf16 (|m| >= 2^-110)."""
    m = m.float()
    m0 = m.to(torch.bfloat16)
    r = m - m0.float()
    m1 = r.to(torch.bfloat16)
    m2 = (r - m1.float()).to(torch.bfloat16)
    return torch.cat([m0, m1, m2], -1).contiguous()


@dataclass
class ParcaeWeights:
    """The step's parameters in the layouts of ``tmu_parcae_step``."""

    c_z: int
    ln_w: torch.Tensor
    ln_b: torch.Tensor
    a: torch.Tensor
    b_split: torch.Tensor
    _struct: _lib.TmuParcaeWeights | None = field(default=None, repr=False)

    @classmethod
    def from_model(cls, model, a, b_mat, device="cuda") -> "ParcaeWeights":
        """``model.parcae_input_norm`` and the loop's ``a`` (scalar or [c_z]) and ``b_mat`` [c_z, c_z]."""
        norm = model.parcae_input_norm
        if abs(float(norm.eps) - 1e-5) > 1e-12:
            raise ValueError("parcae_input_norm.eps must be 1e-5")  # var_6b_mlx_loop.py:130
        c = int(norm.weight.shape[0])
        f32 = lambda t: torch.as_tensor(t).detach().float().cpu()  # noqa: E731
        av = f32(a).reshape(-1)
        av = av.expand(c).contiguous() if av.numel() == 1 else av
        if av.numel() != c or tuple(b_mat.shape) != (c, c):
            raise ValueError("a must be a scalar or [c_z] and b_mat [c_z, c_z]")
        return cls(c_z=c, ln_w=f32(norm.weight).to(device), ln_b=f32(norm.bias).to(device), a=av.to(device),
                   b_split=split_bf16x3(f32(b_mat)).to(device))

    @property
    def struct(self) -> _lib.TmuParcaeWeights:
        if self._struct is None:
            self._struct = _lib.TmuParcaeWeights(_ptr(self.ln_w), _ptr(self.ln_b), _ptr(self.a), _ptr(self.b_split))
        return self._struct


def parcae_step(z: torch.Tensor, z_init: torch.Tensor, refined: torch.Tensor, w: ParcaeWeights,
                out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                status: torch.Tensor | None = None, check_status: bool = False) -> torch.Tensor:
    """``a * z + LN(z_init + refined) @ B^T`` for fp32 [B, L, L, c_z] tensors (``out`` may be ``z``).

    The kernels record a device-side error (a bounded wait that gave up) in ``status``; with
    ``check_status`` the call synchronises and raises ``TmuError`` if one was recorded, otherwise
    the caller reads ``status`` (``ops.read_status``) when it next synchronises."""
    for name, t in (("z", z), ("z_init", z_init), ("refined", refined)):
        if not t.is_cuda or t.dtype != torch.float32 or t.dim() != 4 or not t.is_contiguous() or t.shape != z.shape:
            raise ValueError(f"{name} must be a contiguous CUDA fp32 tensor shaped like z")
    B, L, c = z.shape[0], z.shape[1], z.shape[3]
    if c != w.c_z or z.shape[2] != L:
        raise ValueError(f"z must be [B, L, L, {w.c_z}]")
    lib = _lib.load()
    out = torch.empty_like(z) if out is None else out
    need = int(lib.tmu_parcae_workspace_bytes(B, L, c))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=z.device)
    status = new_status(z.device) if status is None else status
    _lib.check(lib.tmu_parcae_step(_ptr(z), _ptr(z_init), _ptr(refined), ctypes.byref(w.struct), _ptr(out), B, L, c,
                                   _ptr(workspace), workspace.numel(), _ptr(status), _stream_ptr(z.device)),
               "tmu_parcae_step")
    if check_status:
        _check_status(status, "tmu_parcae_step")
    return out


def loop_step(lm_encoder, folding_trunk, w: ParcaeWeights, lz: torch.Tensor, z: torch.Tensor, z_init: torch.Tensor,
              mask=None, workspace: torch.Tensor | None = None, check_status: bool = False) -> torch.Tensor:
    """One step of the 6B recycling loop as ``_step`` composes it (``var_6b_mlx_loop.py:67-71``):
    ``refined = lm_encoder(lz)``, the parcae recurrence, then the folding trunk.  Both trunks are
    modules with the reference trunk call (``CUDAFoldingTrunk``); every tensor stays on the GPU."""
    refined = lm_encoder(lz, pair_attention_mask=mask).float().contiguous()
    zn = parcae_step(z.float().contiguous(), z_init.float().contiguous(), refined, w, workspace=workspace,
                     check_status=check_status)
    return folding_trunk(zn, pair_attention_mask=mask)
