"""Torch-facing wrappers over the C ABI: one function per kernel stage plus the whole update.

These mirror the reference's operator interface for the triangle update
(``src/esmfold2_mlx/mlx_trunk_kernels.py``): ``gate_cf`` + the input projection
(:85-97, :214-216) -> :func:`project_gate`; the batched contraction (:219) -> :func:`contract`;
``ln_cf_to_cl`` + ``@ w_emit`` + ``n @ w_out_gate`` + ``resgate_ln`` (:152-160, :195-203,
:221-227) -> :func:`emit_residual`; ``_trimul`` (:210-229) plus its residual -> :func:`trimul`.
Arguments are CUDA tensors; every launch goes on the current torch stream; nothing here falls
back to another implementation -- a failing call raises :class:`TmuError`.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib

EPS = 1e-5  # mlx_trunk.py:31
CONTRACT_SCALE = 256.0  # mlx_trunk.py:33
MIX_EPS_FP16 = EPS / CONTRACT_SCALE**2  # mlx_trunk.py:114


def _stream_ptr(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def row_pitch(L: int) -> int:
    return (L + 7) // 8 * 8


def proj_row_order(c: int) -> list[int]:
    """Packed row order of ``proj_bundle.weight`` used by the projection kernel."""
    lib = _lib.load()
    arr = (ctypes.c_int * (4 * c))()
    _lib.check(lib.tmu_proj_row_order(c, arr), "tmu_proj_row_order")
    return list(arr)


def proj_row_order_py(c: int) -> list[int]:
    """The same order computed in Python (no library needed): blocks of c packed rows,
    [signal a | gate a | signal b | gate b], from proj_bundle's [signal a | signal b | gate a |
    gate b] (mlx_trunk.py:44)."""
    return list(range(c)) + list(range(2 * c, 3 * c)) + list(range(c, 2 * c)) + list(range(3 * c, 4 * c))


@dataclass
class TrimulWeights:
    """Device-resident weights of one triangle update in the kernels' layouts.

    Built once from a tri-mul module (``_trimul_params``, mlx_trunk.py:40-55): the packed
    projection keeps the fp16 scheme's 1/256 pre-scale of the signal-a rows (:47-48)."""

    c_z: int
    c: int
    ln_in_w: torch.Tensor
    ln_in_b: torch.Tensor
    w_proj: torch.Tensor
    ln_mix_w: torch.Tensor
    ln_mix_b: torch.Tensor
    w_emit: torch.Tensor
    w_gate: torch.Tensor
    b_proj: torch.Tensor | None = None
    b_emit: torch.Tensor | None = None
    b_gate: torch.Tensor | None = None
    _struct: _lib.TmuTrimulWeights | None = field(default=None, repr=False)

    @classmethod
    def from_module(cls, tri, device="cuda", biases: dict | None = None) -> "TrimulWeights":
        eng = tri._engine
        c = int(eng.latent_channels)
        w = eng.proj_bundle.weight.detach().float().cpu()
        c_z = w.shape[1]
        assert w.shape[0] == 4 * c, "proj_bundle must have 4*latent_channels rows"
        w = w.clone()
        w[:c] /= CONTRACT_SCALE  # left contraction operand (mlx_trunk.py:47-48)
        order = torch.tensor(proj_row_order_py(c))
        h16 = lambda t: t.detach().float().cpu().to(torch.float16).to(device).contiguous()  # noqa: E731
        f32 = lambda t: None if t is None else t.detach().float().cpu().to(device).contiguous()  # noqa: E731
        b_proj = None
        if biases is not None and biases.get("b_in") is not None:
            b = biases["b_in"].detach().float().cpu().clone()
            b[:c] /= CONTRACT_SCALE
            b_proj = f32(b[order])
        return cls(
            c_z=c_z, c=c,
            ln_in_w=h16(eng.norm_start.weight), ln_in_b=h16(eng.norm_start.bias),
            w_proj=h16(w[order]),
            ln_mix_w=h16(eng.norm_mix.weight), ln_mix_b=h16(eng.norm_mix.bias),
            w_emit=h16(eng.proj_emit.weight), w_gate=h16(eng.proj_gate.weight),
            b_proj=b_proj,
            b_emit=f32(None if biases is None else biases.get("b_emit")),
            b_gate=f32(None if biases is None else biases.get("b_gate")),
        )

    @property
    def struct(self) -> _lib.TmuTrimulWeights:
        if self._struct is None:
            self._struct = _lib.TmuTrimulWeights(
                _ptr(self.ln_in_w), _ptr(self.ln_in_b), _ptr(self.w_proj), _ptr(self.b_proj),
                _ptr(self.ln_mix_w), _ptr(self.ln_mix_b), _ptr(self.w_emit), _ptr(self.b_emit),
                _ptr(self.w_gate), _ptr(self.b_gate))
        return self._struct

    @property
    def device(self) -> torch.device:
        return self.w_proj.device


def _check_pair(z: torch.Tensor, c_z: int) -> tuple[int, int]:
    if not z.is_cuda or z.dtype != torch.float16:
        raise TypeError("z must be a CUDA fp16 tensor")
    if z.dim() != 4 or z.shape[1] != z.shape[2] or z.shape[3] != c_z or not z.is_contiguous():
        raise ValueError(f"z must be contiguous [B, L, L, {c_z}], got {tuple(z.shape)}")
    return z.shape[0], z.shape[1]


def _check_mask(mask, B, L):
    if mask is None:
        return None
    if not mask.is_cuda or mask.dtype != torch.float16 or tuple(mask.shape) != (B, L, L) or not mask.is_contiguous():
        raise ValueError("mask must be a contiguous CUDA fp16 [B, L, L] tensor or None")
    return mask


def new_status(device) -> torch.Tensor:
    return torch.zeros(_lib.TMU_STATUS_BYTES, dtype=torch.uint8, device=device)


def read_status(status: torch.Tensor) -> tuple[int, int]:
    """Synchronise the current stream and return (code, site) of a device status word."""
    lib = _lib.load()
    code, site = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(lib.tmu_read_status(_ptr(status), _stream_ptr(status.device), ctypes.byref(code), ctypes.byref(site)),
               "tmu_read_status")
    return code.value, site.value


def reset_status(status: torch.Tensor) -> None:
    """Zero a status block on the current stream (both its per-call and since-reset records)."""
    _lib.check(_lib.load().tmu_reset_status(_ptr(status), _stream_ptr(status.device)), "tmu_reset_status")


def read_first_error(status: torch.Tensor) -> tuple[int, int]:
    """Synchronise the current stream and return (code, site) of the first error recorded in
    ``status`` since :func:`reset_status`, by any call."""
    lib = _lib.load()
    code, site = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(lib.tmu_read_first_error(_ptr(status), _stream_ptr(status.device), ctypes.byref(code),
                                        ctypes.byref(site)), "tmu_read_first_error")
    return code.value, site.value


def trace_arm(status: torch.Tensor) -> None:
    """Zero a status block and switch on its launch-span trace (``tmu_trace_arm``)."""
    _lib.check(_lib.load().tmu_trace_arm(_ptr(status), _stream_ptr(status.device)), "tmu_trace_arm")


def trace_read(status: torch.Tensor) -> tuple[int, int]:
    """(t_start, t_end) in %globaltimer ns of the kernel launched with this armed block."""
    lib = _lib.load()
    t0, t1 = ctypes.c_ulonglong(0), ctypes.c_ulonglong(0)
    _lib.check(lib.tmu_trace_read(_ptr(status), _stream_ptr(status.device), ctypes.byref(t0), ctypes.byref(t1)),
               "tmu_trace_read")
    return t0.value, t1.value


def raise_for_status(code: int, site: int, where: str) -> None:
    """Raise :class:`TmuError` for a non-zero device status (a bounded wait that gave up, or a
    kernel that found its shared memory misaligned), naming the kernel site that recorded it."""
    if code != 0:
        raise _lib.TmuError(code, where, f"device status recorded at kernel site {site:#x}; the output is invalid")


def check_status(status: torch.Tensor, where: str) -> None:
    """Synchronise, read the call's status and raise if a kernel recorded an error."""
    raise_for_status(*read_status(status), where)


def project_gate(z: torch.Tensor, mask: torch.Tensor | None, w: TrimulWeights, status: torch.Tensor | None = None):
    """K1: returns channel-major (a, b), each [B*c, L, row_pitch(L)] fp16 (pad columns unset)."""
    lib = _lib.load()
    B, L = _check_pair(z, w.c_z)
    mask = _check_mask(mask, B, L)
    a = torch.empty(B * w.c, L, row_pitch(L), dtype=torch.float16, device=z.device)
    b = torch.empty_like(a)
    status = new_status(z.device) if status is None else status
    _lib.check(lib.tmu_project_gate(_ptr(z), _ptr(mask), ctypes.byref(w.struct), B, L, w.c_z, w.c, _ptr(a), _ptr(b),
                                    _ptr(status), _stream_ptr(z.device)), "tmu_project_gate")
    return a, b


def contract(a: torch.Tensor, b: torch.Tensor, L: int, outgoing: bool, status: torch.Tensor | None = None):
    """K2: x[d] = a[d] b[d]^T (outgoing) or a[d]^T b[d] (incoming); [Bc, L, row_pitch(L)] fp16."""
    lib = _lib.load()
    if a.shape != b.shape or a.dim() != 3 or a.shape[1] != L or a.shape[2] != row_pitch(L):
        raise ValueError("a, b must be [Bc, L, row_pitch(L)]")
    if a.dtype != torch.float16 or b.dtype != torch.float16 or not (a.is_contiguous() and b.is_contiguous()):
        raise ValueError("a, b must be contiguous fp16")
    x = torch.empty_like(a)
    status = new_status(a.device) if status is None else status
    _lib.check(lib.tmu_contract(_ptr(a), _ptr(b), _ptr(x), a.shape[0], L, 1 if outgoing else 0, _ptr(status),
                                _stream_ptr(a.device)), "tmu_contract")
    return x


def emit_residual(x: torch.Tensor, z: torch.Tensor, w: TrimulWeights, mix_eps: float = MIX_EPS_FP16,
                  out: torch.Tensor | None = None, status: torch.Tensor | None = None):
    """K3: z + fp16(LN_mix(x) @ w_emit) * sigmoid(fp16(LN(z) @ w_gate)); ``out`` may be ``z``
    (through a temporary when c_z = 256)."""
    lib = _lib.load()
    B, L = _check_pair(z, w.c_z)
    out = torch.empty_like(z) if out is None else out
    dst = torch.empty_like(z) if w.c_z == 256 and _overlaps(z, out) else out
    status = new_status(z.device) if status is None else status
    _lib.check(lib.tmu_emit_residual(_ptr(x), _ptr(z), _ptr(dst), ctypes.byref(w.struct), B, L, w.c_z, w.c,
                                     float(mix_eps), _ptr(status), _stream_ptr(z.device)), "tmu_emit_residual")
    if dst is not out:
        out.copy_(dst)
    return out


class Workspace:
    """Grow-only device workspace for :func:`trimul` (status word + a + b + x)."""

    def __init__(self):
        self.buf: torch.Tensor | None = None
        self.pair: torch.Tensor | None = None

    def get(self, B: int, L: int, c_z: int, c: int, device) -> torch.Tensor:
        return self.get_bytes(int(_lib.load().tmu_workspace_bytes(B, L, c_z, c)), device)

    def get_bytes(self, need: int, device) -> torch.Tensor:
        """The buffer, grown to at least ``need`` bytes on ``device``."""
        if self.buf is None or self.buf.numel() < need or self.buf.device != torch.device(device):
            self.buf = torch.empty(need + 256, dtype=torch.uint8, device=device)
        return self.buf

    def aux_status(self, device) -> torch.Tensor:
        """A status word for kernels outside the tri-mul (the transition)."""
        if getattr(self, "_aux", None) is None or self._aux.device != torch.device(device):
            self._aux = new_status(device)
        return self._aux

    def pair_like(self, z: torch.Tensor) -> torch.Tensor:
        """A second pair buffer shaped like ``z`` (for updates that cannot run in place)."""
        if self.pair is None or self.pair.shape != z.shape or self.pair.device != z.device:
            self.pair = torch.empty_like(z)
        return self.pair

    @property
    def status(self) -> torch.Tensor | None:
        return None if self.buf is None else self.buf[:_lib.TMU_STATUS_BYTES]


def _overlaps(a: torch.Tensor, b: torch.Tensor) -> bool:
    a0, b0 = a.data_ptr(), b.data_ptr()
    return a0 < b0 + b.numel() * b.element_size() and b0 < a0 + a.numel() * a.element_size()


def trimul(z: torch.Tensor, mask: torch.Tensor | None, w: TrimulWeights, outgoing: bool,
           mix_eps: float = MIX_EPS_FP16, out: torch.Tensor | None = None, workspace: Workspace | None = None):
    """One triangle update: ``z + trimul(z)`` in fp16 (``out`` may be ``z`` for in-place).

    The c_z = 256 kernels cannot write over their input (two CTAs share each tile's z), so an
    in-place call there goes through the workspace's second pair buffer and a copy back."""
    lib = _lib.load()
    B, L = _check_pair(z, w.c_z)
    mask = _check_mask(mask, B, L)
    out = torch.empty_like(z) if out is None else out
    workspace = workspace if workspace is not None else Workspace()
    ws = workspace.get(B, L, w.c_z, w.c, z.device)
    dst = workspace.pair_like(z) if w.c_z == 256 and _overlaps(z, out) else out
    _lib.check(lib.tmu_trimul(_ptr(z), _ptr(dst), _ptr(mask), ctypes.byref(w.struct), B, L, w.c_z, w.c,
                              1 if outgoing else 0, float(mix_eps), _ptr(ws), ws.numel(), _stream_ptr(z.device)),
               "tmu_trimul")
    if dst is not out:
        out.copy_(dst)
    return out


@dataclass
class TransitionWeights:
    """Device-resident weights of one pair transition (``norm``, ``ffn.w12``, ``ffn.w3``) in the
    layouts of ``tmu_transition``: LayerNorm fp16, w12 [2h or h, c_z] and w3 [c_z, h] as
    ``nn.Linear`` stores them (mlx_trunk.py:65-66 keeps the same matrices transposed)."""

    c_z: int
    hidden: int
    activation: str
    ln_w: torch.Tensor
    ln_b: torch.Tensor
    w12: torch.Tensor
    w3: torch.Tensor
    _struct: _lib.TmuTransitionWeights | None = field(default=None, repr=False)

    @classmethod
    def from_module(cls, tr, device="cuda") -> "TransitionWeights":
        h16 = lambda t: t.detach().float().cpu().to(torch.float16).to(device).contiguous()  # noqa: E731
        act = getattr(tr.ffn, "activation", "swiglu")
        w3 = tr.ffn.w3.weight
        return cls(c_z=int(w3.shape[0]), hidden=int(w3.shape[1]), activation=act,
                   ln_w=h16(tr.norm.weight), ln_b=h16(tr.norm.bias), w12=h16(tr.ffn.w12.weight), w3=h16(w3))

    @property
    def struct(self) -> _lib.TmuTransitionWeights:
        if self._struct is None:
            self._struct = _lib.TmuTransitionWeights(_ptr(self.ln_w), _ptr(self.ln_b), _ptr(self.w12), _ptr(self.w3))
        return self._struct

    @property
    def fused(self) -> bool:
        """Whether ``tmu_transition`` covers this shape (c_z = 128 or 256, hidden a multiple of 64)."""
        return self.c_z in (128, 256) and self.hidden % 64 == 0 and 64 <= self.hidden <= 4096


def transition(z: torch.Tensor, w: TransitionWeights, out: torch.Tensor | None = None,
               status: torch.Tensor | None = None) -> torch.Tensor:
    """K4: ``z + ffn(LN(z))`` in fp16 (``out`` may be ``z``)."""
    lib = _lib.load()
    B, L = _check_pair(z, w.c_z)
    out = torch.empty_like(z) if out is None else out
    status = new_status(z.device) if status is None else status
    act = _lib.TMU_ACT_SWIGLU if w.activation == "swiglu" else _lib.TMU_ACT_RELU
    _lib.check(lib.tmu_transition(_ptr(z), _ptr(out), ctypes.byref(w.struct), B, L, w.c_z, w.hidden, act,
                                  _ptr(status), _stream_ptr(z.device)), "tmu_transition")
    return out


def pair_block(z: torch.Tensor, mask: torch.Tensor | None, w_out: TrimulWeights, w_in: TrimulWeights,
               tw: TransitionWeights, mix_eps: float = MIX_EPS_FP16, out: torch.Tensor | None = None,
               workspace: Workspace | None = None) -> torch.Tensor:
    """One PairUpdateBlock (tri-mul out, tri-mul in, transition) in one C-ABI call
    (``tmu_pair_block``; the reference's ``block_forward``, ``mlx_trunk_kernels.py:232-239``).
    ``out`` may be ``z``; the status word is the workspace's (``workspace.status``)."""
    lib = _lib.load()
    B, L = _check_pair(z, w_out.c_z)
    mask = _check_mask(mask, B, L)
    out = torch.empty_like(z) if out is None else out
    workspace = workspace if workspace is not None else Workspace()
    need = int(lib.tmu_pair_block_workspace_bytes(B, L, w_out.c_z, w_out.c))
    ws = workspace.get_bytes(need, z.device)
    act = _lib.TMU_ACT_SWIGLU if tw.activation == "swiglu" else _lib.TMU_ACT_RELU
    _lib.check(lib.tmu_pair_block(_ptr(z), _ptr(out), _ptr(mask), ctypes.byref(w_out.struct), ctypes.byref(w_in.struct),
                                  ctypes.byref(tw.struct), B, L, w_out.c_z, w_out.c, tw.hidden, act, float(mix_eps),
                                  _ptr(ws), ws.numel(), _stream_ptr(z.device)), "tmu_pair_block")
    return out
