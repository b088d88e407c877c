"""Adaptive recycling on B200: stop running trunk passes once the pair representation has
converged (the reference's ``var_adaptive_loops.py``), with the convergence signal computed by
the fused distogram kernel K5 (``tmu_disto_expected``).

The reference compares consecutive trunk outputs through the distogram head's expected distance
per pair, ``E = softmax(head(z + z^T)) @ centres`` (``var_adaptive_loops.py:43-46``), and stops
once the 95th percentile of ``|E_cur - E_prev|`` over all pairs is below 0.6 Å, from the second
pass on (``:31-34,115-121,135-137``).  Here ``E`` is one kernel over the pair grid (two tcgen05
GEMM chains for ``z W^T + z^T W^T``, softmax and the weighted sum in the epilogue) instead of
materialising ``z + z^T``, the ``[L, L, 128]`` logits and their softmax; the percentile is
``torch.quantile`` of the ``L^2`` differences, as in the reference.
"""

from __future__ import annotations

import ctypes

import torch
from torch import nn

from . import _lib, ops

METRIC = "disto_p95"
THRESHOLD = 0.6  # var_adaptive_loops.py:31-32
MIN_PASSES = 2   # :33
MAX_EXTRA = 0    # :36

_EDGES = torch.linspace(2.0, 52.0, 127)
CENTRES = torch.cat([_EDGES[:1] - 0.2, (_EDGES[1:] + _EDGES[:-1]) / 2, _EDGES[-1:] + 0.2])  # :39-40


class DistoHead:
    """The distogram head ``Linear(c_z, 128)`` in the layout of ``tmu_disto_expected``: weight fp16
    (rounded from the module's fp32), bias and bin centres fp32."""

    def __init__(self, head: nn.Module, device="cuda"):
        w = head.weight.detach()
        if w.shape[0] != 128:
            raise ValueError("the distogram head must have 128 bins")
        self.c_z = int(w.shape[1])
        self.w = w.float().to(torch.float16).to(device).contiguous()
        b = getattr(head, "bias", None)
        self.b = None if b is None else b.detach().float().to(device).contiguous()
        self.centres = CENTRES.to(device)
        self.status = ops.new_status(device)


def expected_distance(z: torch.Tensor, head: DistoHead) -> torch.Tensor:
    """E [B, L, L] fp32 for fp16 ``z`` [B, L, L, c_z] (K5)."""
    if not z.is_cuda or z.dtype != torch.float16 or z.dim() != 4 or z.shape[1] != z.shape[2] or not z.is_contiguous():
        raise ValueError("z must be a contiguous CUDA fp16 [B, L, L, c_z] tensor")
    B, L = z.shape[0], z.shape[1]
    out = torch.empty(B, L, L, dtype=torch.float32, device=z.device)
    lib = _lib.load()
    _lib.check(lib.tmu_disto_expected(ops._ptr(z), ops._ptr(head.w), ops._ptr(head.b), ops._ptr(head.centres),
                                      ops._ptr(out), B, L, head.c_z, 128, ops._ptr(head.status),
                                      ops._stream_ptr(z.device)), "tmu_disto_expected")
    return out


def disto_p95(e_prev: torch.Tensor, e_cur: torch.Tensor) -> float:
    """95th percentile of |E_cur - E_prev| over all pairs (Å) -- one host sync per pass."""
    return float((e_cur - e_prev).abs().flatten().quantile(0.95))


class CUDAAdaptiveTrunk(nn.Module):
    """Wraps a folding trunk (``CUDAFoldingTrunk`` or any module with the same call) and skips
    the passes after convergence, returning the converged output for every remaining call; the
    fold is then identical to one run with fewer loops (``var_adaptive_loops.py:76-142``)."""

    def __init__(self, trunk, model, threshold: float = THRESHOLD, min_passes: int = MIN_PASSES,
                 max_extra: int = MAX_EXTRA, extra_threshold: float | None = None):
        super().__init__()
        self.trunk = trunk
        # Plain attributes (not submodules) so the model's state dict is unchanged.
        self.__dict__["_proj"] = getattr(model, "pair_loop_proj", None)
        device = next(iter(p for p in model.distogram_head.parameters())).device
        self.__dict__["_head"] = DistoHead(model.distogram_head, device if device.type == "cuda" else "cuda")
        self.threshold, self.min_passes, self.max_extra = threshold, min_passes, max_extra
        self.extra_threshold = threshold if extra_threshold is None else extra_threshold
        self.metric = METRIC
        self.reset(None)

    def set_chunk_size(self, chunk_size):
        self.trunk.set_chunk_size(chunk_size)

    def set_kernel_backend(self, backend):
        self.trunk.set_kernel_backend(backend)

    def reset(self, scheduled_passes):
        self.scheduled = scheduled_passes
        self.calls = 0
        self.passes = 0
        self.prev = self.prev_ed = None
        self.z_init = None
        self.converged = False
        self.history = []

    def _pass(self, pair, mask):
        out = self.trunk(pair, pair_attention_mask=mask)
        self.passes += 1
        z16 = out.to(torch.float16).contiguous()  # exact: the trunk computes in fp16
        ed = expected_distance(z16, self._head)
        if self.prev_ed is not None:
            self.history.append({"disto_p95": disto_p95(self.prev_ed, ed)})
        self.prev_ed = ed
        self.prev = out
        return out

    def forward(self, pair, pair_attention_mask=None):
        self.calls += 1
        if self.converged:
            return self.prev
        if self.calls == 1 and self.max_extra:
            self.z_init = pair - self._proj(torch.zeros_like(pair))
        out = self._pass(pair, pair_attention_mask)
        if self.passes >= self.min_passes and self.history[-1][self.metric] < self.threshold:
            self.converged = True
            return out
        if self.scheduled is not None and self.calls == self.scheduled and self.max_extra:
            for _ in range(self.max_extra):
                out = self._pass(self.z_init + self._proj(out), pair_attention_mask)
                if self.history[-1][self.metric] < self.extra_threshold:
                    break
        return out


def apply(model, **kw):
    """Wrap ``model.folding_trunk`` (apply after the trunk swap) and reset per fold."""
    trunk = CUDAAdaptiveTrunk(model.folding_trunk, model, **kw)
    model.folding_trunk = trunk
    forward = model.forward

    def adaptive_forward(*a, num_loops=None, **k):
        n = num_loops if num_loops is not None else model.config.num_loops
        trunk.reset(n + 1)
        return forward(*a, num_loops=num_loops, **k)

    model.forward = adaptive_forward
    return trunk
