"""Adaptive recycling on B200: skip the trunk passes that no longer change the fold.

Behaviour is the reference's adaptive-loops variant (``var_adaptive_loops.py:76-156``): after
every trunk pass the distogram head's expected distance per pair is computed,
``E = softmax(head(z + z^T)) @ centres`` (``:43-46``); from the second pass on, once the 95th
percentile over all pairs of ``|E - E_previous|`` drops below 0.6 Å (``:31-34``), the fold is
settled and every later trunk call of that fold returns the settled output without running the
trunk, which makes the fold identical to one run with fewer loops.  Optionally (off by default,
``:36``) the last scheduled call runs extra passes of the recurrence
``z = trunk(z_init + pair_loop_proj(z))`` while the fold keeps moving.

What is different here is how the signal is computed and how the state is kept:

* :class:`ExpectedDistance` evaluates ``E`` with one kernel over the pair grid (K5,
  ``tmu_disto_expected``): two tcgen05 GEMM chains accumulate ``z W^T + z^T W^T`` in TMEM and the
  epilogue runs an online softmax over the 128 bins, so neither ``z + z^T`` nor the
  ``[L, L, 128]`` logits are ever stored.  The head's weight is rounded to fp16 once.
* :class:`SettleMonitor` keeps the previous pass's ``E`` on the device and reduces each new pass
  to one number (the p95 change), read with one host synchronisation per pass, as the
  reference does.
* :class:`FoldRecord` is the per-fold state; :meth:`CUDAAdaptiveTrunk.start_fold` replaces it
  when the model's ``forward`` begins a new fold (installed by :func:`apply`).

:func:`expected_distance` has the reference's hook signature ``(z, disto_head)``, so the
reference's own wrapper can also take K5 as its signal.
"""

from __future__ import annotations

import weakref
from dataclasses import dataclass, field

import torch
from torch import nn

from . import _lib, ops

SIGNAL = "disto_p95"
SETTLE_A = 0.6      # Å; var_adaptive_loops.py:31-32
FIRST_CHECK = 2     # a change needs two passes (:33)
EXTRA_PASSES = 0    # :36

N_BINS = 128


def bin_centres(n_bins: int = N_BINS, lo: float = 2.0, hi: float = 52.0) -> torch.Tensor:
    """Centres of the distogram's bins: ``n_bins - 1`` evenly spaced edges over [lo, hi] Å,
    each inner bin centred between its edges and the two open-ended bins 0.2 Å outside the
    outer edges (``var_adaptive_loops.py:38-40``)."""
    edges = torch.linspace(lo, hi, n_bins - 1)
    inner = 0.5 * (edges[1:] + edges[:-1])
    return torch.cat([(edges[0] - 0.2).reshape(1), inner, (edges[-1] + 0.2).reshape(1)])


CENTRES = bin_centres()


class ExpectedDistance:
    """K5 for one distogram head ``Linear(c_z, 128)``: weight fp16 (rounded once from the
    module's fp32), bias and bin centres fp32, all resident on ``device``; calling it with fp16
    ``z`` [B, L, L, c_z] returns ``E`` [B, L, L] fp32."""

    def __init__(self, head: nn.Module, device="cuda"):
        w = head.weight.detach()
        if w.shape[0] != N_BINS:
            raise ValueError(f"the distogram head must have {N_BINS} bins, got {w.shape[0]}")
        self.c_z = int(w.shape[1])
        self.w = w.float().to(torch.float16).to(device).contiguous()
        b = getattr(head, "bias", None)
        self.b = None if b is None else b.detach().float().to(device).contiguous()
        self.centres = CENTRES.to(device)
        self.status = ops.new_status(device)

    def __call__(self, z: torch.Tensor) -> torch.Tensor:
        if (not z.is_cuda or z.dtype != torch.float16 or z.dim() != 4 or z.shape[1] != z.shape[2]
                or not z.is_contiguous()):
            raise ValueError("z must be a contiguous CUDA fp16 [B, L, L, c_z] tensor")
        B, L = z.shape[0], z.shape[1]
        out = torch.empty(B, L, L, dtype=torch.float32, device=z.device)
        lib = _lib.load()
        _lib.check(lib.tmu_disto_expected(ops._ptr(z), ops._ptr(self.w), ops._ptr(self.b), ops._ptr(self.centres),
                                          ops._ptr(out), B, L, self.c_z, N_BINS, ops._ptr(self.status),
                                          ops._stream_ptr(z.device)), "tmu_disto_expected")
        return out


# head module -> {device: ExpectedDistance}; an entry goes away with its head module
_evaluators: "weakref.WeakKeyDictionary[nn.Module, dict]" = weakref.WeakKeyDictionary()


def expected_distance(z: torch.Tensor, disto_head: nn.Module) -> torch.Tensor:
    """``E`` for a trunk output ``z`` [B, L, L, c_z] (fp32 or fp16, on a CUDA device) and the
    model's distogram head, with the reference's hook signature (``var_adaptive_loops.py:43``).
    The trunk computes in fp16, so rounding its fp32 output back to fp16 is exact.  The head's
    device copy is made on first use and kept for the life of the head module."""
    per_device = _evaluators.setdefault(disto_head, {})
    ev = per_device.get(z.device)
    if ev is None:
        ev = per_device[z.device] = ExpectedDistance(disto_head, z.device)
    return ev(z.to(torch.float16).contiguous())


class SettleMonitor:
    """Turns consecutive trunk outputs into the p95 change of their expected distances."""

    def __init__(self, evaluate):
        self.evaluate = evaluate
        self.previous = None

    def clear(self):
        self.previous = None

    def observe(self, out: torch.Tensor) -> float | None:
        """Record one pass's output; the p95 |ΔE| against the previous pass (Å), or None for
        the first pass of a fold."""
        e = self.evaluate(out.to(torch.float16).contiguous())
        change = None
        if self.previous is not None:
            change = float((e - self.previous).abs().flatten().quantile(0.95))
        self.previous = e
        return change


@dataclass
class FoldRecord:
    """State of one fold: the number of trunk calls the model will make (None if unknown),
    the calls and passes so far, the latest output and the changes between passes."""

    scheduled: int | None = None
    calls: int = 0
    passes: int = 0
    latest: torch.Tensor | None = None
    z_init: torch.Tensor | None = None
    settled: bool = False
    changes: list = field(default_factory=list)


class CUDAAdaptiveTrunk(nn.Module):
    """Wraps a folding trunk (``CUDAFoldingTrunk`` or any module with its call signature) and
    stops running it once a fold has settled."""

    def __init__(self, trunk, model, threshold: float = SETTLE_A, min_passes: int = FIRST_CHECK,
                 max_extra: int = EXTRA_PASSES, extra_threshold: float | None = None):
        super().__init__()
        self.trunk = trunk
        # kept out of the module tree, so the model's state dict does not change
        self.__dict__["_loop_proj"] = getattr(model, "pair_loop_proj", None)
        head_dev = next(iter(model.distogram_head.parameters())).device
        ev = ExpectedDistance(model.distogram_head, head_dev if head_dev.type == "cuda" else "cuda")
        self.__dict__["_monitor"] = SettleMonitor(ev)
        self.threshold, self.min_passes, self.max_extra = threshold, min_passes, max_extra
        self.extra_threshold = threshold if extra_threshold is None else extra_threshold
        self.fold = FoldRecord()

    # the FoldingTrunk setters the model calls reach the wrapped trunk
    def set_chunk_size(self, chunk_size):
        self.trunk.set_chunk_size(chunk_size)

    def set_kernel_backend(self, backend):
        self.trunk.set_kernel_backend(backend)

    def start_fold(self, scheduled_calls: int | None):
        """Forget the previous fold; the model will call the trunk ``scheduled_calls`` times."""
        self.fold = FoldRecord(scheduled=scheduled_calls)
        self._monitor.clear()

    @property
    def passes(self) -> int:
        return self.fold.passes

    @property
    def converged(self) -> bool:
        return self.fold.settled

    def _run_pass(self, pair, mask) -> torch.Tensor:
        out = self.trunk(pair, pair_attention_mask=mask)
        f = self.fold
        f.passes += 1
        change = self._monitor.observe(out)
        if change is not None:
            f.changes.append(change)
        f.latest = out
        return out

    def _below(self, limit: float) -> bool:
        return bool(self.fold.changes) and self.fold.changes[-1] < limit

    def _extend(self, out, mask) -> torch.Tensor:
        """Extra passes of the loop's recurrence while the fold keeps moving."""
        f = self.fold
        for _ in range(self.max_extra):
            out = self._run_pass(f.z_init + self._loop_proj(out), mask)
            if self._below(self.extra_threshold):
                break
        return out

    def forward(self, pair, pair_attention_mask=None):
        f = self.fold
        f.calls += 1
        if f.settled:
            return f.latest  # the fold stopped here: same as a run with fewer loops
        if self.max_extra and f.calls == 1:
            # the first call's input is z_init + pair_loop_proj(0): recover z_init exactly
            f.z_init = pair - self._loop_proj(torch.zeros_like(pair))
        out = self._run_pass(pair, pair_attention_mask)
        if f.passes >= self.min_passes and self._below(self.threshold):
            f.settled = True
            return out
        if self.max_extra and f.calls == f.scheduled:
            out = self._extend(out, pair_attention_mask)
        return out


def apply(model, **kw):
    """Wrap ``model.folding_trunk`` (after the trunk swap) and start a new fold record at every
    ``model.forward``, which calls the trunk ``num_loops + 1`` times."""
    wrapper = CUDAAdaptiveTrunk(model.folding_trunk, model, **kw)
    model.folding_trunk = wrapper
    inner_forward = model.forward

    def forward_with_fold_record(*args, num_loops=None, **kwargs):
        loops = model.config.num_loops if num_loops is None else num_loops
        wrapper.start_fold(loops + 1)
        return inner_forward(*args, num_loops=num_loops, **kwargs)

    model.forward = forward_with_fold_record  # an instance attribute shadows nn.Module.forward
    return wrapper
