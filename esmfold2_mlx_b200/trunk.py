"""The folding trunk on B200: a drop-in for the reference's MLX trunk module.

Mirrors ``src/esmfold2_mlx/mlx_trunk.py`` / ``mlx_trunk_kernels.py`` / ``var_mlx_trunk.py``:

* :func:`trunk_params` (``mlx_trunk.py:58-69``) copies every block's weights once into
  device-resident fp16 buffers in the kernels' layouts (fp16 scheme with the 1/256 pre-scale);
* :func:`block_forward` / :func:`trunk_forward` / :func:`make_trunk`
  (``mlx_trunk_kernels.py:232-255``) run tri-mul out, tri-mul in and the pair transition;
* :class:`CUDAFoldingTrunk` (``var_mlx_trunk.py:24-46``) is an ``nn.Module`` with the same
  surface as ``MLXFoldingTrunk``: ``params``, ``_fn(params, z, mask)``, ``set_chunk_size``,
  ``set_kernel_backend`` and ``forward(pair, pair_attention_mask=None)`` -> fp32 on
  ``pair.device``.

Each triangle update is one C-ABI call (three sm_100a kernels) and, at c_z = 128, the pair
transition is one more (K4, ``tmu_transition``).  At other widths the transition runs as torch
ops on the GPU (cuBLAS GEMMs + element-wise ops with the reference's fp16 rounding points).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from . import ops

EPS = ops.EPS


def _transition_params(tr, device) -> dict:
    h16 = lambda t: t.detach().float().cpu().to(torch.float16).to(device).contiguous()  # noqa: E731
    act = getattr(tr.ffn, "activation", "swiglu")
    tw = ops.TransitionWeights.from_module(tr, device)
    p = {"tw": tw, "activation": act}
    if not tw.fused:  # shapes K4 does not cover run as torch ops on the GPU
        p.update({
            "ln_w": h16(tr.norm.weight), "ln_b": h16(tr.norm.bias),
            "w12": h16(tr.ffn.w12.weight),  # nn.Linear layout [2h or h, c_z]
            "w3t": h16(tr.ffn.w3.weight.T),  # [h, c_z] so that z + s @ w3t is one addmm
        })
    return p


def trunk_params(folding_trunk, dtype=torch.float16, device="cuda", biases: list | None = None) -> list:
    """Copy every block's weights out of a trunk-shaped module (``mlx_trunk.py:58-69``).

    ``biases``: optional per-block ``{"out": {...}, "in": {...}}`` tri-mul biases (not part of
    the reference module tree; see :func:`esmfold2_mlx_b200.synthetic.trimul_biases`)."""
    if dtype != torch.float16:
        raise ValueError("the B200 trunk implements the reference's fp16 scheme only")
    blocks = []
    for i, blk in enumerate(folding_trunk.blocks):
        bb = biases[i] if biases is not None else {}
        blocks.append({
            "out": ops.TrimulWeights.from_module(blk.tri_mul_out, device, bb.get("out")),
            "in": ops.TrimulWeights.from_module(blk.tri_mul_in, device, bb.get("in")),
            **_transition_params(blk.pair_transition, device),
        })
    return blocks


def transition_(p: dict, z: torch.Tensor, workspace: ops.Workspace | None = None) -> torch.Tensor:
    """``z + ffn(LN(z))`` in place (``mlx_trunk_kernels.py:236-239``): fp16 LayerNorm output,
    fp16 GEMM output, three fp16 element-wise ops for SwiGLU, one-rounding ``addmm`` residual.
    c_z = 128 and 256 run the fused kernel K4 (``tmu_transition``); other shapes run torch ops."""
    if p["tw"].fused:
        # the tri-mul workspace's status word, so one read after the pass covers every kernel
        status = workspace.status if workspace is not None and workspace.status is not None else None
        return ops.transition(z, p["tw"], out=z, status=status)
    c_z = z.shape[-1]
    h = F.layer_norm(z, (c_z,), p["ln_w"], p["ln_b"], EPS)
    x = F.linear(h, p["w12"])
    if p["activation"] == "swiglu":
        x1, x2 = x.chunk(2, dim=-1)
        s = x1 * torch.sigmoid(x1) * x2
    else:
        s = torch.relu(x)
    z2 = z.view(-1, c_z)
    torch.addmm(z2, s.reshape(-1, s.shape[-1]), p["w3t"], out=z2)
    return z


def block_forward(p: dict, z: torch.Tensor, mask, mix_eps: float = ops.MIX_EPS_FP16,
                  workspace: ops.Workspace | None = None) -> torch.Tensor:
    """One PairUpdateBlock, updating fp16 ``z`` [B, L, L, c_z] in place."""
    if z.shape[-1] == 256:  # the wide kernels write a second buffer: out z -> t, in t -> z
        workspace = workspace if workspace is not None else ops.Workspace()
        t = workspace.pair_like(z)
        ops.trimul(z, mask, p["out"], True, mix_eps, out=t, workspace=workspace)
        ops.trimul(t, mask, p["in"], False, mix_eps, out=z, workspace=workspace)
    else:
        ops.trimul(z, mask, p["out"], True, mix_eps, out=z, workspace=workspace)
        ops.trimul(z, mask, p["in"], False, mix_eps, out=z, workspace=workspace)
    return transition_(p, z, workspace)


def trunk_forward(params: list, z: torch.Tensor, mask=None, mix_eps: float = ops.MIX_EPS_FP16,
                  workspace: ops.Workspace | None = None) -> torch.Tensor:
    """z in any float dtype on any device; computed in fp16 on the params' device; returns fp32
    there (``mlx_trunk_kernels.py:242-249``)."""
    device = params[0]["out"].device
    if device.type != "cuda":
        raise TypeError(f"the B200 trunk runs on a CUDA device; its weights are on {device}")
    z = z.to(device=device, dtype=torch.float16).contiguous().clone()
    if mask is not None:
        mask = mask.to(device=device, dtype=torch.float16).contiguous()
    ws = workspace if workspace is not None else ops.Workspace()
    # Size the workspace before zeroing its status word, so the word stays put for the pass: the
    # kernels of all blocks record into it and its since-reset record is read once afterwards.
    ws.get(z.shape[0], z.shape[1], params[0]["out"].c_z, params[0]["out"].c, device)
    ops.reset_status(ws.status)
    for p in params:
        block_forward(p, z, mask, mix_eps, ws)
    return z.float()


class _Trunk:
    """The compiled-trunk callable ``fn(params, z, mask)`` (``make_trunk``'s return value)."""

    def __init__(self, mix_eps: float):
        self.mix_eps = mix_eps
        self.workspace = ops.Workspace()

    def __call__(self, params, z, mask=None):
        return trunk_forward(params, z, mask, self.mix_eps, self.workspace)


def make_trunk(dtype=torch.float16):
    """Trunk function for params from :func:`trunk_params` (``mlx_trunk_kernels.py:252-255``)."""
    if dtype != torch.float16:
        raise ValueError("the B200 trunk implements the reference's fp16 scheme only")
    return _Trunk(ops.MIX_EPS_FP16)


class _GraphEntry:
    """One captured trunk pass: static input / mask / output buffers, the CUDA graph, and the
    trunk function whose workspace the captured kernels address.  The entry must own that
    function: a later capture's ``torch.cuda.graph`` runs ``gc.collect()`` and ``empty_cache()``,
    which would hand an orphaned workspace back to the driver while this graph still writes it."""

    def __init__(self, graph, z_in, mask_in, out, fn):
        self.graph, self.z_in, self.mask_in, self.out, self.fn = graph, z_in, mask_in, out, fn


class CUDAFoldingTrunk(nn.Module):
    """Drop-in replacement for ``model.folding_trunk`` (``var_mlx_trunk.py:24-46``).

    With ``graphs=True`` (default) each pass on CUDA input is replayed from a CUDA graph captured
    once per (B, L, mask present, device) -- the reference recompiles its MLX trunk per new L in
    the same way (``var_mlx_trunk.py:28-30``) -- so a 24-block pass is one launch instead of
    ~170; up to ``max_graphs`` shapes are kept (least recently used evicted), each holding its
    own static buffers.  The graph's output buffer is reused, so the returned tensor is a copy.

    Device-side errors (a bounded wait in a kernel that gave up, which leaves the output invalid)
    are reported per pass through the pass's status word, copied to the host after the pass:
    ``check_status="deferred"`` (default) raises ``TmuError`` at the start of the next call (or
    at :meth:`check_status`), which costs no synchronisation; ``"sync"`` waits for the pass and
    raises before returning; ``"off"`` leaves the word unread.  Passes run inside the caller's
    own stream capture are not checked (the caller reads the status word after its replay)."""

    def __init__(self, folding_trunk, dtype=torch.float16, device="cuda", biases: list | None = None,
                 graphs: bool = True, max_graphs: int = 4, check_status: str = "deferred"):
        super().__init__()
        if check_status not in ("deferred", "sync", "off"):
            raise ValueError("check_status must be 'deferred', 'sync' or 'off'")
        self.params = trunk_params(folding_trunk, dtype, device, biases)
        self._fn = make_trunk(dtype)
        self.graphs, self.max_graphs = graphs, max_graphs
        self._graph_cache: dict = {}
        self.check_mode = check_status
        self._pending = None  # (event, pinned host copy of the status word) of the last pass
        self._status_host = None

    def _note_status(self, status):
        """Copy the pass's status word to pinned host memory behind the pass (no sync)."""
        if self.check_mode == "off" or status is None:
            return
        if self._status_host is None:
            self._status_host = torch.zeros(8, dtype=torch.int32).pin_memory()
        self._status_host.copy_(status[:32].view(torch.int32), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._pending = ev
        if self.check_mode == "sync":
            self.check_status()

    def check_status(self):
        """Raise ``TmuError`` if the last unchecked pass recorded a device-side error (waits for
        that pass to finish)."""
        ev, self._pending = self._pending, None
        if ev is None:
            return
        ev.synchronize()
        h = self._status_host
        ops.raise_for_status(int(h[4]), int(h[5]), "CUDAFoldingTrunk pass")

    # FoldingTrunk API the model calls on its trunk; the fused kernels ignore both.
    def set_chunk_size(self, chunk_size):
        pass

    def set_kernel_backend(self, backend):
        pass

    def _graph_pass(self, pair, mask):
        dev = self.params[0]["out"].device
        key = (tuple(pair.shape), mask is not None, dev)
        entry = self._graph_cache.pop(key, None)
        if entry is None:
            z_in = torch.empty(pair.shape, dtype=torch.float16, device=dev)
            mask_in = None if mask is None else torch.empty(mask.shape, dtype=torch.float16, device=dev)
            z_in.copy_(pair)
            if mask_in is not None:
                mask_in.copy_(mask)
            fn = make_trunk()  # its own workspace, owned by this graph
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):  # eager pass first: sizes every allocation before capture
                fn(self.params, z_in, mask_in)
            torch.cuda.current_stream(dev).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = fn(self.params, z_in, mask_in)
            entry = _GraphEntry(graph, z_in, mask_in, out, fn)
            while len(self._graph_cache) >= self.max_graphs:
                self._graph_cache.pop(next(iter(self._graph_cache)))
        self._graph_cache[key] = entry  # most recently used last
        entry.z_in.copy_(pair)
        if entry.mask_in is not None:
            entry.mask_in.copy_(mask)
        entry.graph.replay()
        self._note_status(entry.fn.workspace.status)
        return entry.out.clone()

    def forward(self, pair, pair_attention_mask=None):
        capturing = pair.is_cuda and torch.cuda.is_current_stream_capturing()
        if not capturing:
            self.check_status()  # the previous pass's device status (deferred mode)
        # A single-chain fold has an all-ones mask; skipping it saves a multiply per tri-mul.
        mask = None
        if pair_attention_mask is not None and not bool(pair_attention_mask.all()):
            mask = pair_attention_mask
        if self.graphs and pair.is_cuda and not capturing:
            out = self._graph_pass(pair, mask)
        else:
            out = self._fn(self.params, pair, mask)
            if not capturing:
                self._note_status(getattr(getattr(self._fn, "workspace", None), "status", None))
        return out.to(pair.device)
