"""One long sequence's triangle update row-sharded over the GPUs of a process group.

Two partitions of the contraction share the row-sharded pair tensor: :class:`RowShardedTrimul`
(below: an all-gather of b, an all-to-all transpose of z for the incoming form) and
:class:`ChannelShardedTrimul` (the contraction split over channels by two all-to-alls, at the
end of this file).

The reference runs one fold on one device; this path (L = 3072 over 2/4/8
B200s) has no counterpart there.  Rank r holds rows [r*Lr, (r+1)*Lr) of the pair tensor
z [1, L, L, c_z] (Lr = L / P) and returns the same rows of z + update.

Outgoing, x[d,i,j] = sum_k a[d,i,k] b[d,j,k]: a and b are projected on the local rows (K1); the
ranks' b slabs are all-gathered by NCCL on its own stream into [P, B*c, Lr, pitch] -- the block
layout the contraction kernel reads through a 4-D tensor map -- while the local block of b is
contracted into its column block of x (K2 writes a column block through its row pitch, on a
grid that leaves SMs to NCCL); then the remote blocks are contracted and each rank finishes its
rows (K3).

Incoming, x[d,i,j] = sum_k a[d,k,i] b[d,k,j]: with a'[d,i,k] = a[d,k,i] (the projection of
z^T[i,k] = z[k,i]) it is the outgoing form of the transposed grid.  An all-to-all sends each
rank's [Lr, Lr] blocks to the rank owning those columns, which then holds z[:, its columns] as a
[P, Lr, Lr, c_z] buffer; K1 reads that buffer as the transposed slab z^T[its columns, :] through
strides alone (element (i, k) sits at k*Lr*c_z + i*c_z), b' is gathered and contracted as above,
and K3 finishes the local rows of z in their original orientation.

The collectives are NCCL through torch.distributed (the all-gather asynchronous, joined to the
current stream before the remote blocks are read).  The three stages and the exchange are
injectable (``stages=``, ``exchange=``) so the data movement can be exercised on CPU ranks
with gloo, or by threads standing in for ranks on one GPU.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops


class CudaStages:
    """The three sm_100a kernels through the slab entry points of the C ABI."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.status = ops.new_status(self.device)

    def project_gate(self, z, layout, mask, w, b_out=None, a_out=None):
        """z: storage holding a [B, rows, cols, c_z] view with element strides
        (stride_b, stride_row, stride_col); mask likewise with mask strides (or None).
        Returns a, b: [B*c, rows, pitch(cols)] (written into ``a_out`` / ``b_out`` when given)."""
        B, rows, cols, sb, sr, sc, msb, msr, msc = layout
        lib = _lib.load()
        g = _lib.TmuPairLayout(B, rows, cols, sb, sr, sc, msb, msr, msc)
        a = a_out if a_out is not None else torch.empty(B * w.c, rows, ops.row_pitch(cols), dtype=torch.float16,
                                                        device=self.device)
        b = torch.empty_like(a) if b_out is None else b_out
        _lib.check(lib.tmu_project_gate_ex(ops._ptr(z), ops._ptr(mask), ctypes.byref(g), ctypes.byref(w.struct),
                                           w.c_z, w.c, ops._ptr(a), ops._ptr(b), ops._ptr(self.status),
                                           ops._stream_ptr(self.device)), "tmu_project_gate_ex")
        return a, b

    def contract(self, a, b_parts, M, N, K, rows_per_part, x=None, max_ctas=0):
        """a [Bc, M, pitch(K)], b_parts [P, Bc, rows_per_part, pitch(K)] -> x [Bc, M, >= N].

        ``x`` may be a column block x_full[:, :, c0:] of a wider row-major matrix (its row pitch is
        taken from its stride); by default a new [Bc, M, pitch(N)] tensor.  ``max_ctas`` > 0 caps
        the kernel's grid so that SMs stay free for a transfer running alongside."""
        lib = _lib.load()
        Bc = a.shape[0]
        if x is None:
            x = torch.empty(Bc, M, ops.row_pitch(N), dtype=torch.float16, device=self.device)
        _lib.check(lib.tmu_contract_ex(ops._ptr(a), ops._ptr(b_parts), ops._ptr(x), Bc, M, N, K, rows_per_part,
                                       x.stride(1), int(max_ctas), ops._ptr(self.status),
                                       ops._stream_ptr(self.device)),
                   "tmu_contract_ex")
        return x

    def contract_full(self, a, b, L, outgoing, x=None):
        """K2 over whole channels: a, b [Bc, L, pitch(L)] -> x[d] = a[d] b[d]^T (outgoing) or
        a[d]^T b[d] (incoming), written into ``x`` ([Bc, L, pitch(L)], contiguous) when given."""
        lib = _lib.load()
        x = torch.empty_like(a) if x is None else x
        _lib.check(lib.tmu_contract(ops._ptr(a), ops._ptr(b), ops._ptr(x), a.shape[0], L, 1 if outgoing else 0,
                                    ops._ptr(self.status), ops._stream_ptr(self.device)), "tmu_contract")
        return x

    def emit_residual(self, x, z, w, mix_eps, out):
        lib = _lib.load()
        B, rows, cols = z.shape[0], z.shape[1], z.shape[2]
        _lib.check(lib.tmu_emit_residual_ex(ops._ptr(x), ops._ptr(z), ops._ptr(out), B, rows, cols,
                                            ctypes.byref(w.struct), w.c_z, w.c, float(mix_eps),
                                            ops._ptr(self.status), ops._stream_ptr(self.device)),
                   "tmu_emit_residual_ex")
        return out


class DistExchange:
    """The two collectives of the sharded update over a torch.distributed process group."""

    def __init__(self, group=None):
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, local):
        """Every rank's ``local`` stacked along a new leading dim: [P, *local.shape]."""
        out = torch.empty((self.size * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
        return out.view((self.size,) + tuple(local.shape))

    def all_to_all(self, send):
        """send[q] goes to rank q; returns recv with recv[q] from rank q (same shape as send)."""
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send.contiguous(), group=self.group)
        return recv

    def all_gather_start(self, local):
        """Start an all-gather of ``local``; returns ([P, *local.shape] buffer, handle).  NCCL runs it
        on its own stream, so kernels enqueued before ``wait(handle)`` overlap the transfer."""
        out = torch.empty((self.size * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        work = dist.all_gather_into_tensor(out, local.contiguous(), group=self.group, async_op=True)
        return out.view((self.size,) + tuple(local.shape)), work

    def wait(self, handle):
        """Order the current stream (CPU: block) after an ``all_gather_start``."""
        handle.wait()


class _SharedPair:
    """Two persistent device buffers of one shape that every peer maps once through CUDA IPC
    (``tmu_ipc_export`` / ``tmu_ipc_import``), used alternately by successive calls, with an
    interprocess "ready" event (the owner recorded it after writing the buffer) and "read" event
    (a rank recorded it after pulling every peer's buffer of that parity) per buffer."""

    def __init__(self, ex, shape, dtype, device):
        lib = _lib.load()
        P, r = ex.size, ex.rank
        self.ex, self.shape = ex, tuple(shape)
        self.bufs = [torch.empty(shape, dtype=dtype, device=device) for _ in range(2)]
        self.ready = [torch.cuda.Event(interprocess=True) for _ in range(2)]
        self.read = [torch.cuda.Event(interprocess=True) for _ in range(2)]
        for e in self.ready + self.read:  # materialise the events on this device before export
            e.record(torch.cuda.current_stream(device))
        rec = bytearray()
        for b in self.bufs:
            h = ctypes.create_string_buffer(_lib.TMU_IPC_HANDLE_BYTES)
            off = ctypes.c_ulonglong(0)
            _lib.check(lib.tmu_ipc_export(ops._ptr(b), h, ctypes.byref(off)), "tmu_ipc_export")
            rec += h.raw + off.value.to_bytes(8, "little")
        for e in self.ready + self.read:
            rec += bytes(e.ipc_handle())
        mine = torch.frombuffer(bytearray(rec), dtype=torch.uint8).to(device)
        every = torch.empty(P * mine.numel(), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, mine, group=ex.group)
        every = every.view(P, -1).cpu().numpy().tobytes()
        n = mine.numel()
        self.peer_bufs, self.peer_ready, self.peer_read = {}, {}, {}
        for q in range(P):
            if q == r:
                continue
            blob = every[q * n:(q + 1) * n]
            ptrs = []
            for i in range(2):
                h = blob[i * 72:i * 72 + 64]
                off = int.from_bytes(blob[i * 72 + 64:i * 72 + 72], "little")
                ptr = ctypes.c_void_p()
                _lib.check(lib.tmu_ipc_import(h, off, ctypes.byref(ptr)), "tmu_ipc_import")
                ptrs.append(ptr.value)
            self.peer_bufs[q] = ptrs
            ev = [blob[144 + 64 * i:144 + 64 * (i + 1)] for i in range(4)]
            self.peer_ready[q] = [torch.cuda.Event.from_ipc_handle(device, ev[i]) for i in range(2)]
            self.peer_read[q] = [torch.cuda.Event.from_ipc_handle(device, ev[2 + i]) for i in range(2)]
        self.nbytes = self.bufs[0].numel() * self.bufs[0].element_size()
        self.calls = 0

    def for_write(self, device):
        """This call's buffer; the current stream first waits until every peer has finished
        copying what it held two calls ago."""
        par = self.calls & 1
        if self.calls >= 2:
            cur = torch.cuda.current_stream(device)
            for q in self.peer_read:
                cur.wait_event(self.peer_read[q][par])
        return self.bufs[par]

    def publish(self):
        """Mark this call's buffer written (on the current stream) and meet the peers at a host
        barrier, so every wait they enqueue next sees this record.  Returns the parity."""
        par = self.calls & 1
        self.calls += 1
        self.ready[par].record(torch.cuda.current_stream())
        dist.barrier(group=self.ex.host_group)
        return par

    def close(self):
        lib = _lib.load()
        for ptrs in self.peer_bufs.values():
            for p in ptrs:
                lib.tmu_ipc_close(ctypes.c_void_p(p))
        self.peer_bufs = {}


def channel_pull_jobs(rank: int, P: int, c: int, Lr: int, pitch: int, groups: int, dst_base: int,
                      esize: int = 2) -> list:
    """The pitched copies that bring rank ``rank`` its c/P channels of a and b over the whole grid.

    Source: every rank's [2, c, Lr, pitch] row slab (a, then b); destination: this rank's
    [2, c/P, P * Lr, pitch] buffer at address ``dst_base``.  One job per channel group g and
    tensor t, as (dst, dst_pitch, src_off, src_pitch, width, height, dst_step): from rank q, the
    group's c/P/groups channels (runs of Lr * pitch elements) into rows [q Lr, (q + 1) Lr) of each
    destination channel (dst + q * dst_step).  Jobs are ordered by group, a before b."""
    cp = c // P
    cg = cp // groups
    blk = Lr * pitch * esize
    jobs = []
    for g in range(groups):
        for t in range(2):
            dst = dst_base + (t * cp + g * cg) * P * blk
            jobs.append((dst, P * blk, (t * c + rank * cp + g * cg) * blk, blk, blk, cg, blk))
    return jobs


def row_pull_job(rank: int, P: int, cp: int, L: int, pitch: int, groups: int, g: int, dst_base: int,
                 esize: int = 2) -> tuple:
    """The pitched copy that brings rank ``rank`` channel group g of x for its rows: from every rank
    q's [c/P / groups, L, pitch] buffer of that group, rows [rank Lr, (rank + 1) Lr) of each channel
    (one run of Lr * pitch elements, L * pitch apart) into channels q c/P + g c/P/groups .. of
    this rank's [c, Lr, pitch] buffer at ``dst_base`` (dst + q * dst_step)."""
    cg = cp // groups
    blk = (L // P) * pitch * esize
    return (dst_base + g * cg * blk, blk, rank * blk, L * pitch * esize, blk, cg, cp * blk)


class CopyEngineExchange(DistExchange):
    """The slabs moved by the GPUs' copy engines instead of NCCL kernels.

    Outgoing b: each rank's K1 writes its b slab into one of two persistent buffers
    (alternating per call) that every peer mapped once through CUDA IPC.  Per call the owner
    records an interprocess "ready" event; the ranks meet at a host barrier (gloo), so every
    peer enqueues its wait after that record; each rank's copy stream waits on the peers' ready
    events and pulls their slabs with ``cudaMemcpyAsync`` over NVLink (``tmu_copy_async``) -- no
    SM time, so the local block's contraction runs at full speed beside it -- and records a
    "read" event that the owner waits on before it rewrites the same buffer two calls later.

    Incoming z: the all-to-all and the transpose into column blocks are one pitched copy per
    peer (``tmu_copy2d_async``): rank r pulls, from each peer q's exported row slab
    z_q [Lr, L, c_z], the block of its own columns (Lr rows of Lr * c_z contiguous elements,
    L * c_z apart) straight into slot q of its [P, Lr, Lr, c_z] buffer, with the same
    ready / read protocol.  No kernel reads another GPU's memory.  A mask, when present, still
    travels by NCCL (2 bytes per position against z's 2 c_z)."""

    def __init__(self, group=None, host_group=None):
        super().__init__(group)
        self.host_group = host_group if host_group is not None else dist.new_group(backend="gloo")
        self._b = None
        self._z = None
        self._ab = None  # channel partition: the local a and b row slabs [2, c, Lr, pitch]
        self._xc = None  # channel partition: this rank's channels of x over the grid [c/P, L, pitch]
        self.copy_stream = None

    def _stream(self, device):
        if self.copy_stream is None:
            self.copy_stream = torch.cuda.Stream(device)
            self.copied = torch.cuda.Event()
        return self.copy_stream

    # ---- outgoing b slabs
    def slab_for_write(self, shape, dtype, device):
        """This call's persistent buffer for the local b slab (K1 writes into it)."""
        if self._b is None or self._b.shape != tuple(shape):
            if self._b is not None:
                self._b.close()
            self._b = _SharedPair(self, shape, dtype, device)
            self.parts = torch.empty((self.size,) + tuple(shape), dtype=dtype, device=device)
            dist.barrier(group=self.host_group)
        return self._b.for_write(device)

    def gather_start(self):
        """Publish this call's slab and start pulling the peers' into ``parts``; returns
        (parts [P, *shape], handle).  The local slot of ``parts`` is left unwritten."""
        lib = _lib.load()
        sp = self._b
        par = sp.publish()
        cs = self._stream(sp.bufs[0].device)
        # ``parts`` is rewritten below: the previous call's contractions, which read it on the
        # current stream, must be done first
        cs.wait_stream(torch.cuda.current_stream(sp.bufs[0].device))
        for q, ptrs in sp.peer_bufs.items():
            cs.wait_event(sp.peer_ready[q][par])
            _lib.check(lib.tmu_copy_async(ops._ptr(self.parts[q]), ptrs[par], sp.nbytes, cs.cuda_stream),
                       "tmu_copy_async")
        sp.read[par].record(cs)
        self.copied.record(cs)
        return self.parts, self.copied

    # ---- incoming z column blocks
    def columns(self, z_rows: torch.Tensor, Lr: int) -> torch.Tensor:
        """z_rows [Lr, L, c] (this rank's rows) -> [P, Lr, Lr, c] with slot q = z[q's rows, my
        columns], pulled by the copy engines; the current stream waits for the result."""
        lib = _lib.load()
        device = z_rows.device
        shape = tuple(z_rows.shape)
        if self._z is None or self._z.shape != shape:
            if self._z is not None:
                self._z.close()
            self._z = _SharedPair(self, shape, z_rows.dtype, device)
            self.zt = torch.empty((self.size, Lr, Lr) + shape[2:], dtype=z_rows.dtype, device=device)
            dist.barrier(group=self.host_group)
        sp = self._z
        buf = sp.for_write(device)
        if buf.data_ptr() != z_rows.data_ptr():
            buf.copy_(z_rows)
        par = sp.publish()
        cs = self._stream(device)
        cs.wait_stream(torch.cuda.current_stream(device))
        row_bytes = shape[1] * shape[2] * z_rows.element_size()  # one row of z: L positions x c
        blk = Lr * shape[2] * z_rows.element_size()               # this rank's Lr columns of it
        col0 = self.rank * blk
        for q in range(self.size):
            dst = self.zt[q]
            if q == self.rank:
                src = buf.data_ptr() + col0
            else:
                cs.wait_event(sp.peer_ready[q][par])
                src = sp.peer_bufs[q][par] + col0
            _lib.check(lib.tmu_copy2d_async(ops._ptr(dst), blk, ctypes.c_void_p(src), row_bytes, blk, Lr,
                                            cs.cuda_stream), "tmu_copy2d_async")
        sp.read[par].record(cs)
        done = torch.cuda.Event()
        done.record(cs)
        torch.cuda.current_stream(device).wait_event(done)
        return self.zt

    # ---- channel partition (ChannelShardedTrimul)
    def _pull_blocks(self, sp, jobs, wait=True):
        """Publish this call's buffer of ``sp`` and, for each job (dst, dst_pitch, src_off,
        src_pitch, width, height, dst_step), pull from every rank q (this one included) ``height``
        rows of ``width`` bytes at byte offset ``src_off`` of q's buffer (rows ``src_pitch`` apart)
        to ``dst + q * dst_step`` (rows ``dst_pitch`` apart): one pitched copy per rank and job on
        the copy stream.  Returns one event per job, recorded after that job's copies; with
        ``wait`` the current stream waits for the last."""
        lib = _lib.load()
        device = sp.bufs[0].device
        par = sp.publish()
        cs = self._stream(device)
        # the destinations may still be read by earlier work; this rank's own block is written there
        cs.wait_stream(torch.cuda.current_stream(device))
        for q in range(self.size):
            if q != self.rank:
                cs.wait_event(sp.peer_ready[q][par])
        events = []
        for dst, dst_pitch, src_off, src_pitch, width, height, dst_step in jobs:
            for q in range(self.size):
                base = sp.bufs[par].data_ptr() if q == self.rank else sp.peer_bufs[q][par]
                _lib.check(lib.tmu_copy2d_async(ctypes.c_void_p(dst + q * dst_step), dst_pitch,
                                                ctypes.c_void_p(base + src_off), src_pitch, width, height,
                                                cs.cuda_stream), "tmu_copy2d_async")
            ev = torch.cuda.Event()
            ev.record(cs)
            events.append(ev)
        sp.read[par].record(cs)
        if wait:
            torch.cuda.current_stream(device).wait_event(events[-1])
        return events

    def row_slabs(self, c: int, Lr: int, pitch: int, device) -> torch.Tensor:
        """This call's persistent [2, c, Lr, pitch] buffer for the local a and b (K1 writes them)."""
        shape = (2, c, Lr, pitch)
        if self._ab is None or self._ab.shape != shape:
            if self._ab is not None:
                self._ab.close()
            self._ab = _SharedPair(self, shape, torch.float16, device)
            self.ab_ch = torch.empty((2, c // self.size, self.size * Lr, pitch), dtype=torch.float16, device=device)
            dist.barrier(group=self.host_group)
        return self._ab.for_write(device)

    def to_channels(self, groups: int = 1):
        """a, b of this rank's c/P channels over the whole grid, [c/P, L, pitch] each: from every
        rank q its rows of those channels (runs of Lr * pitch contiguous elements), pulled in
        ``groups`` consecutive channel groups.  Returns (a, b, events): event g completes when
        group g has landed; the caller orders its readers after them."""
        _, c, Lr, pitch = self._ab.shape
        jobs = channel_pull_jobs(self.rank, self.size, c, Lr, pitch, groups, self.ab_ch.data_ptr())
        events = self._pull_blocks(self._ab, jobs, wait=False)
        return self.ab_ch[0], self.ab_ch[1], events[1::2]

    def channel_slabs(self, cp: int, L: int, pitch: int, device, groups: int = 1) -> list:
        """This call's persistent buffers for this rank's channels of x, one [c/P / groups, L, pitch]
        buffer per channel group (K2 writes them group by group)."""
        cg = cp // groups
        shape = (cg, L, pitch)
        if self._xc is None or len(self._xc) != groups or self._xc[0].shape != shape:
            for sp in self._xc or []:
                sp.close()
            self._xc = [_SharedPair(self, shape, torch.float16, device) for _ in range(groups)]
            self.x_rows = torch.empty((self.size * cp, L // self.size, pitch), dtype=torch.float16, device=device)
            dist.barrier(group=self.host_group)
        return [sp.for_write(device) for sp in self._xc]

    def to_rows(self, g: int = 0):
        """Publish channel group g of x and pull from every rank q its group-g channels of this
        rank's rows (runs of Lr * pitch contiguous elements, L * pitch apart) into [c, Lr, pitch];
        after the last group the current stream waits for all of them.  Returns that buffer."""
        groups = len(self._xc)
        sp = self._xc[g]
        cg, L, pitch = sp.shape
        self._pull_blocks(sp, [row_pull_job(self.rank, self.size, cg * groups, L, pitch, groups, g,
                                            self.x_rows.data_ptr())], wait=g == groups - 1)
        return self.x_rows

    def wait(self, handle):
        torch.cuda.current_stream().wait_event(handle)

    def close(self):
        """Release the imported peer mappings (after every rank is done with them)."""
        pairs = (self._b, self._z, self._ab, *(self._xc or []))
        if all(sp is None for sp in pairs):
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.host_group)
        for sp in pairs:
            if sp is not None:
                sp.close()
        self._b = self._z = self._ab = self._xc = None


class LocalExchange:
    """The exchange of a single rank (P = 1): the collectives are identities."""

    size, rank = 1, 0

    def all_gather(self, local):
        return local.unsqueeze(0)

    def all_gather_start(self, local):
        return local.unsqueeze(0), None

    def wait(self, handle):
        pass

    def all_to_all(self, send):
        return send


class RowShardedTrimul:
    """Triangle update of a pair tensor row-sharded over the ranks of ``group`` (B = 1).

    ``NCCL_SMS``: SMs left free during the overlapped contraction steps.

    ``exchange`` replaces the process-group collectives (an object with ``size``, ``rank``,
    ``all_to_all``, ``all_gather_start`` and ``wait`` as in :class:`DistExchange`)."""

    NCCL_SMS = 16

    def __init__(self, L: int, group=None, device=None, stages=None, exchange=None):
        self.exchange = exchange if exchange is not None else DistExchange(group)
        self.P = self.exchange.size
        self.rank = self.exchange.rank
        if L % self.P:
            raise ValueError(f"L={L} is not divisible by the {self.P} ranks")
        self.L = L
        self.Lr = L // self.P
        if self.P > 1 and self.Lr % 128:
            raise ValueError("rows per rank must be a multiple of 128 (the contraction's B-operand tiles)")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.stages = stages if stages is not None else CudaStages(self.device)
        # SMs the contraction may use while a block of b is in flight (the rest run NCCL's copy)
        self.contract_ctas = 0
        if self.P > 1 and self.device.type == "cuda":
            self.contract_ctas = max(1, torch.cuda.get_device_properties(self.device).multi_processor_count
                                     - self.NCCL_SMS)

    def _to_columns(self, t):
        """[Lr(my rows), L, ...] -> [P(source), Lr(source rows), Lr(my columns), ...]."""
        P, Lr = self.P, self.Lr
        if hasattr(self.exchange, "columns") and t.dim() == 3:  # z: one pitched copy per peer
            return self.exchange.columns(t, Lr)
        # [Lr, P, Lr, ...] -> [P(dest), Lr, Lr, ...]: one copy with Lr*c contiguous elements per run
        send = t.reshape((Lr, P, Lr) + tuple(t.shape[2:])).transpose(0, 1).contiguous()
        return self.exchange.all_to_all(send)

    def __call__(self, z_local: torch.Tensor, mask_local, w: ops.TrimulWeights, outgoing: bool,
                 mix_eps: float = ops.MIX_EPS_FP16, out: torch.Tensor | None = None) -> torch.Tensor:
        """z_local: [1, Lr, L, c_z] fp16 (this rank's rows); mask_local: [1, Lr, L] fp16 or None."""
        L, Lr, P = self.L, self.Lr, self.P
        cz = w.c_z
        if tuple(z_local.shape) != (1, Lr, L, cz):
            raise ValueError(f"z_local must be [1, {Lr}, {L}, {cz}], got {tuple(z_local.shape)}")
        z_local = z_local.contiguous()
        out = torch.empty_like(z_local) if out is None else out
        b_out = None
        if hasattr(self.exchange, "slab_for_write"):
            b_out = self.exchange.slab_for_write((w.c, Lr, ops.row_pitch(L)), torch.float16, z_local.device)
        if outgoing:
            layout = (1, Lr, L, Lr * L * cz, L * cz, cz, Lr * L, L, 1)
            a, b = self.stages.project_gate(z_local, layout, None if mask_local is None else mask_local.contiguous(), w,
                                            b_out=b_out)
        else:
            zt = self._to_columns(z_local[0])  # [P, Lr(k within source), Lr(i), cz]: z[k, i] at k*Lr*cz + i*cz
            mt = None
            if mask_local is not None:
                mt = self._to_columns(mask_local[0])  # [P, Lr(k), Lr(i)]: mask[k, i] at k*Lr + i
            layout = (1, Lr, L, L * Lr * cz, cz, Lr * cz, L * Lr, 1, Lr)
            a, b = self.stages.project_gate(zt, layout, mt, w, b_out=b_out)
        x = self._contract_ring(a, b)
        return self.stages.emit_residual(x, z_local, w, mix_eps, out)

    def _contract_ring(self, a, b_local):
        """x = a [all ranks' b]^T, [Bc, Lr, pitch(L)].  The all-gather of b runs on NCCL's stream
        while the local block is contracted into its column block of x on a grid that leaves
        SMs to NCCL; then the other blocks are contracted (one call per contiguous run of them)."""
        P, r, Lr, L = self.P, self.rank, self.Lr, self.L
        if P == 1:
            return self.stages.contract(a, b_local.unsqueeze(0), Lr, L, L, Lr)
        Bc = a.shape[0]
        x = torch.empty(Bc, Lr, ops.row_pitch(L), dtype=a.dtype, device=a.device)
        if hasattr(self.exchange, "gather_start"):  # copy engines: no SMs taken from the contraction
            parts, handle = self.exchange.gather_start()
            ctas = 0
        else:
            parts, handle = self.exchange.all_gather_start(b_local)  # [P, Bc, Lr, pitch(L)]
            ctas = self.contract_ctas
        self.stages.contract(a, b_local.unsqueeze(0), Lr, Lr, L, Lr, x=x[:, :, r * Lr:], max_ctas=ctas)
        self.exchange.wait(handle)
        for q0, q1 in ((0, r), (r + 1, P)):  # the remote blocks before and after this rank's
            if q1 > q0:
                self.stages.contract(a, parts[q0:q1], Lr, (q1 - q0) * Lr, L, Lr, x=x[:, :, q0 * Lr:])
        return x


class ChannelShardedTrimul:
    """Triangle update of a row-sharded pair tensor, the contraction sharded over channels (B = 1).

    Rank r holds rows [r*Lr, (r+1)*Lr) of z, as for :class:`RowShardedTrimul`, and returns the
    same rows of z + update.  The row partition must bring every rank all of b, so the bytes a
    rank receives grow towards b's size as P grows while its share of the contraction falls as
    1/P.  The contraction is independent per channel (mlx_trunk.py:84-88: one L x L x L product
    per channel d), so this driver moves channels instead:

      K1 on the local rows, all c channels -> a, b [c, Lr, pitch]
      all-to-all: rank r receives every rank's rows of its channels [rc, (r+1)c) / P
                                           -> a, b [c/P, L, pitch] over the whole grid
      K2 on those channels, the single-GPU kernel (outgoing or incoming form: the incoming
         update needs no transposed z)      -> x [c/P, L, pitch]
      all-to-all back to row ownership     -> x [c, Lr, pitch]
      K3 on the local rows.

    A rank receives (P-1)/P^2 of a, b and x per update: falling as 1/P.  With the copy-engine
    exchange each all-to-all is one pitched copy per rank, tensor and channel group from the
    peers' exported buffers (K1 and K2 write straight into them), and the c/P channels go through
    in ``groups`` groups so that the copies of one group overlap the contraction of another; any
    other exchange (NCCL, gloo, threads) runs ``all_to_all`` on [P, c/P, Lr, pitch] blocks.
    Needs c % P == 0.
    """

    def __init__(self, L: int, group=None, device=None, stages=None, exchange=None, groups: int = 4):
        self.exchange = exchange if exchange is not None else DistExchange(group)
        self.P = self.exchange.size
        self.rank = self.exchange.rank
        if L % self.P:
            raise ValueError(f"L={L} is not divisible by the {self.P} ranks")
        self.L, self.Lr = L, L // self.P
        self.groups = groups  # channel groups pipelined through the copy-engine exchange
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.stages = stages if stages is not None else CudaStages(self.device)

    def _to_channels(self, t):
        """[c, Lr, pitch] (my rows) -> [c/P, L, pitch] (my channels) through ``all_to_all``."""
        P, Lr = self.P, self.Lr
        c, pitch = t.shape[0], t.shape[2]
        recv = self.exchange.all_to_all(t.reshape(P, c // P, Lr, pitch))  # [P(source rows), c/P, Lr, pitch]
        return recv.permute(1, 0, 2, 3).reshape(c // P, P * Lr, pitch)

    def _to_rows(self, x):
        """[c/P, L, pitch] (my channels) -> [c, Lr, pitch] (my rows) through ``all_to_all``."""
        P, Lr = self.P, self.Lr
        cp, pitch = x.shape[0], x.shape[2]
        send = x.reshape(cp, P, Lr, pitch).permute(1, 0, 2, 3).contiguous()  # send[q] = q's rows
        return self.exchange.all_to_all(send).reshape(P * cp, Lr, pitch)  # [P(source channels) * c/P, ...]

    def __call__(self, z_local: torch.Tensor, mask_local, w: ops.TrimulWeights, outgoing: bool,
                 mix_eps: float = ops.MIX_EPS_FP16, out: torch.Tensor | None = None) -> torch.Tensor:
        """z_local: [1, Lr, L, c_z] fp16 (this rank's rows); mask_local: [1, Lr, L] fp16 or None."""
        L, Lr, P = self.L, self.Lr, self.P
        cz, c = w.c_z, w.c
        if c % P:
            raise ValueError(f"c={c} channels do not split over {P} ranks")
        if tuple(z_local.shape) != (1, Lr, L, cz):
            raise ValueError(f"z_local must be [1, {Lr}, {L}, {cz}], got {tuple(z_local.shape)}")
        z_local = z_local.contiguous()
        out = torch.empty_like(z_local) if out is None else out
        pitch = ops.row_pitch(L)
        ex = self.exchange
        engines = P > 1 and hasattr(ex, "row_slabs")
        layout = (1, Lr, L, Lr * L * cz, L * cz, cz, Lr * L, L, 1)
        mask = None if mask_local is None else mask_local.contiguous()
        if engines:
            # K1 into the exported row slabs; then per channel group: its a, b land (copy stream),
            # K2 contracts it (this stream) while the next group lands, and its x goes back to
            # the rows' owners while the next group is contracted
            cp = c // P
            groups = self.groups if cp % self.groups == 0 else 1
            cg = cp // groups
            ab = ex.row_slabs(c, Lr, pitch, z_local.device)
            self.stages.project_gate(z_local, layout, mask, w, b_out=ab[1], a_out=ab[0])
            a_ch, b_ch, landed = ex.to_channels(groups)
            xs = ex.channel_slabs(cp, L, pitch, z_local.device, groups)
            cur = torch.cuda.current_stream(z_local.device)
            for g in range(groups):
                cur.wait_event(landed[g])
                self.stages.contract_full(a_ch[g * cg:(g + 1) * cg], b_ch[g * cg:(g + 1) * cg], L, outgoing, x=xs[g])
                x = ex.to_rows(g)
        else:
            a, b = self.stages.project_gate(z_local, layout, mask, w)
            x_ch = self.stages.contract_full(self._to_channels(a), self._to_channels(b), L, outgoing)
            x = self._to_rows(x_ch)
        return self.stages.emit_residual(x, z_local, w, mix_eps, out)
