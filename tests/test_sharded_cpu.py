"""Row-sharded tri-mul data movement on CPU ranks (gloo, world_size 2).

``RowShardedTrimul`` drives the exchange (all-to-all into columns for the incoming form, an
asynchronous all-gather of b) and hands slabs to three stages; ``ChannelShardedTrimul`` moves
a and b to channel ownership and x back by two all-to-alls.  The copy-engine form of those
all-to-alls is a list of pitched copies per rank; their addresses are checked here for 2, 4 and
8 emulated ranks on host buffers.  Here the stages are the CPU oracle applied to
exactly the buffers the CUDA kernels would see -- the strided (possibly transposed) z view, the
[B*c, rows, pitch] projections, b blocks contracted into column blocks of x -- so the test checks
the layouts and the collectives; the kernels themselves are checked on the GPU.
"""

from __future__ import annotations

import os
import types

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from esmfold2_mlx_b200 import ops
from esmfold2_mlx_b200.sharded import ChannelShardedTrimul, RowShardedTrimul
from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_mask, pair_tensor
from oracle import trimul_oracle as orc

L = 256
P = 2


class OracleStages:
    def __init__(self, p):
        self.p = p

    def project_gate(self, z, layout, mask, w, b_out=None, a_out=None):
        B, rows, cols, sb, sr, sc, msb, msr, msc = layout
        zv = torch.as_strided(z.reshape(-1).float(), (B, rows, cols, 128), (sb, sr, sc, 1))
        mv = None if mask is None else torch.as_strided(mask.reshape(-1).float(), (B, rows, cols), (msb, msr, msc))
        _, a, b = orc.project_gate_fp16(self.p, zv, mv)
        pitch = ops.row_pitch(cols)

        def pack(t):  # [B, c, rows, cols] -> [B*c, rows, pitch] fp16 (pad never read)
            o = torch.full((B * 128, rows, pitch), float("nan"), dtype=torch.float16)
            o[:, :, :cols] = t.reshape(B * 128, rows, cols).half()
            return o

        pb = pack(b)
        if b_out is not None:
            b_out.copy_(pb)
            pb = b_out
        return pack(a), pb

    def contract(self, a, b_parts, M, N, K, rows_per_part, x=None, max_ctas=0):
        Pp, Bc, R, pitch = b_parts.shape
        assert Pp * R == N and R == rows_per_part
        b_full = b_parts.permute(1, 0, 2, 3).reshape(Bc, N, pitch)
        xv = orc.r16(a[:, :, :K].float() @ b_full[:, :, :K].float().transpose(1, 2))
        if x is None:
            x = torch.full((Bc, M, ops.row_pitch(N)), float("nan"), dtype=torch.float16)
        x[:, :, :N] = xv.half()
        return x

    def contract_full(self, a, b, L, outgoing, x=None):
        A, Bm = a[:, :, :L].float(), b[:, :, :L].float()
        xv = orc.r16(A @ Bm.transpose(1, 2) if outgoing else A.transpose(1, 2) @ Bm)
        if x is None:
            x = torch.full(a.shape, float("nan"), dtype=torch.float16)
        x[:, :, :L] = xv.half()
        return x

    def emit_residual(self, x, z, w, mix_eps, out):
        B, rows, cols = z.shape[0], z.shape[1], z.shape[2]
        xg = x[:, :, :cols].float().reshape(B, 128, rows, cols)
        z_new, _ = orc.emit_residual_fp16(self.p, z.float(), xg, mix_eps)
        out.copy_(z_new.half())
        return out


def _worker(rank, port, q):
    import datetime
    import traceback

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=P, timeout=datetime.timedelta(seconds=60))
    try:
        _run(rank, q)
    except Exception:  # report instead of leaving the peer blocked in a collective
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        dist.destroy_process_group()


def _run(rank, q):
    if True:
        trunk = FoldingTrunk(1, 128, 128, hidden=256, seed=5, ln_noise=0.1)
        z = pair_tensor(1, L, 128, 77).half()
        mask = pair_mask(1, L, 9).half()
        Lr = L // P
        w = types.SimpleNamespace(c_z=128, c=128)
        res = {}
        for (direction, outgoing), Driver in ((d, D) for D in (RowShardedTrimul, ChannelShardedTrimul)
                                              for d in (("out", True), ("in", False))):
            p = orc.trimul_params(getattr(trunk.blocks[0], "tri_mul_" + direction), True)
            st = Driver(L, device="cpu", stages=OracleStages(p))
            z_loc = z[:, rank * Lr:(rank + 1) * Lr].contiguous()
            m_loc = mask[:, rank * Lr:(rank + 1) * Lr].contiguous()
            out = st(z_loc, m_loc, w, outgoing)
            full = torch.empty(P * 1, Lr, L, 128, dtype=torch.float16)
            dist.all_gather_into_tensor(full, out)
            got = full.reshape(1, L, L, 128).float()
            if rank == 0:
                ref = orc.trimul_fp16(p, z.float(), mask.float(), outgoing)
                res[f"{Driver.__name__}/{direction}"] = float((got - ref).abs().max())
        q.put((rank, res))


@pytest.mark.timeout(600)
def test_row_and_channel_sharded_match_unsharded_oracle():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(P)]
    for pr in procs:
        pr.start()
    out = dict(q.get(timeout=300) for _ in range(P))
    for pr in procs:
        pr.join(timeout=60)
    for r in range(P):
        assert "error" not in out[r], out[r]["error"]
    for pr in procs:
        assert pr.exitcode == 0
    res = out[0]
    assert set(res) == {f"{n}/{d}" for n in ("RowShardedTrimul", "ChannelShardedTrimul") for d in ("out", "in")}
    for d, err in res.items():
        assert err <= 4e-3, f"{d}: sharded vs unsharded max |diff| {err}"


def _copy2d(dst, dst_pitch, src, src_pitch, width, height):
    """cudaMemcpy2D's semantics on host addresses."""
    import ctypes

    for r in range(height):
        ctypes.memmove(dst + r * dst_pitch, src + r * src_pitch, width)


@pytest.mark.parametrize("P,groups", [(2, 1), (2, 4), (4, 2), (4, 4), (8, 4)])
def test_channel_exchange_copy_jobs_move_the_right_blocks(P, groups):
    """The copy-engine channel partition's pitched copies (``channel_pull_jobs``,
    ``row_pull_job``), applied to host buffers of P emulated ranks, give every rank exactly the
    all-to-all results of the generic path: a, b of its channels over the grid, then x of its rows."""
    from esmfold2_mlx_b200.sharded import channel_pull_jobs, row_pull_job

    c, Lr, pitch = 32, 6, 16
    L, cp = P * Lr, c // P
    g = torch.Generator().manual_seed(P * 10 + groups)
    ab = [torch.randn(2, c, Lr, pitch, generator=g).half() for _ in range(P)]  # each rank's row slabs
    full = torch.cat(ab, dim=2)  # [2, c, L, pitch]: the whole grid
    for r in range(P):
        dst = torch.zeros(2, cp, L, pitch, dtype=torch.float16)
        for job in channel_pull_jobs(r, P, c, Lr, pitch, groups, dst.data_ptr()):
            d, dp, off, sp_, w, h, step = job
            for q in range(P):
                _copy2d(d + q * step, dp, ab[q].data_ptr() + off, sp_, w, h)
        assert torch.equal(dst, full[:, r * cp:(r + 1) * cp])
    # x: rank q holds channels [q cp, (q + 1) cp) of the grid, split into `groups` buffers
    x = torch.randn(c, L, pitch, generator=g).half()
    cg = cp // groups
    xbufs = [[x[q * cp + k * cg:q * cp + (k + 1) * cg].clone() for k in range(groups)] for q in range(P)]
    for r in range(P):
        dst = torch.zeros(c, Lr, pitch, dtype=torch.float16)
        for k in range(groups):
            d, dp, off, sp_, w, h, step = row_pull_job(r, P, cp, L, pitch, groups, k, dst.data_ptr())
            for q in range(P):
                _copy2d(d + q * step, dp, xbufs[q][k].data_ptr() + off, sp_, w, h)
        assert torch.equal(dst, x[:, r * Lr:(r + 1) * Lr])
