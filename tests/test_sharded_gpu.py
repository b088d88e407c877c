"""GPU parity of the slab entry points and of the row-sharded triangle update.

* ``tmu_project_gate_ex`` on a transposed stride layout must give exactly what the square entry
  point gives on the explicitly transposed tensor (same kernel, same values, only the addressing
  differs); on a rectangular slab it is checked against the oracle's projections.
* ``tmu_contract_ex`` with a B operand made of gathered row blocks is checked against float64.
* ``tmu_emit_residual_ex`` on a rectangular slab is checked against the oracle.
* ``RowShardedTrimul`` and ``ChannelShardedTrimul`` are run for P ranks emulated by threads on
  one GPU (the collectives become stacks of the ranks' buffers) and, where two GPUs exist, for
  two NCCL ranks (NCCL collectives, or the copy engines over CUDA IPC); all are compared with the
  unsharded oracle under the same error bounds as the unsharded kernels.
"""

from __future__ import annotations

import ctypes
import os
import threading

import pytest
import torch

from esmfold2_mlx_b200 import _lib, ops
from esmfold2_mlx_b200.sharded import ChannelShardedTrimul, CudaStages, RowShardedTrimul
from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_mask, pair_tensor, trimul_biases
from oracle import trimul_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ulp16(x: float) -> float:
    import math
    x = max(abs(x), 2.0**-14)
    return 2.0 ** (math.floor(math.log2(x)) - 10)


def _trunk_and_pair(L, seed, n_pad=0, biases=False):
    trunk = FoldingTrunk(1, 128, 128, hidden=256, seed=seed + 7, ln_noise=0.1)
    z = pair_tensor(1, L, 128, seed).half().float()
    mask = pair_mask(1, L, n_pad) if n_pad else None
    bias = {d: trimul_biases(128, 128, seed + 31 + i) for i, d in enumerate(("out", "in"))} if biases else None
    return trunk, z, mask, bias


def _weights(trunk, direction, bias):
    tri = getattr(trunk.blocks[0], "tri_mul_" + direction)
    b = None if bias is None else bias[direction]
    return ops.TrimulWeights.from_module(tri, DEV, b), orc.trimul_params(tri, True, b)


@pytest.mark.parametrize("L,n_pad", [(200, 0), (256, 17)])
def test_project_gate_ex_transposed_strides_match_square(L, n_pad):
    trunk, z, mask, bias = _trunk_and_pair(L, seed=L, n_pad=n_pad, biases=True)
    w, _ = _weights(trunk, "in", bias)
    zd = z.half().to(DEV)
    md = None if mask is None else mask.half().to(DEV)
    st = CudaStages(DEV)
    layout = (1, L, L, L * L * 128, 128, L * 128, L * L, 1, L)  # element (i, k) = z[k, i]
    a_t, b_t = st.project_gate(zd, layout, md, w)
    zt = zd.transpose(1, 2).contiguous()
    mt = None if md is None else md.transpose(1, 2).contiguous()
    a_r, b_r = ops.project_gate(zt, mt, w)
    torch.cuda.synchronize()
    assert ops.read_status(st.status)[0] == 0
    assert torch.equal(a_t[:, :, :L], a_r[:, :, :L])
    assert torch.equal(b_t[:, :, :L], b_r[:, :, :L])


@pytest.mark.parametrize("rows,cols,row0,n_pad", [(128, 300, 64, 0), (40, 256, 200, 13)])
def test_project_gate_ex_row_slab_matches_oracle(rows, cols, row0, n_pad):
    L = cols
    trunk, z, mask, bias = _trunk_and_pair(L, seed=rows + cols, n_pad=n_pad, biases=bool(n_pad))
    w, p = _weights(trunk, "out", bias)
    zs = z[:, row0:row0 + rows]
    ms = None if mask is None else mask[:, row0:row0 + rows]
    _, a_ref, b_ref = orc.project_gate_fp16(p, zs, ms)
    zd = zs.half().contiguous().to(DEV)
    md = None if ms is None else ms.half().contiguous().to(DEV)
    st = CudaStages(DEV)
    a, b = st.project_gate(zd, (1, rows, cols, rows * cols * 128, cols * 128, 128, rows * cols, cols, 1), md, w)
    torch.cuda.synchronize()
    assert ops.read_status(st.status)[0] == 0
    for name, got, ref in (("a", a, a_ref), ("b", b, b_ref)):
        got = got[:, :, :cols].float().cpu().reshape(ref.shape)
        diff = (got - ref).abs()
        assert float(diff.max()) <= 2 * _ulp16(float(ref.abs().max())), name
        assert float((diff > 0).float().mean()) < 0.05, name


@pytest.mark.parametrize("P,R,K,Bc", [(2, 128, 256, 4), (3, 128, 384, 2), (2, 256, 300, 3), (4, 128, 200, 2)])
def test_contract_ex_gathered_parts_matches_fp64(P, R, K, Bc):
    g = torch.Generator().manual_seed(P * 1000 + R + K)
    M, N = 192, P * R
    kp = ops.row_pitch(K)
    a = torch.full((Bc, M, kp), 1e4, dtype=torch.float16)  # pad columns must never be read
    bp = torch.full((P, Bc, R, kp), -1e4, dtype=torch.float16)
    a[:, :, :K] = torch.randn(Bc, M, K, generator=g).half()
    bp[..., :K] = torch.randn(P, Bc, R, K, generator=g).half()
    st = CudaStages(DEV)
    x = st.contract(a.to(DEV), bp.to(DEV), M, N, K, R)
    torch.cuda.synchronize()
    assert ops.read_status(st.status)[0] == 0
    A = a[:, :, :K].double()
    Bf = bp[..., :K].double().permute(1, 0, 2, 3).reshape(Bc, N, K)
    ref = A @ Bf.transpose(1, 2)
    got = x[:, :, :N].double().cpu()
    err = (got - ref).abs()
    assert bool((err <= 2 * ref.abs().clamp_min(1.0) * 2.0**-11 + 1e-2).all()), float(err.max())


def test_contract_ex_column_blocks_through_row_pitch():
    """Each block of b contracted on its own into its column block of one wide x (ldx > N)."""
    g = torch.Generator().manual_seed(11)
    P, R, K, Bc, M = 3, 128, 384, 2, 128
    kp = ops.row_pitch(K)
    a = torch.randn(Bc, M, kp, generator=g).half()
    bp = torch.randn(P, Bc, R, kp, generator=g).half()
    a[:, :, K:] = 0
    bp[..., K:] = 0
    st = CudaStages(DEV)
    ad, bd = a.to(DEV), bp.to(DEV)
    full = st.contract(ad, bd, M, P * R, K, R)
    x = torch.full((Bc, M, ops.row_pitch(P * R) + 8), float("nan"), dtype=torch.float16, device=DEV)
    for q in (2, 0, 1):  # one block on a capped grid (fewer CTAs than tiles)
        st.contract(ad, bd[q:q + 1], M, R, K, R, x=x[:, :, q * R:], max_ctas=7 if q == 0 else 0)
    torch.cuda.synchronize()
    assert ops.read_status(st.status)[0] == 0
    assert torch.equal(x[:, :, :P * R], full[:, :, :P * R])
    assert bool(torch.isnan(x[:, :, P * R:]).all())  # nothing written past N


@pytest.mark.parametrize("rows,cols,outgoing", [(128, 300, True), (56, 256, False)])
def test_emit_residual_ex_row_slab_matches_oracle(rows, cols, outgoing):
    direction = "out" if outgoing else "in"
    trunk, z, _, bias = _trunk_and_pair(cols, seed=rows + 3 * cols, biases=True)
    w, p = _weights(trunk, direction, bias)
    zs = z[:, :rows]
    g = torch.Generator().manual_seed(rows)
    xg = (torch.randn(1, 128, rows, cols, generator=g) * 3).half().float()
    ref, _ = orc.emit_residual_fp16(p, zs, xg, ops.MIX_EPS_FP16)
    x = torch.zeros(128, rows, ops.row_pitch(cols), dtype=torch.float16)
    x[:, :, :cols] = xg.reshape(128, rows, cols).half()
    zd = zs.half().contiguous().to(DEV)
    st = CudaStages(DEV)
    out = st.emit_residual(x.to(DEV), zd, w, ops.MIX_EPS_FP16, torch.empty_like(zd))
    torch.cuda.synchronize()
    assert ops.read_status(st.status)[0] == 0
    diff = (out.float().cpu() - ref).abs()
    assert float(diff.max()) <= 4 * _ulp16(float(ref.abs().max()))


class _ThreadExchange:
    """Collectives between P threads that share one GPU and its default stream."""

    def __init__(self, hub, rank):
        self.hub, self.rank, self.size = hub, rank, hub["P"]

    def _swap(self, t):
        self.hub["slots"][self.rank] = t.contiguous()
        self.hub["barrier"].wait()
        got = list(self.hub["slots"])
        self.hub["barrier"].wait()
        return got

    def all_gather(self, local):
        return torch.stack(self._swap(local))

    def all_to_all(self, send):
        slots = self._swap(send)
        return torch.stack([slots[q][self.rank] for q in range(self.size)])

    def all_gather_start(self, local):
        return torch.stack(self._swap(local)), None

    def wait(self, handle):
        pass


class _SerialStages(CudaStages):
    """One launch at a time across the emulating threads."""

    lock = threading.Lock()

    def project_gate(self, *a, **kw):
        with self.lock:
            return super().project_gate(*a, **kw)

    def contract(self, *a, **kw):
        with self.lock:
            return super().contract(*a, **kw)

    def contract_full(self, *a, **kw):
        with self.lock:
            return super().contract_full(*a, **kw)

    def emit_residual(self, *a):
        with self.lock:
            return super().emit_residual(*a)


def _emulate(P, L, z, mask, w, outgoing, driver=RowShardedTrimul):
    hub = {"P": P, "slots": [None] * P, "barrier": threading.Barrier(P, timeout=120)}
    Lr = L // P
    outs, errs, stages = [None] * P, [], []

    def rank_fn(r):
        try:
            st = _SerialStages(DEV)
            stages.append(st)
            sh = driver(L, device=DEV, stages=st, exchange=_ThreadExchange(hub, r))
            zl = z[:, r * Lr:(r + 1) * Lr].contiguous()
            ml = None if mask is None else mask[:, r * Lr:(r + 1) * Lr].contiguous()
            outs[r] = sh(zl, ml, w, outgoing)
        except Exception as e:  # noqa: BLE001 - reported below
            errs.append(e)
            hub["barrier"].abort()

    th = [threading.Thread(target=rank_fn, args=(r,)) for r in range(P)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    if errs:
        raise errs[0]
    torch.cuda.synchronize()
    for st in stages:
        assert ops.read_status(st.status)[0] == 0
    return torch.cat(outs, dim=1)


@pytest.mark.parametrize("P,L,n_pad", [(2, 256, 0), (2, 512, 30), (4, 512, 0), (3, 384, 11)])
@pytest.mark.parametrize("outgoing", [True, False])
def test_row_sharded_emulated_ranks_match_oracle(P, L, n_pad, outgoing):
    direction = "out" if outgoing else "in"
    trunk, z, mask, bias = _trunk_and_pair(L, seed=L + P, n_pad=n_pad, biases=bool(n_pad))
    w, p = _weights(trunk, direction, bias)
    zd = z.half().to(DEV)
    md = None if mask is None else mask.half().to(DEV)
    got = _emulate(P, L, zd, md, w, outgoing).float().cpu()
    ref16 = orc.trimul_fp16(p, z, mask, outgoing)
    exact = orc.trimul_fp32(orc.trimul_params(getattr(trunk.blocks[0], "tri_mul_" + direction), False,
                                              None if bias is None else bias[direction]),
                            z.double(), mask, outgoing, dtype=torch.float64)
    e_ref, e_got = orc.error_stats(exact, ref16), orc.error_stats(exact, got)
    assert e_got["finite"]
    assert e_got["max_abs"] <= 2 * e_ref["max_abs"] + 1e-3, (e_got, e_ref)
    assert e_got["rel_l2"] <= 2 * e_ref["rel_l2"] + 1e-3, (e_got, e_ref)
    assert float((got - ref16).abs().max()) <= 4 * _ulp16(float(ref16.abs().max()))
    # the unsharded kernels on the same inputs
    full = ops.trimul(zd, md, w, outgoing).float().cpu()
    assert float((got - full).abs().max()) <= 2 * _ulp16(float(full.abs().max()))


@pytest.mark.parametrize("P,L,n_pad", [(2, 256, 0), (4, 512, 30), (8, 512, 0)])
@pytest.mark.parametrize("outgoing", [True, False])
def test_channel_sharded_emulated_ranks_match_oracle(P, L, n_pad, outgoing):
    direction = "out" if outgoing else "in"
    trunk, z, mask, bias = _trunk_and_pair(L, seed=L + P + 5, n_pad=n_pad, biases=bool(n_pad))
    w, p = _weights(trunk, direction, bias)
    zd = z.half().to(DEV)
    md = None if mask is None else mask.half().to(DEV)
    got = _emulate(P, L, zd, md, w, outgoing, ChannelShardedTrimul).float().cpu()
    ref16 = orc.trimul_fp16(p, z, mask, outgoing)
    assert float((got - ref16).abs().max()) <= 4 * _ulp16(float(ref16.abs().max()))
    # the same kernels on the same values: the unsharded update, bit for bit
    full = ops.trimul(zd, md, w, outgoing).float().cpu()
    assert torch.equal(got, full)


def _nccl_worker(rank, port, q, L, copy_engines=False, driver="rows"):
    import datetime
    import traceback

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        res = {}
        for direction, outgoing in (("out", True), ("in", False)):
            trunk, z, mask, bias = _trunk_and_pair(L, seed=L + 11, n_pad=21, biases=True)
            w, p = _weights(trunk, direction, bias)
            Lr = L // 2
            zl = z[:, rank * Lr:(rank + 1) * Lr].half().contiguous().cuda()
            ml = mask[:, rank * Lr:(rank + 1) * Lr].half().contiguous().cuda()
            Driver = RowShardedTrimul if driver == "rows" else ChannelShardedTrimul
            if copy_engines:
                from esmfold2_mlx_b200.sharded import CopyEngineExchange
                if direction == "out":
                    ex = CopyEngineExchange()
                sh = Driver(L, exchange=ex)
            else:
                sh = Driver(L)
            out = sh(zl, ml, w, outgoing)
            full = torch.empty(2, Lr, L, 128, dtype=torch.float16, device=out.device)
            dist.all_gather_into_tensor(full, out)
            assert ops.read_status(sh.stages.status)[0] == 0
            if rank == 0:
                got = full.reshape(1, L, L, 128).float().cpu()
                ref16 = orc.trimul_fp16(p, z, mask, outgoing)
                res[direction] = (float((got - ref16).abs().max()), _ulp16(float(ref16.abs().max())))
        if copy_engines:
            ex.close()
        q.put((rank, res))
    except Exception:  # noqa: BLE001 - reported to the parent instead of hanging the peer
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.timeout(600)
@pytest.mark.parametrize("copy_engines", [False, True])
@pytest.mark.parametrize("driver", ["rows", "channels"])
def test_sharded_two_nccl_ranks_match_oracle(copy_engines, driver):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 150 + (7 if copy_engines else 0) + (3 if driver == "channels" else 0)
    procs = [ctx.Process(target=_nccl_worker, args=(r, port, q, 512, copy_engines, driver)) for r in range(2)]
    for pr in procs:
        pr.start()
    out = dict(q.get(timeout=400) for _ in range(2))
    for pr in procs:
        pr.join(timeout=60)
    for r in range(2):
        assert "error" not in out[r], out[r]["error"]
    for d, (err, ulp) in out[0].items():
        assert err <= 4 * ulp, f"{d}: {err} vs ulp {ulp}"


@pytest.mark.parametrize("driver", [RowShardedTrimul, ChannelShardedTrimul])
@pytest.mark.parametrize("outgoing", [True, False])
def test_sharded_emulated_ranks_wide_pair(outgoing, driver):
    """c_z = c = 256 through the same sharded drivers (P = 2, L = 256)."""
    P, L, cz = 2, 256, 256
    direction = "out" if outgoing else "in"
    trunk = FoldingTrunk(1, cz, cz, hidden=512, seed=41, ln_noise=0.1)
    z = pair_tensor(1, L, cz, 40).half().float()
    mask = pair_mask(1, L, 13)
    tri = getattr(trunk.blocks[0], "tri_mul_" + direction)
    w, p = ops.TrimulWeights.from_module(tri, DEV), orc.trimul_params(tri, True)
    zd, md = z.half().to(DEV), mask.half().to(DEV)
    got = _emulate(P, L, zd, md, w, outgoing, driver).float().cpu()
    ref16 = orc.trimul_fp16(p, z, mask, outgoing)
    assert float((got - ref16).abs().max()) <= 4 * _ulp16(float(ref16.abs().max()))
