#!/usr/bin/env python
"""Benchmark: triangle-multiplicative-update pair-cells/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {b200,reference}]

Workload: one fold, L = 238, c_z = c = 128, fp16 storage, outgoing then
incoming tri-mul back to back, the last 24 residues masked out (pair mask m_i*m_j), Linear
weights N(0, 1/fan_in) plus N(0, 0.02) biases, z ~ N(0, 1).  One step = tri-mul out + tri-mul in
= 2 * 238^2 pair-cells.  Inputs are seeded synthetic tensors with the reference's shapes
(Biohub checkpoints are not available); weights are random-init with the reference architecture.

* value      device throughput: inputs resident in HBM, each step one CUDA-graph replay of the
             two C-ABI tri-mul calls, timed with CUDA events on the launching stream; L2 is
             flushed (256 MiB write) between steps, outside the timed intervals.
* e2e        the same metric through the public API (``ops.trimul``) with the step's input
             copied from pinned host memory and the result copied back, inside the interval.
* roofline   the kernel with the largest time share, from per-kernel CUDA events captured in a
             second graph (K1 project+gate, K2 contraction, K3 emit+residual, each launched
             through its own C-ABI entry point); algorithmic bytes / FLOPs per launch are
             the per-cell figures in ``_kernel_costs`` times the cells a launch processes;
             peaks from MEASURED_PEAKS.json.
* N > 1      one process per GPU (torchrun), each rank runs its own fold (seed + rank): weak
             scaling, no collective on the data path; times are the max over ranks.
* --impl reference   the reference's CPU path (the PyTorch restatement in oracle/, all host
             threads) on the same workload; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "tri-mul pair-cells/s (L^2 x tri-mul blocks / s)"
UNIT = "pair-cells/s"
C_Z = C = 128


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _init_pg(ws, local, backend):
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)


def _max_over_ranks(x: float, ws: int, device) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.lines: list[str] = []
        self.proc = None
        self.device_index = device_index

    def start(self):
        ident = str(self.device_index)
        try:
            uuid = str(torch.cuda.get_device_properties(self.device_index).uuid)
            if uuid:
                ident = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", ident, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


WORKLOADS = ("c2", "c1", "c4", "L2048", "c5", "c2w", "L2048w", "pc", "pc476")
PAIR_COND_L = {"pc": 238, "pc476": 476}  # diffusion pair conditioning, one fold of L residues
SHARDED_WORKLOADS = ("c5",)


def _workload(rank: int, device, name: str = "c2", world: int = 1):
    """Seeded weights and one step's input for a named configuration (``synthetic.workload``,
    the same inputs the parity tests check); ``device=None`` keeps everything on the CPU
    (reference arm)."""
    from esmfold2_mlx_b200.synthetic import workload

    wl = workload(name, rank, world)
    w = None
    if device is not None:
        from esmfold2_mlx_b200 import ops

        w = {d: ops.TrimulWeights.from_module(getattr(wl.trunk.blocks[0], "tri_mul_" + d), device, wl.biases[d])
             for d in ("out", "in")}
    return wl.cfg, wl.trunk, wl.biases, w, wl.z, wl.mask


def _cpu_sample(trunk, biases, z, mask, min_seconds: float):
    """Oracle (CPU) out+in tri-muls on the first fold of the workload, repeated until
    ``min_seconds`` have elapsed.  Returns (pair-cells processed, seconds)."""
    from oracle import trimul_oracle as orc

    p = {d: orc.trimul_params(getattr(trunk.blocks[0], "tri_mul_" + d), True, biases[d]) for d in ("out", "in")}
    zf = z[:1].float()
    mf = None if mask is None else mask[:1].float()
    L = zf.shape[1]
    n, t0 = 0, time.perf_counter()
    while True:
        z1 = orc.trimul_fp16(p["out"], zf, mf, True)
        orc.trimul_fp16(p["in"], z1, mf, False)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return n * 2 * L * L, el


def run_reference(args, ws, rank, local):
    """The reference arm: the reference's CPU path (the oracle port, all host threads) on the
    same workload; one step = out+in tri-mul of one fold (a bounded sample for batched configs)."""
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    if args.workload in PAIR_COND_L:
        _reference_pair_cond(args, threads)
        return
    cfg, trunk, biases, _, z, mask = _workload(0, None, args.workload)
    L = cfg.L
    from oracle import trimul_oracle as orc

    p = {d: orc.trimul_params(getattr(trunk.blocks[0], "tri_mul_" + d), True, biases[d]) for d in ("out", "in")}
    zf = z[:1].float()
    mf = None if mask is None else mask[:1].float()
    for _ in range(args.warmup):
        orc.trimul_fp16(p["in"], orc.trimul_fp16(p["out"], zf, mf, True), mf, False)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.trimul_fp16(p["in"], orc.trimul_fp16(p["out"], zf, mf, True), mf, False)
    el = time.perf_counter() - t0
    cells = 2 * L * L
    value = cells * args.steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": _config_dict(cfg, 1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps, each out+in tri-mul of one fold at L={L}; "
                                   "oracle/trimul_oracle.py on torch CPU (fp32 math, fp16 rounding points)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _reference_pair_cond(args, threads):
    """Reference arm of the pair-conditioning workloads: the oracle port of pair_biases
    (mlx_diffusion16.py:81-87) on the host cores, one fold per step."""
    from esmfold2_mlx_b200.synthetic import DiffusionHead, pair_tensor
    from oracle import pair_cond_oracle as pco

    L = PAIR_COND_L[args.workload]
    p = pco.pair_cond_params(DiffusionHead(seed=11))
    zt, rp = pair_tensor(1, L, 256, 12) * 20.0, pair_tensor(1, L, 256, 13)
    for _ in range(min(args.warmup, 1)):
        pco.pair_biases_fp16(p, zt, rp)
    steps = max(1, min(args.steps, 5))
    t0 = time.perf_counter()
    for _ in range(steps):
        pco.pair_biases_fp16(p, zt, rp)
    el = time.perf_counter() - t0
    value = L * L * steps / el
    line = {"impl": "reference", "metric": "pair_cond_cells_per_s", "value": value, "unit": "pair-cells/s",
            "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": f"{args.workload}_pair_conditioning_L{L}", "B": 1, "L": L},
            "cpu_baseline": {"value": value, "unit": "pair-cells/s", "cores": threads, "kind": "port",
                             "sample": f"{steps} x pair_biases of one fold at L={L}; oracle/pair_cond_oracle.py"},
            "e2e": {"value": value, "unit": "pair-cells/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _config_dict(cfg, ws):
    return {"workload": cfg.name, "L": cfg.L, "B": cfg.B, "c_z": cfg.c_z, "c": cfg.c, "directions": ["out", "in"],
            "mask_pad": cfg.n_pad, "biases": cfg.biases, "parallelism": f"folds x{ws} (one fold group per GPU)",
            "l2": "flushed between steps (256 MiB write, outside the timed intervals)",
            "launch": "one CUDA graph per step"}


def _kernel_costs(L: int, B: int, masked: bool, C_Z: int = 128, C: int = 128):
    """Algorithmic bytes and FLOPs per launch of each kernel (one tri-mul)."""
    cells = B * L * L
    return {
        "K1_project_gate": {"bytes": cells * (2 * C_Z + (2 if masked else 0) + 2 * 2 * C),
                            "flops": cells * 2 * C_Z * 4 * C},
        "K2_contract": {"bytes": cells * (2 * 2 * C + 2 * C), "flops": cells * 2 * C * L},
        "K3_emit_residual": {"bytes": cells * (2 * C + 2 * C_Z + 2 * C_Z), "flops": cells * 2 * (C * C_Z + C_Z * C_Z)},
    }


def _trunk_recycle(device, flush, reps: int = 3):
    """ms per trunk recycle on BASELINE config 3: a 16-block pair stack (tri-mul out, tri-mul in,
    ReLU transition 128 -> 512 -> 128), L = 384, run for 3 recycles with z fed back; random
    N(0, 1/fan_in) weights (seed 2), z0 ~ N(0, 1).  The whole 3-recycle forward is one CUDA graph
    through the public module (CUDAFoldingTrunk); L2 flushed before each timed replay."""
    from esmfold2_mlx_b200.synthetic import recycle_workload
    from esmfold2_mlx_b200.trunk import CUDAFoldingTrunk

    cfg, trunk, z0 = recycle_workload("c3")
    mod = CUDAFoldingTrunk(trunk, device=device)
    z0 = z0.to(device)

    def forward():
        z = z0
        for _ in range(cfg.recycles):
            z = mod(z)
        return z

    out = forward()  # eager warm-up (first-call host setup, workspace)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = forward()
    for _ in range(2):
        flush.zero_()
        g.replay()
    torch.cuda.synchronize()
    ms = []
    for _ in range(reps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        e1.synchronize()
        ms.append(e0.elapsed_time(e1))
    finite = bool(torch.isfinite(out).all())
    per_recycle = statistics.median(ms) / cfg.recycles
    L = cfg.L
    cells = 2 * cfg.blocks * L * L  # tri-mul pair cells per recycle
    del g

    # K4 alone: the fused transition of block 0, 20 launches in one graph on an L2-flushed z
    from esmfold2_mlx_b200 import ops

    tw = mod.params[0]["tw"]
    zt = z0.half().contiguous()
    st = ops.new_status(device)
    ops.transition(zt, tw, out=zt, status=st)
    gk = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gk):
        for _ in range(20):
            ops.transition(zt, tw, out=zt, status=st)
    flush.zero_()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record()
    gk.replay()
    k1.record()
    k1.synchronize()
    k4_us = k0.elapsed_time(k1) * 1e3 / 20
    del gk
    hbm, tflops, _ = _peaks()
    k4_flops = L * L * 2 * 2 * C_Z * tw.hidden * (1.5 if tw.activation == "swiglu" else 1.0)
    k4_bytes = L * L * 2 * 2 * C_Z
    return {"workload": cfg.name, "L": L, "blocks": cfg.blocks, "recycles": cfg.recycles,
            "ms_per_recycle": round(per_recycle, 4), "trimul_pair_cells_per_s": cells / (per_recycle * 1e-3),
            "roofline_ms_per_recycle": 2.4,
            "transition": "ReLU 128->512->128, fused kernel K4 (tmu_transition)",
            "k4_us_per_launch": round(k4_us, 2),
            "k4_roofline": {"bound": "tensor", "achieved": round(k4_flops / (k4_us * 1e-6) / 1e12, 1),
                            "peak": tflops, "unit": "TFLOP/s", "frac": round(k4_flops / (k4_us * 1e-6) / 1e12 / tflops, 4),
                            "hbm_gbs": round(k4_bytes / (k4_us * 1e-6) / 1e9, 1)},
            "output_finite": finite}


def _c5_measure(ws, rank, local, steps, warmup, nccl=False, parity=True, partition="rows", groups=4) -> dict:
    """one fold of L = 3072, outgoing then incoming tri-mul, its rows split over
    the N ranks (strong scaling: the total work is fixed).

    ``partition="rows"`` (the configuration's own scheme): each rank projects its rows (for the
    incoming form from its columns, which the copy engines pull from every rank's rows with one
    pitched copy per peer), b is exchanged while the local block is contracted (copy engines over
    NVLink by default, ``nccl``: an NCCL all-gather), and each rank finishes its rows.
    ``partition="channels"``: each rank projects its rows, two all-to-alls move a and b to channel
    ownership and x back (copy engines, or NCCL with ``nccl``), and the contraction of c/N
    channels over the whole grid runs between them.  Eager launches; the inputs per rank
    (>= 302 MB at N = 8) exceed L2, so no flush is needed."""
    from esmfold2_mlx_b200 import ops
    from esmfold2_mlx_b200.sharded import (ChannelShardedTrimul, CopyEngineExchange, DistExchange, LocalExchange,
                                           RowShardedTrimul)

    device = torch.device("cuda", local)
    cfg, trunk, _, w, z_host, _ = _workload(rank, device, "c5", ws)
    L = cfg.L
    if ws == 1:
        ex = LocalExchange()
    elif nccl:
        ex = DistExchange(None)
    else:
        ex = CopyEngineExchange(None)
    if partition == "rows":
        sh = RowShardedTrimul(L, device=device, exchange=ex)
    else:
        sh = ChannelShardedTrimul(L, device=device, exchange=ex, groups=groups)
    Lr = sh.Lr
    z0 = z_host.to(device)
    z1 = torch.empty_like(z0)
    z2 = torch.empty_like(z0)

    def step(zin):
        sh(zin, None, w["out"], True, out=z1)
        return sh(z1, None, w["in"], False, out=z2)

    for _ in range(max(3, warmup)):
        step(z0)
    torch.cuda.synchronize()
    _barrier(ws)
    sampler = ClockSampler(local)
    sampler.start()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    _barrier(ws)
    for e0, e1 in evs:
        e0.record()
        step(z0)
        e1.record()
    torch.cuda.synchronize()
    _barrier(ws)
    clocks = sampler.stop()
    step_ms = sum(e0.elapsed_time(e1) for e0, e1 in evs)
    ms_per_step = _max_over_ranks(step_ms, ws, device) / steps
    cells = 2 * L * L
    code, site = ops.read_status(sh.stages.status)
    if code != 0:
        raise RuntimeError(f"device status {code} at site {site:#x}")

    # end to end: this rank's rows from pinned host memory and back, inside the interval
    zh = z_host.pin_memory()
    outh = torch.empty_like(z_host).pin_memory()
    z_in = torch.empty_like(z0)
    e2e_ms = 0.0
    for i in range(steps + 1):
        _barrier(ws)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        z_in.copy_(zh, non_blocking=True)
        outh.copy_(step(z_in), non_blocking=True)
        e1.record()
        e1.synchronize()
        if i >= 1:
            e2e_ms += e0.elapsed_time(e1)
    e2e_ms = _max_over_ranks(e2e_ms, ws, device) / steps
    pitch = ops.row_pitch(L)
    if partition == "rows":
        # bytes each rank receives per step: (P-1)/P of b for both directions, plus z's column blocks
        recv = (ws - 1) * (2 * cfg.c * Lr * pitch * 2 + Lr * Lr * cfg.c_z * 2)
    else:
        # per direction, from each peer: its rows of this rank's c/P channels of a and b, and this
        # rank's rows of the peer's channels of x
        recv = 2 * 3 * (ws - 1) * (cfg.c // ws) * Lr * pitch * 2
    link_gbs = 770.0  # measured peer copy per direction on this pool's NVLink (bytes / s / 1e9)
    comm_ms = recv / (link_gbs * 1e9) * 1e3
    flops = 2 * (2 * cfg.c * L) * Lr * L  # the contraction's FLOPs per rank per step (both directions)
    hbm, tflops, peak_kind = _peaks()
    tensor_ms = flops / (tflops * 1e12) * 1e3
    # K1 and K3 of both directions on this rank's Lr x L cells, at the HBM peak (algorithmic bytes)
    costs = _kernel_costs(L, 1, False, cfg.c_z, cfg.c)
    k13_ms = 2 * (costs["K1_project_gate"]["bytes"] + costs["K3_emit_residual"]["bytes"]) * (Lr / L) / (hbm * 1e9) * 1e3
    # the exchange overlaps the contraction, not the position-wise kernels before and after it
    bound_ms = k13_ms + max(comm_ms, tensor_ms)
    res = {"workload": cfg.name, "L": L, "B": 1, "c_z": cfg.c_z, "n_gpus": ws, "scaling": "strong",
           "value": cells / (ms_per_step * 1e-3), "unit": UNIT, "ms_per_step": round(ms_per_step, 4),
           "steps": steps,
           "parallelism": (f"rows x{ws} (row-sharded fold)" if partition == "rows" else
                           f"rows x{ws} (row-sharded fold), contraction over c/{ws} channels per rank"),
           "exchange": ("none" if ws == 1 else
                        ("NCCL all-gather of b" if nccl else
                         "copy engines over NVLink (CUDA IPC): b slabs by cudaMemcpyAsync, z column blocks "
                         "(incoming all-to-all + transpose) by one cudaMemcpy2DAsync per peer")
                        if partition == "rows" else
                        ("NCCL all-to-all of a, b and x" if nccl else
                         "copy engines over NVLink (CUDA IPC): a, b to channel ownership and x back to rows, "
                         f"one cudaMemcpy2DAsync per peer, tensor and channel group ({groups} groups, each "
                         "group's copies overlapping another group's contraction)")),
           "roofline": {"bound": "nvlink" if comm_ms > tensor_ms else "tensor",
                        "recv_bytes_per_rank_per_step": recv, "nvlink_gbs_per_direction": link_gbs,
                        "comm_floor_ms": round(comm_ms, 4), "contraction_floor_ms": round(tensor_ms, 4),
                        "k1_k3_hbm_floor_ms": round(k13_ms, 4), "step_floor_ms": round(bound_ms, 4),
                        "frac": round(bound_ms / ms_per_step, 4),
                        "note": "floor = K1 + K3 algorithmic bytes / measured HBM peak + max(received bytes / "
                                "measured 770 GB/s peer copy, contraction FLOPs / "
                                f"{tflops} TFLOP/s {peak_kind} peak); frac = floor / measured step"},
           "e2e": {"value": cells / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": zh.numel() * 2,
                   "d2h_bytes_per_step": outh.numel() * 2, "ms_per_step": round(e2e_ms, 4)},
           "gpu_launches": 6 * steps, "clocks": clocks}
    if parity:
        res["parity"] = _c5_parity(cfg, trunk, z2 if ws > 1 else z2, z1, rank, ws)
    if hasattr(ex, "close"):
        ex.close()
    return res


def _c5_parity(cfg, trunk, z2, z1, rank, ws) -> dict | None:
    """Rows [124, 128) of the row-sharded step's outgoing result (rank 0 holds them) against the
    oracle's row slab; the exact reference here is float32 arithmetic without the fp16 rounding
    points (2^13 finer than the fp16 errors it measures; the test suite uses float64)."""
    if rank != 0:
        _barrier(ws)
        return None
    from esmfold2_mlx_b200.synthetic import pair_rows
    from oracle import trimul_oracle as orc

    threads = torch.get_num_threads()
    torch.set_num_threads(len(os.sched_getaffinity(0)))  # the other ranks wait at the barrier below
    z = pair_rows(cfg.L, cfg.c_z, cfg.seed, 0, cfg.L).half()
    rows = range(124, 128)
    tri = trunk.blocks[0].tri_mul_out
    ref16 = orc.trimul_rows(orc.trimul_params(tri, True), z, None, True, rows)
    exact = orc.trimul_rows(orc.trimul_params(tri, False), z, None, True, rows, exact=True,
                            exact_dtype=torch.float32)
    res = orc.parity(exact, ref16, z1[:, rows.start:rows.stop].float().cpu())
    res.update({"rows": [rows.start, rows.stop], "direction": "out",
                "exact": "float32 arithmetic (no fp16 rounding points)"})
    torch.set_num_threads(threads)
    _barrier(ws)
    return res


def run_sharded(args, ws, rank, local):
    """``--workload c5``: the row-sharded long fold as the line's own metric."""
    from esmfold2_mlx_b200 import _lib

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _lib.check(_lib.load().tmu_device_check(), "tmu_device_check")
    res = _c5_measure(ws, rank, local, args.steps, args.warmup, args.c5_nccl, not args.no_parity,
                      args.c5_partition, args.c5_groups)
    if rank == 0:
        line = {"metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
                "config": {"workload": res["workload"], "L": res["L"], "B": 1, "c_z": res["c_z"],
                           "directions": ["out", "in"], "parallelism": res["parallelism"],
                           "exchange": res["exchange"], "l2": "inputs larger than L2 (no flush)", "launch": "eager"},
                "e2e": res["e2e"], "gpu_launches": res["gpu_launches"], "roofline": res["roofline"],
                "parity": res.get("parity"), "clocks": res["clocks"]}
        print(json.dumps(line), flush=True)


def _c4_measure(ws, rank, local, steps, warmup, flush, stream, parity=True) -> dict:
    """BASELINE config 4 as a fixed batch: 64 folds of L = 146 split 64 / N per rank (strong
    scaling, no collective on the data path), out + in per fold; max over ranks."""
    device = torch.device("cuda", local)
    case = TrimulCase("c4", rank, device, stream, world=ws)
    for _ in range(max(3, warmup)):
        flush.zero_()
        case.g_step.replay()
    torch.cuda.synchronize()
    _barrier(ws)
    ms = _max_over_ranks(case.time_steps(flush, steps), ws, device) / steps
    code, site = case.ops.read_status(case.wsp.status)
    if code != 0:
        raise RuntimeError(f"device status {code} at site {site:#x}")
    total_cells = 2 * case.cfg.B * case.cfg.L * case.cfg.L  # all 64 folds, out + in
    tr = case.trace(flush, 5)
    dom, kernels = case.kernel_table(tr)
    res = {"workload": case.cfg.name, "L": case.cfg.L, "folds": case.cfg.B, "folds_per_gpu": case.cfg.B // ws,
           "n_gpus": ws, "scaling": "strong", "value": total_cells / (ms * 1e-3), "unit": UNIT,
           "ms_per_step": round(ms, 5), "steps": steps, "dominant_kernel": dom, "kernels": kernels,
           "parallelism": f"folds x{ws} (64 / {ws} folds per GPU, no collective)"}
    if parity and rank == 0:
        res["parity"] = case.parity(folds=[0, case.z0.shape[0] - 1])
    _barrier(ws)
    return res


class TrimulCase:
    """One configuration's out+in tri-mul step on the GPU: inputs resident in HBM, the step as a
    CUDA graph of the two ``tmu_trimul`` calls (the timed form), and the same six kernels launched
    through the per-kernel entry points, each with its own armed trace block (the traced form:
    the same programmatic-dependent-launch chain, timed kernel by kernel on the device)."""

    NAMES = ("K1_project_gate", "K2_contract", "K3_emit_residual")

    def __init__(self, name: str, rank: int, device, stream, world: int = 1):
        from esmfold2_mlx_b200 import _lib, ops

        self.ops, self.lib = ops, _lib.load()
        self.cfg, self.trunk, self.biases, self.w, self.z_host, self.mask_host = _workload(rank, device, name, world)
        cfg = self.cfg
        self.B = self.z_host.shape[0]  # folds on this rank
        self.device, self.stream = device, stream
        self.z0 = self.z_host.to(device)
        self.mask = None if self.mask_host is None else self.mask_host.to(device)
        self.z1, self.z2 = torch.empty_like(self.z0), torch.empty_like(self.z0)
        self.wsp = ops.Workspace()
        self.wsp.get(self.B, cfg.L, cfg.c_z, cfg.c, device)
        Lp = ops.row_pitch(cfg.L)
        self.a = torch.empty(self.B * cfg.c, cfg.L, Lp, dtype=torch.float16, device=device)
        self.b, self.x = torch.empty_like(self.a), torch.empty_like(self.a)
        self.trace_st = torch.zeros(6, 256, dtype=torch.uint8, device=device)
        self.cells = 2 * self.B * cfg.L * cfg.L  # pair-cells per step on this rank (out + in)
        self.step()
        self.step_traced()
        torch.cuda.synchronize()
        self.g_step, self.g_trace = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.g_step, stream=stream):
            self.step()
        with torch.cuda.graph(self.g_trace, stream=stream):
            self.step_traced()
        torch.cuda.synchronize()

    def step(self):
        ops = self.ops
        ops.trimul(self.z0, self.mask, self.w["out"], True, out=self.z1, workspace=self.wsp)
        ops.trimul(self.z1, self.mask, self.w["in"], False, out=self.z2, workspace=self.wsp)

    def step_traced(self):
        ops, lib, cfg = self.ops, self.lib, self.cfg
        sp = ops._stream_ptr(self.device)
        zin = self.z0
        for k, (d, outgoing, zout) in enumerate((("out", True, self.z1), ("in", False, self.z2))):
            wt = self.w[d]
            st = [self.trace_st[3 * k + j] for j in range(3)]
            _check(lib.tmu_project_gate(ops._ptr(zin), ops._ptr(self.mask), ops.ctypes.byref(wt.struct), self.B, cfg.L,
                                        cfg.c_z, cfg.c, ops._ptr(self.a), ops._ptr(self.b), ops._ptr(st[0]), sp), "K1")
            _check(lib.tmu_contract(ops._ptr(self.a), ops._ptr(self.b), ops._ptr(self.x), self.B * cfg.c, cfg.L,
                                    1 if outgoing else 0, ops._ptr(st[1]), sp), "K2")
            _check(lib.tmu_emit_residual(ops._ptr(self.x), ops._ptr(zin), ops._ptr(zout), ops.ctypes.byref(wt.struct),
                                         self.B, cfg.L, cfg.c_z, cfg.c, ops.MIX_EPS_FP16, ops._ptr(st[2]), sp), "K3")
            zin = zout

    def time_steps(self, flush, steps: int) -> float:
        """Milliseconds of ``steps`` graph replays, each bracketed by events, L2 flushed between."""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            flush.zero_()
            e0.record()
            self.g_step.replay()
            e1.record()
        torch.cuda.synchronize()
        return sum(e0.elapsed_time(e1) for e0, e1 in evs)

    def trace(self, flush, reps: int) -> dict:
        """Replays of the traced form: per launch, the span from its first CTA past the dependency
        wait to its last CTA's exit (%globaltimer), averaged over ``reps`` L2-flushed replays."""
        spans = [[0.0] * 6 for _ in range(reps)]
        gaps = [[0.0] * 6 for _ in range(reps)]
        step_ms = []
        for r in range(reps):
            flush.zero_()
            for i in range(6):
                self.ops.trace_arm(self.trace_st[i])
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            self.g_trace.replay()
            e1.record()
            e1.synchronize()
            step_ms.append(e0.elapsed_time(e1))
            marks = [self.ops.trace_read(self.trace_st[i]) for i in range(6)]
            for i, (t0, t1) in enumerate(marks):
                spans[r][i] = (t1 - t0) * 1e-3
                if i:
                    gaps[r][i] = (t0 - marks[i - 1][1]) * 1e-3
        mean = lambda rows, i: statistics.fmean(row[i] for row in rows)  # noqa: E731
        return {"spans_us": [round(mean(spans, i), 3) for i in range(6)],
                "gaps_us": [round(mean(gaps, i), 3) for i in range(6)],
                "traced_step_ms": round(statistics.fmean(step_ms), 5)}

    def kernel_table(self, tr: dict) -> tuple[str, dict]:
        """Per kernel: its in-step time (mean span of its two launches), the share of the summed
        spans, and the fraction of the roofline its algorithmic bytes or FLOPs reach in that time."""
        hbm, tflops, _ = _peaks()
        cfg = self.cfg
        costs = _kernel_costs(cfg.L, self.B, self.mask is not None, cfg.c_z, cfg.c)
        total = sum(tr["spans_us"])
        kernels = {}
        for j, n in enumerate(self.NAMES):
            us = 0.5 * (tr["spans_us"][j] + tr["spans_us"][3 + j])
            t = us * 1e-6
            byt, fl = costs[n]["bytes"], costs[n]["flops"]
            bound = "tensor" if fl / (tflops * 1e12) > byt / (hbm * 1e9) else "hbm"
            ach = (fl / t / 1e12) if bound == "tensor" else (byt / t / 1e9)
            pk = tflops if bound == "tensor" else hbm
            kernels[n] = {"us_in_step": round(us, 3), "share": round(2 * us / total, 4), "bound": bound,
                          "achieved": round(ach, 2), "frac": round(ach / pk, 4),
                          "algorithmic_per_launch": costs[n]}
        dom = max(self.NAMES, key=lambda n: kernels[n]["us_in_step"])
        return dom, kernels

    def parity(self, slab_rows: int | None = None, folds=None, exact_dtype=torch.float64) -> dict:
        """The step's outputs (left by the last replay) against the CPU oracle, used as the checker:
        e_cuda vs e_ref (exact float64 update) and the distance in fp16 ulps, per direction, each
        on the same input (in: the CUDA out result).  Large L: rows [124, 124 + slab_rows) only;
        ``folds``: those folds only."""
        from oracle import trimul_oracle as orc

        torch.cuda.synchronize()
        sel = slice(None) if folds is None else list(folds)
        z1h, z2h = self.z1.cpu()[sel], self.z2.cpu()[sel]
        m = None if self.mask_host is None else self.mask_host.float()[sel]
        res = {}
        steps = (("out", True, self.z_host[sel], z1h), ("in", False, z1h, z2h))
        if slab_rows is not None:
            steps = steps[:1]  # the outgoing update; both directions are checked in the test suite
        for d, outgoing, zin, got in steps:
            tri = getattr(self.trunk.blocks[0], "tri_mul_" + d)
            p16 = orc.trimul_params(tri, True, self.biases[d])
            pex = orc.trimul_params(tri, False, self.biases[d])
            if slab_rows is None:
                ref16 = orc.trimul_fp16(p16, zin.float(), m, outgoing)
                exact = orc.trimul_fp32(pex, zin.double(), m, outgoing, dtype=torch.float64)
                res[d] = orc.parity(exact, ref16, got.float())
            else:
                rows = range(124, 124 + slab_rows)
                ref16 = orc.trimul_rows(p16, zin, m, outgoing, rows)
                exact = orc.trimul_rows(pex, zin, m, outgoing, rows, exact=True, exact_dtype=exact_dtype)
                res[d] = orc.parity(exact, ref16, got[:, rows.start:rows.stop].float())
                res[d]["rows"] = [rows.start, rows.stop]
                if exact_dtype != torch.float64:
                    res[d]["exact"] = "float32 arithmetic (no fp16 rounding points)"
        res["checker"] = "oracle/trimul_oracle.py (CPU), after the timed region"
        res["tolerance"] = "e_cuda <= 2 e_ref + 1e-3 (max-abs, rel-L2); max_ulps <= 4"
        res["within_tolerance"] = all(v["within_tolerance"] and v["max_ulps"] <= 4
                                      for k, v in res.items() if isinstance(v, dict))
        return res


def _check(code, where):
    if code != 0:
        from esmfold2_mlx_b200 import _lib

        _lib.check(code, where)


def _case_summary(case, flush, steps, warmup, with_parity=True, slab_rows=None, exact_dtype=torch.float64) -> dict:
    """A sub-measurement of the default line: another configuration's step (value, ms/step,
    in-step kernel table and parity), one GPU."""
    for _ in range(max(3, warmup)):
        flush.zero_()
        case.g_step.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    time.sleep(0.2)
    ms = case.time_steps(flush, steps) / steps
    clocks = sampler.stop()
    tr = case.trace(flush, max(3, min(steps, 10)))
    dom, kernels = case.kernel_table(tr)
    out = {"workload": case.cfg.name, "L": case.cfg.L, "B": case.cfg.B, "c_z": case.cfg.c_z,
           "value": case.cells / (ms * 1e-3), "unit": UNIT, "ms_per_step": round(ms, 5), "steps": steps,
           "dominant_kernel": dom, "kernels": kernels, "trace": tr, "clocks": clocks}
    code, site = case.ops.read_status(case.wsp.status)
    if code != 0:
        raise RuntimeError(f"device status {code} at site {site:#x}")
    if with_parity:
        out["parity"] = case.parity(slab_rows, exact_dtype=exact_dtype)
    return out


def _host_link(device, nbytes: int, reps: int = 10) -> dict:
    """Host-link figures for the e2e leg: pinned H2D and D2H of one step's bytes alone and both
    directions at once, the GPU's NUMA node and this process's CPU affinity."""
    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    hd = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d = torch.empty(nbytes, dtype=torch.uint8, device=device)
    d2 = torch.empty(nbytes, dtype=torch.uint8, device=device)
    s1, s2 = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def timed(fn):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    timed(lambda: d.copy_(h, non_blocking=True))

    def both():
        cur = torch.cuda.current_stream(device)
        s1.wait_stream(cur)
        s2.wait_stream(cur)
        with torch.cuda.stream(s1):
            d.copy_(h, non_blocking=True)
        with torch.cuda.stream(s2):
            hd.copy_(d2, non_blocking=True)
        cur.wait_stream(s1)
        cur.wait_stream(s2)

    t_h2d = timed(lambda: d.copy_(h, non_blocking=True))
    t_d2h = timed(lambda: hd.copy_(d2, non_blocking=True))
    t_both = timed(both)
    numa = None
    try:
        pr = torch.cuda.get_device_properties(device)
        path = f"/sys/bus/pci/devices/{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0/numa_node"
        with open(path) as f:
            numa = int(f.read().strip())
    except (OSError, ValueError, AttributeError):
        numa = None
    aff = sorted(os.sched_getaffinity(0))
    return {"bytes": nbytes, "h2d_gbs": round(nbytes / (t_h2d * 1e-3) / 1e9, 2),
            "d2h_gbs": round(nbytes / (t_d2h * 1e-3) / 1e9, 2),
            "both_directions_gbs_each": round(nbytes / (t_both * 1e-3) / 1e9, 2),
            "gpu_numa_node": numa, "cpu_affinity": f"{aff[0]}-{aff[-1]} ({len(aff)} cpus)" if aff else None}


def run_b200(args, ws, rank, local):
    from esmfold2_mlx_b200 import _lib, ops

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _lib.check(_lib.load().tmu_device_check(), "tmu_device_check")
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=device)
    case = TrimulCase(args.workload, rank, device, stream)
    cfg, w = case.cfg, case.w
    L, B = cfg.L, case.B
    C_Z, C = cfg.c_z, cfg.c  # noqa: N806 - the pair and latent widths of this workload
    mask, z_host, mask_host = case.mask, case.z_host, case.mask_host
    trunk, biases = case.trunk, case.biases
    cells_per_step = case.cells

    for _ in range(max(3, args.warmup)):
        flush.zero_()
        case.g_step.replay()
    torch.cuda.synchronize()
    _barrier(ws)

    # ---------------- timed region: K steps ----------------
    sampler = ClockSampler(local)
    sampler.start()
    torch.cuda.synchronize()
    _barrier(ws)
    step_ms = case.time_steps(flush, args.steps)
    _barrier(ws)
    clocks = sampler.stop()
    step_ms_max = _max_over_ranks(step_ms, ws, device)
    ms_per_step = step_ms_max / args.steps
    value = ws * cells_per_step / (ms_per_step * 1e-3)
    code, site = ops.read_status(case.wsp.status)
    if code != 0:
        raise RuntimeError(f"device status {code} at site {site:#x}")
    z2_timed = case.z2.clone()

    # ---------------- sustained run (clocks under load for >= 0.5 s) ----------------
    n_sus = max(args.steps, int(math.ceil(args.sustain_seconds * 1e3 / max(ms_per_step, 1e-3))))  # timed device time
    sampler2 = ClockSampler(local)
    sampler2.start()
    time.sleep(0.25)
    sus_ms = case.time_steps(flush, n_sus)
    clocks_sus = sampler2.stop()
    sustained = {"steps": n_sus, "ms_per_step": round(sus_ms / n_sus, 5), "device_seconds": round(sus_ms * 1e-3, 3),
                 "value": cells_per_step / (sus_ms / n_sus * 1e-3), "clocks": clocks_sus}

    # ---------------- per-kernel in-step times (traced form of the same chain) ----------------
    tr = case.trace(flush, max(3, min(args.steps, 20)))
    dom, kernels = case.kernel_table(tr)
    hbm, tflops, peak_kind = _peaks()
    traffic = None  # DRAM bytes per launch of the dominant kernel, from a committed ncu capture
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        traffic = json.load(open(tpath)).get(cfg.name, {}).get(dom, {}).get("dram_bytes_per_launch")
    d = kernels[dom]
    roofline = {"kernel": dom, "bound": d["bound"], "achieved": d["achieved"],
                "peak": tflops if d["bound"] == "tensor" else hbm,
                "unit": "TFLOP/s" if d["bound"] == "tensor" else "GB/s", "frac": d["frac"], "traffic": traffic,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json burst)" if peak_kind == "measured" else "fallback",
                "algorithmic_per_launch": d["algorithmic_per_launch"],
                "timing": "in-step: per launch, first CTA past its dependency wait to last CTA exit (%globaltimer), "
                          "in the same PDL-chained launch sequence as the timed step; mean over L2-flushed replays",
                "kernels": kernels, "trace": tr,
                "step_vs_trace": {"timed_ms_per_step": round(ms_per_step, 5),
                                  "sum_of_spans_ms": round(sum(tr["spans_us"]) * 1e-3, 5)}}

    # ---------------- end to end through the public API, host buffers ----------------
    # Every step copies its own input from pinned host memory and reads its result back.  Serial:
    # H2D, compute, D2H, host sync, one step at a time.  Pipelined (the headline): three streams,
    # step k+1's H2D and step k-1's D2H overlap step k's tri-muls (double-buffered device and
    # host buffers, event-ordered), as a serving loop runs; timed from the first H2D to the last
    # D2H on the device.
    zh = z_host.pin_memory()
    mh = None if mask_host is None else mask_host.pin_memory()
    outh = [torch.empty_like(z_host).pin_memory() for _ in range(2)]
    z_in = [torch.empty_like(case.z0) for _ in range(2)]
    m_in = [None if mask is None else torch.empty_like(mask) for _ in range(2)]
    z_mid = [torch.empty_like(case.z0) for _ in range(2)]
    z_out = [torch.empty_like(case.z0) for _ in range(2)]
    wsp2 = [case.wsp, ops.Workspace()]
    wsp2[1].get(B, L, C_Z, C, device)

    def e2e_step(i, s_in, s_out):
        b = i % 2
        with torch.cuda.stream(s_in):
            z_in[b].copy_(zh, non_blocking=True)
            if m_in[b] is not None:
                m_in[b].copy_(mh, non_blocking=True)
        ops.trimul(z_in[b], m_in[b], w["out"], True, out=z_mid[b], workspace=wsp2[b])
        ops.trimul(z_mid[b], m_in[b], w["in"], False, out=z_out[b], workspace=wsp2[b])
        with torch.cuda.stream(s_out):
            outh[b].copy_(z_out[b], non_blocking=True)

    # serial
    e2e_serial = 0.0
    for i in range(args.steps + 2):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        e2e_step(i, stream, stream)
        e1.record()
        e1.synchronize()
        if i >= 2:
            e2e_serial += e0.elapsed_time(e1)
    e2e_serial = _max_over_ranks(e2e_serial, ws, device) / args.steps
    # pipelined: NB buffer sets; each step's input and output copies split in two halves on two
    # streams each (one copy engine per half: a single 14.5 MB H2D beside a D2H ran at 36 GB/s,
    # two halves at 55 GB/s on this pool's boxes)
    NB = 3
    while len(z_in) < NB:
        z_in.append(torch.empty_like(case.z0))
        m_in.append(None if mask is None else torch.empty_like(mask))
        z_mid.append(torch.empty_like(case.z0))
        z_out.append(torch.empty_like(case.z0))
        outh.append(torch.empty_like(z_host).pin_memory())
        wsp2.append(ops.Workspace())
        wsp2[-1].get(B, L, C_Z, C, device)
    s_h2d = [torch.cuda.Stream(device) for _ in range(2)]
    s_d2h = [torch.cuda.Stream(device) for _ in range(2)]
    n_pipe = args.steps + NB
    h2d_done = [torch.cuda.Event() for _ in range(n_pipe)]
    comp_done = [torch.cuda.Event() for _ in range(n_pipe)]
    d2h_done = [torch.cuda.Event() for _ in range(n_pipe)]
    zh_flat, half_in = zh.view(-1), (zh.numel() + 1) // 2
    half_out = (outh[0].numel() + 1) // 2
    torch.cuda.synchronize()
    _barrier(ws)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(s_h2d[0])
    for i in range(n_pipe):
        b = i % NB
        for h, sh_ in enumerate(s_h2d):
            if i >= NB:
                sh_.wait_event(comp_done[i - NB])  # z_in[b] was read by step i-NB's tri-muls
            with torch.cuda.stream(sh_):
                z_in[b].view(-1)[h * half_in:(h + 1) * half_in].copy_(zh_flat[h * half_in:(h + 1) * half_in],
                                                                      non_blocking=True)
                if h == 1 and m_in[b] is not None:
                    m_in[b].copy_(mh, non_blocking=True)
        s_h2d[0].wait_stream(s_h2d[1])
        h2d_done[i].record(s_h2d[0])
        stream.wait_event(h2d_done[i])
        if i >= NB:
            stream.wait_event(d2h_done[i - NB])  # z_out[b] was read by step i-NB's D2H
        ops.trimul(z_in[b], m_in[b], w["out"], True, out=z_mid[b], workspace=wsp2[b])
        ops.trimul(z_mid[b], m_in[b], w["in"], False, out=z_out[b], workspace=wsp2[b])
        comp_done[i].record(stream)
        for h, sd in enumerate(s_d2h):
            sd.wait_event(comp_done[i])
            with torch.cuda.stream(sd):
                outh[b].view(-1)[h * half_out:(h + 1) * half_out].copy_(
                    z_out[b].view(-1)[h * half_out:(h + 1) * half_out], non_blocking=True)
        s_d2h[0].wait_stream(s_d2h[1])
        d2h_done[i].record(s_d2h[0])
    p1.record(s_d2h[0])
    p1.synchronize()
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(p0.elapsed_time(p1), ws, device) / n_pipe
    h2d = zh.numel() * zh.element_size() + (0 if mh is None else mh.numel() * mh.element_size())
    d2h = outh[0].numel() * outh[0].element_size()
    e2e_matches = bool(torch.equal(outh[(n_pipe - 1) % NB].to(device), z2_timed))
    link = _host_link(device, h2d)
    e2e = {"value": ws * cells_per_step / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
           "mode": "pipelined: later steps' H2D and earlier steps' D2H overlap step k (3 buffer sets, each copy "
                   "split in two halves on two streams per direction, events)",
           "serial": {"value": ws * cells_per_step / (e2e_serial * 1e-3), "ms_per_step": round(e2e_serial, 4)},
           "host_link": link, "output_equals_timed_step": e2e_matches,
           "host_link_bound_ms": round(max(h2d / (link["both_directions_gbs_each"] * 1e9),
                                           d2h / (link["both_directions_gbs_each"] * 1e9)) * 1e3, 4)}

    # ---------------- parity of the timed step (oracle as the checker, after timing) ----------------
    case.z2.copy_(z2_timed)
    parity = case.parity() if not args.no_parity else None

    # ---------------- other configurations, N = 1 only ----------------
    recycle = None
    extra = {}
    if ws == 1 and not args.no_trunk:
        recycle = _trunk_recycle(device, flush)
    if ws == 1 and not args.no_extra and args.workload == "c2":
        # L2048w: the released model's width at the metric's second anchor (parity on a row slab in
        # float32, the whole-grid float64 projection being the slow part on the host)
        for name, slab, edt in (("L2048", 8, torch.float64), ("c2w", None, torch.float64),
                                ("L2048w", 8, torch.float32)):
            sub = TrimulCase(name, 0, device, stream)
            extra[name] = _case_summary(sub, flush, min(args.steps, 20), args.warmup, not args.no_parity, slab, edt)
            del sub
            torch.cuda.empty_cache()
    if not args.no_extra and args.workload == "c2":
        # the two multi-GPU configurations, at every N (N = 1 is their scaling baseline)
        extra["c4"] = _c4_measure(ws, rank, local, min(args.steps, 20), args.warmup, flush, stream,
                                  not args.no_parity)
        torch.cuda.empty_cache()
        extra["c5"] = _c5_measure(ws, rank, local, min(args.steps, 10), args.warmup, False, not args.no_parity)
        if ws > 1:  # at N = 1 both partitions run the same three kernels on the whole fold
            try:  # the alternative partition: a failure is reported in its sub-object, not the line
                extra["c5_channels"] = _c5_measure(ws, rank, local, min(args.steps, 10), args.warmup, False,
                                                   not args.no_parity, partition="channels")
            except Exception as e:  # noqa: BLE001
                extra["c5_channels"] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.empty_cache()

    # ---------------- CPU baseline (rank 0, N = 1) ----------------
    cpu = None
    if ws == 1 and not args.no_cpu_baseline and L <= 512:
        threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(threads)
        ncells, el = _cpu_sample(trunk, biases, z_host, mask_host, args.cpu_seconds)
        cpu = {"value": ncells / el, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{ncells // (2 * L * L)} x (out+in tri-mul of one fold at L={L}) in {el:.1f} s; "
                         "oracle/trimul_oracle.py on torch CPU (fp32 math, fp16 rounding points)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": _config_dict(cfg, ws),
            "e2e": e2e, "gpu_launches": 6 * args.steps, "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks,
            "sustained": sustained, "parity": parity, "trunk_recycle": recycle, **extra,
        }
        print(json.dumps(line), flush=True)


def run_pair_cond(args, ws, rank, local):
    """The diffusion head's per-fold pair conditioning (``tmu_pair_cond``: LayerNorm pass + K6,
    2 x (LayerNorm pass + K4 in h mode), LayerNorm pass + K6) on the stand-in head's default shape
    (c_trunk = c_rel = c_pair = 256, hidden 512, 12 blocks x 16 heads).  One step = one fold's
    call; N > 1 runs independent replicas (weak scaling)."""
    from esmfold2_mlx_b200 import _lib, ops, pair_cond
    from esmfold2_mlx_b200.synthetic import DiffusionHead, pair_tensor

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _lib.check(_lib.load().tmu_device_check(), "tmu_device_check")
    L, B = PAIR_COND_L[args.workload], 1
    head = DiffusionHead(seed=11)
    pw = pair_cond.PairCondWeights.from_head(head, device)
    zt_h = (pair_tensor(B, L, 256, 12 + rank) * 20.0).contiguous()
    rp_h = pair_tensor(B, L, 256, 13 + rank).contiguous()
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    zt, rp = zt_h.to(device), rp_h.to(device)
    wbuf = torch.empty(pair_cond.workspace_bytes(B, L, 512, 256, 2), dtype=torch.uint8, device=device)
    out = torch.empty(pw.n_bias // pw.heads, B, pw.heads, L, L, dtype=torch.float16, device=device)
    status = ops.new_status(device)
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=device)

    def step():
        pair_cond.pair_biases(pw, zt, rp, out=out, workspace=wbuf, status=status)

    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    for _ in range(max(3, args.warmup)):
        flush.zero_()
        g.replay()
    torch.cuda.synchronize()
    _barrier(ws)
    sampler = ClockSampler(local)
    sampler.start()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    _barrier(ws)
    for e0, e1 in evs:
        flush.zero_()
        e0.record()
        g.replay()
        e1.record()
    torch.cuda.synchronize()
    _barrier(ws)
    clocks = sampler.stop()
    ms_per_step = _max_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in evs), ws, device) / args.steps
    code, site = ops.read_status(status)
    if code != 0:
        raise RuntimeError(f"device status {code} at site {site:#x}")
    cells = B * L * L
    value = ws * cells / (ms_per_step * 1e-3)
    # algorithmic work per pair cell: proj 2*512*256, 2 transitions x (2*256*1024 + 2*512*256), bias 2*256*192
    flops_cell = 2 * 512 * 256 + 2 * (2 * 256 * 1024 + 2 * 512 * 256) + 2 * 256 * 192
    bytes_cell = 2 * 256 * 4 + pw.n_bias * 2  # fp32 inputs in, fp16 biases out
    hbm, tflops, peak_kind = _peaks()
    ach = flops_cell * cells / (ms_per_step * 1e-3) / 1e12
    roofline = {"kernel": "tmu_pair_cond (8 launches: 4 LayerNorm passes, 2 x K6, 2 x K4 h mode)",
                "bound": "tensor", "achieved": round(ach, 2), "peak": tflops, "unit": "TFLOP/s",
                "frac": round(ach / tflops, 4), "traffic": None,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json burst)" if peak_kind == "measured" else "fallback",
                "algorithmic_per_cell": {"flops": flops_cell, "bytes": bytes_cell},
                "note": "whole-call roofline over the eight launches of one call"}
    # end to end through the public API: fp32 inputs from pinned host memory, biases back to host
    zp, rpp = zt_h.pin_memory(), rp_h.pin_memory()
    outh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    e2e_ms = 0.0
    for i in range(args.steps + 2):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        zt.copy_(zp, non_blocking=True)
        rp.copy_(rpp, non_blocking=True)
        pair_cond.pair_biases(pw, zt, rp, out=out, workspace=wbuf, status=status)
        outh.copy_(out, non_blocking=True)
        e1.record()
        e1.synchronize()
        if i >= 2:
            e2e_ms += e0.elapsed_time(e1)
    e2e_ms = _max_over_ranks(e2e_ms, ws, device) / args.steps
    e2e = {"value": ws * cells / (e2e_ms * 1e-3), "unit": "pair-cells/s",
           "h2d_bytes_per_step": 2 * cells * 256 * 4, "d2h_bytes_per_step": out.numel() * 2,
           "ms_per_step": round(e2e_ms, 4)}
    cpu = None
    if ws == 1 and not args.no_cpu_baseline:
        from oracle import pair_cond_oracle as pco

        threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(threads)
        p = pco.pair_cond_params(head)
        n, t0 = 0, time.perf_counter()
        while True:
            pco.pair_biases_fp16(p, zt_h, rp_h)
            n += 1
            el = time.perf_counter() - t0
            if el >= min(args.cpu_seconds, 5.0):
                break
        cpu = {"value": n * cells / el, "unit": "pair-cells/s", "cores": threads, "kind": "port",
               "sample": f"{n} x pair_biases of one fold at L={L} in {el:.1f} s; oracle/pair_cond_oracle.py on "
                         "torch CPU (fp32 math, fp16 rounding points)"}
    if rank == 0:
        line = {"metric": "pair_cond_cells_per_s", "value": value, "unit": "pair-cells/s", "n_gpus": ws,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
                "config": {"workload": f"{args.workload}_pair_conditioning_L{L}", "B": B, "L": L, "c_trunk": 256,
                           "c_rel": 256, "c_pair": 256, "hidden": 512, "transitions": 2, "bias_heads": "12 x 16",
                           "l2": "flushed between steps (256 MiB write)", "parallelism": f"replicas x{ws}"},
                "e2e": e2e, "gpu_launches": 8 * args.steps, "roofline": roofline, "cpu_baseline": cpu,
                "clocks": clocks}
        print(json.dumps(line), flush=True)
    del g


def run_stage(args):
    """``--stage``: one kernel (or one whole update) at a chosen size, for profilers.  Every stage
    runs once untimed, then ``--reps`` more times; the device status word is checked and the mean
    CUDA-event time per launch is printed.  Select kernels in ncu with ``-k regex:`` and
    ``project_gate``, ``contract``, ``emit_residual``, ``transition`` (k4), ``disto`` (k5), ``ln_rows``
    / ``gemm_kernel`` (pc: the diffusion pair conditioning; parcae: the 6B loop's parcae step)."""
    from torch import nn

    from esmfold2_mlx_b200 import _lib, ops
    from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_mask, pair_tensor

    dev = torch.device("cuda", 0)
    _lib.check(_lib.load().tmu_device_check(), "tmu_device_check")
    L, B, cz = args.L, args.B, args.cz
    trunk = FoldingTrunk(1, cz, cz, hidden=args.hidden, seed=0, activation=args.activation)
    w = ops.TrimulWeights.from_module(getattr(trunk.blocks[0], "tri_mul_" + args.direction), dev)
    z = pair_tensor(B, L, cz, 0).half().to(dev)
    mask = pair_mask(B, L, args.mask_pad).half().to(dev) if args.mask_pad else None
    outgoing = args.direction == "out"
    status = ops.new_status(dev)
    a, b = ops.project_gate(z, mask, w, status)
    x = ops.contract(a, b, L, outgoing, status)
    out = ops.emit_residual(x, z, w, out=torch.empty_like(z), status=status)
    torch.cuda.synchronize()
    stages = {
        "k1": lambda: ops.project_gate(z, mask, w, status),
        "k2": lambda: ops.contract(a, b, L, outgoing, status),
        "k3": lambda: ops.emit_residual(x, z, w, out=out, status=status),
        "all": lambda: ops.trimul(z, mask, w, outgoing, out=out),
    }
    if args.stage == "k5":
        from esmfold2_mlx_b200.adaptive import ExpectedDistance

        ev = ExpectedDistance(nn.Linear(cz, 128), dev)
        stages["k5"] = lambda: ev(z)
    if args.stage == "k4":
        tw = ops.TransitionWeights.from_module(trunk.blocks[0].pair_transition, dev)
        stages["k4"] = lambda: ops.transition(z, tw, out=out, status=status)
    if args.stage == "pc":
        from esmfold2_mlx_b200 import pair_cond
        from esmfold2_mlx_b200.synthetic import DiffusionHead

        pw = pair_cond.PairCondWeights.from_head(DiffusionHead(), dev)
        zt = pair_tensor(B, L, 256, 1).to(dev) * 20.0
        rp = pair_tensor(B, L, 256, 2).to(dev)
        ws = torch.empty(pair_cond.workspace_bytes(B, L, pw.c_in, pw.c_pair, 2), dtype=torch.uint8, device=dev)
        pout = torch.empty(pw.n_bias // pw.heads, B, pw.heads, L, L, dtype=torch.float16, device=dev)
        stages["pc"] = lambda: pair_cond.pair_biases(pw, zt, rp, out=pout, workspace=ws, status=status)
    if args.stage == "parcae":
        from esmfold2_mlx_b200 import parcae

        m = nn.Module()
        m.parcae_input_norm = nn.LayerNorm(cz)
        pwt = parcae.ParcaeWeights.from_model(m, torch.full((cz,), 0.5), torch.randn(cz, cz) / 16, dev)
        zf = pair_tensor(B, L, cz, 3).to(dev)
        zi, rf = pair_tensor(B, L, cz, 4).to(dev), pair_tensor(B, L, cz, 5).to(dev)
        pws = torch.empty(_lib.load().tmu_parcae_workspace_bytes(B, L, cz), dtype=torch.uint8, device=dev)
        pout = torch.empty_like(zf)
        stages["parcae"] = lambda: parcae.parcae_step(zf, zi, rf, pwt, out=pout, workspace=pws, status=status)
    fn = stages[args.stage]
    fn()  # the stage's own output allocations happen here, outside the timed launches
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    code, site = ops.read_status(status)
    if code != 0:
        raise SystemExit(f"device status {code} at site {site:#x}")
    ms = e0.elapsed_time(e1) / max(1, args.reps)
    print(f"L={L} B={B} c_z={cz} {args.direction} stage={args.stage}: {ms * 1e3:.1f} us per launch")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-trunk", action="store_true", help="skip the trunk-recycle (config 3) measurement")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--sustain-seconds", type=float, default=0.6,
                    help="device seconds of the sustained replay that records clocks under load")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the timed step's output")
    ap.add_argument("--no-extra", action="store_true", help="skip the L2048, c2w and L2048w sub-measurements")
    ap.add_argument("--c5-nccl", action="store_true",
                    help="c5: move b with an NCCL all-gather instead of copy-engine peer copies")
    ap.add_argument("--c5-groups", type=int, default=4,
                    help="c5 channel partition: channel groups pipelined through the copy engines")
    ap.add_argument("--c5-partition", choices=["rows", "channels"], default="rows",
                    help="c5: contraction partition (rows: all-gather of b, the configuration's scheme; "
                         "channels: all-to-alls of a, b and x)")
    ap.add_argument("--workload", choices=WORKLOADS, default="c2",
                    help="c2 (default: the metric's configuration), c1, c4 (64 folds x L=146), L2048, "
                         "c5 (one L=3072 fold row-sharded over the N ranks), c2w / L2048w (c_z = c = 256), "
                         "pc / pc476 (diffusion pair conditioning of one fold, L = 238 / 476)")
    prof = ap.add_argument_group("profiling (--stage): one kernel at a chosen size, for ncu")
    prof.add_argument("--stage", choices=["all", "k1", "k2", "k3", "k4", "k5", "pc", "parcae"], default=None)
    prof.add_argument("--L", type=int, default=1024)
    prof.add_argument("--B", type=int, default=1)
    prof.add_argument("--direction", choices=["out", "in"], default="out")
    prof.add_argument("--reps", type=int, default=3)
    prof.add_argument("--mask-pad", type=int, default=0)
    prof.add_argument("--cz", type=int, choices=[128, 256], default=128, help="c_z = c")
    prof.add_argument("--hidden", type=int, default=512, help="transition hidden width (k4)")
    prof.add_argument("--activation", choices=["swiglu", "relu"], default="swiglu", help="transition activation (k4)")
    args = ap.parse_args()
    if args.stage is not None:
        run_stage(args)
        return
    ws, rank, local = _dist()
    if args.impl == "reference":
        run_reference(args, ws, rank, local)
        return
    _init_pg(ws, local, "nccl")
    try:
        if args.workload in SHARDED_WORKLOADS:
            run_sharded(args, ws, rank, local)
        elif args.workload in PAIR_COND_L:
            run_pair_cond(args, ws, rank, local)
        else:
            run_b200(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
