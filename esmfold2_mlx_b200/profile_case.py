"""Run one triangle update (or one of its kernels) at a chosen size, for profilers.

    python -m esmfold2_mlx_b200.profile_case --L 1024 [--B 1] [--direction out|in]
           [--stage all|k1|k2|k3|k4|k5] [--reps 3] [--mask-pad 0] [--cz 128|256]
           [--hidden 512] [--activation swiglu|relu]

Inputs are seeded synthetic tensors (``synthetic``); weights are random-init.  The chosen stage
is launched ``--reps`` times after one untimed launch of every stage (and one more of itself), then the script checks the
device status word and prints the mean CUDA-event time per launch.  Use ``ncu -k regex:<name>``
with ``project_gate``, ``contract``, ``emit_residual`` or ``transition`` to select a kernel
(k4 is the fused pair transition; k5 the distogram expected distance, ``disto``; pc the diffusion
pair conditioning, ``ln_gemm`` and ``transition``).
"""

from __future__ import annotations

import argparse

import torch

from . import _lib, ops
from .synthetic import FoldingTrunk, pair_mask, pair_tensor


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--L", type=int, default=1024)
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--direction", choices=["out", "in"], default="out")
    ap.add_argument("--stage", choices=["all", "k1", "k2", "k3", "k4", "k5", "pc", "parcae"], default="all",
                    help="pc: the diffusion pair conditioning (tmu_pair_cond); parcae: the 6B loop's parcae step")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--mask-pad", type=int, default=0)
    ap.add_argument("--cz", type=int, choices=[128, 256], default=128, help="c_z = c")
    ap.add_argument("--hidden", type=int, default=512, help="transition hidden width (k4)")
    ap.add_argument("--activation", choices=["swiglu", "relu"], default="swiglu", help="transition activation (k4)")
    args = ap.parse_args()

    dev = torch.device("cuda", 0)
    _lib.check(_lib.load().tmu_device_check(), "tmu_device_check")
    L, B = args.L, args.B
    trunk = FoldingTrunk(1, args.cz, args.cz, hidden=args.hidden, seed=0, activation=args.activation)
    w = ops.TrimulWeights.from_module(getattr(trunk.blocks[0], "tri_mul_" + args.direction), dev)
    z = pair_tensor(B, L, args.cz, 0).half().to(dev)
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
        from torch import nn

        from .adaptive import DistoHead, expected_distance
        head = DistoHead(nn.Linear(args.cz, 128), dev)
        stages["k5"] = lambda: expected_distance(z, head)
    if args.stage == "k4":
        tw = ops.TransitionWeights.from_module(trunk.blocks[0].pair_transition, dev)
        stages["k4"] = lambda: ops.transition(z, tw, out=out, status=status)
    if args.stage == "pc":
        from . import pair_cond
        from .synthetic import DiffusionHead
        pw = pair_cond.PairCondWeights.from_head(DiffusionHead(), dev)
        zt = pair_tensor(B, L, 256, 1).to(dev) * 20.0
        rp = pair_tensor(B, L, 256, 2).to(dev)
        ws = torch.empty(pair_cond.workspace_bytes(B, L, pw.c_in, pw.c_pair, 2), dtype=torch.uint8, device=dev)
        pout = torch.empty(pw.n_bias // pw.heads, B, pw.heads, L, L, dtype=torch.float16, device=dev)
        stages["pc"] = lambda: pair_cond.pair_biases(pw, zt, rp, out=pout, workspace=ws, status=status)
    if args.stage == "parcae":
        from torch import nn

        from . import parcae
        m = nn.Module()
        m.parcae_input_norm = nn.LayerNorm(args.cz)
        pwt = parcae.ParcaeWeights.from_model(m, torch.full((args.cz,), 0.5), torch.randn(args.cz, args.cz) / 16, dev)
        zf = pair_tensor(B, L, args.cz, 3).to(dev)
        zi, rf = pair_tensor(B, L, args.cz, 4).to(dev), pair_tensor(B, L, args.cz, 5).to(dev)
        pws = torch.empty(_lib.load().tmu_parcae_workspace_bytes(B, L, args.cz), dtype=torch.uint8, device=dev)
        pout = torch.empty_like(zf)
        stages["parcae"] = lambda: parcae.parcae_step(zf, zi, rf, pwt, out=pout, workspace=pws, status=status)
    fn = stages[args.stage]
    fn()  # warm-up: the stage's own output allocations happen here, outside the timed launches
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
    print(f"L={L} B={B} c_z={args.cz} {args.direction} stage={args.stage}: {ms * 1e3:.1f} us per launch")


if __name__ == "__main__":
    main()
