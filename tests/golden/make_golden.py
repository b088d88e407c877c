"""Generate ``trimul_golden.npz`` by running the reference's own trunk code on the CPU.

Run in a container that has the reference checkout (read-only is fine)::

    python tests/golden/make_golden.py --reference /path/to/esmfold2-mlx

It imports ``esmfold2_mlx.mlx_trunk`` and ``esmfold2_mlx.mlx_trunk_kernels`` unmodified from
``<reference>/src`` with ``tests/golden/mlx_standin`` providing ``mlx.core`` (MLX 0.32.3 is
not installable here; the stand-in restates the primitives the trunk calls).  The reference's
``trunk_params`` extracts the weights from a seeded trunk-shaped module tree
(``esmfold2_mlx_b200.synthetic.FoldingTrunk``); its ``_trimul``/``block_forward``/
``make_trunk`` then produce the outputs stored here.  The GPU never runs this and the test
suite only reads the ``.npz``.

Stored cases (c_z = c = 128, one PairUpdateBlock, transition hidden 128):
  * ``tm_{out,in}_{nomask,mask}``: ``mlx_trunk_kernels._trimul`` (fused fp16 path) on z of
    shape [B, L, L, 128] for (B, L) = (1, 20) and (2, 13); outputs z' and n'.
  * ``trunk16_{nomask,mask}``: ``mlx_trunk_kernels.make_trunk(float16)`` (default stack path).
  * ``trunk16_unfused_mask``: ``make_trunk(float16, use=())`` (plain MLX ops, no Metal kernels).
  * ``trunk32_mask``: ``mlx_trunk.make_trunk(float32)`` (the exact fp32 trunk).

``--c-z 256`` writes ``trimul_golden_cz256.npz`` instead: the same cases at c_z = c = 256 (the
released trunk's width, ``mlx_trunk.py:4``) for (B, L) = (1, 12) and (2, 7), the trunk cases on
the first.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

SEED_WEIGHTS = 11
C_Z = C = 128
HIDDEN = 128


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of abhi0raj/esmfold2-mlx")
    ap.add_argument("--out", default=None)
    ap.add_argument("--c-z", type=int, default=C_Z, choices=(128, 256))
    args = ap.parse_args()
    c_z = c = args.c_z
    cases = ((1, 20), (2, 13)) if c_z == 128 else ((1, 12), (2, 7))
    if args.out is None:
        args.out = os.path.join(HERE, "trimul_golden.npz" if c_z == 128 else f"trimul_golden_cz{c_z}.npz")

    sys.path.insert(0, os.path.join(HERE, "mlx_standin"))
    sys.path.insert(0, os.path.join(args.reference, "src"))
    sys.path.insert(0, REPO)
    import mlx.core as mx  # the stand-in
    from esmfold2_mlx import mlx_trunk as mt  # reference code, unmodified
    from esmfold2_mlx import mlx_trunk_kernels as mk  # reference code, unmodified

    from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_mask

    trunk = FoldingTrunk(1, c_z, c, hidden=HIDDEN, seed=SEED_WEIGHTS, ln_noise=0.1)
    out = {}
    sd = {k: v.detach().numpy().astype(np.float32) for k, v in trunk.state_dict().items()}
    for k, v in sd.items():
        out["w/" + k] = v.astype(np.float16) if v.ndim == 2 else v  # 2-D weights fit fp16 storage
    # the module tree is rebuilt from the stored weights (fp16 storage of Linear weights)
    with torch.no_grad():
        for k, v in trunk.state_dict().items():
            v.copy_(torch.from_numpy(out["w/" + k].astype(np.float32)))

    p16 = mt.trunk_params(trunk, mx.float16)
    p32 = mt.trunk_params(trunk, mx.float32)
    mix_eps16 = mt.EPS / mt.CONTRACT_SCALE**2

    for (B, L) in cases:
        g = torch.Generator().manual_seed(1000 + L)
        z = torch.randn(B, L, L, c_z, generator=g).to(torch.float16)
        msk = pair_mask(B, L, n_pad=3).to(torch.float16)
        tag = f"B{B}L{L}"
        out[f"z/{tag}"] = z.numpy()
        out[f"mask/{tag}"] = msk.numpy()
        zm = mx.array(z.float().numpy()).astype(mx.float16)
        mm = mx.array(msk.float().numpy()).astype(mx.float16)
        blk = p16[0]
        for direction, outgoing in (("out", True), ("in", False)):
            pt = blk[direction]
            for mname, mask in (("nomask", None), ("mask", mm)):
                n = mx.fast.layer_norm(zm, pt["ln_in_w"], pt["ln_in_b"], mt.EPS)
                nxt = (blk["in"]["ln_in_w"], blk["in"]["ln_in_b"]) if outgoing else (blk["ln_w"], blk["ln_b"])
                z2, n2 = mk._trimul(pt, zm, n, mask, outgoing, mix_eps16, nxt, mk.ALL)
                out[f"tm_{direction}_{mname}/{tag}/z"] = np.asarray(z2).astype(np.float16)
                out[f"tm_{direction}_{mname}/{tag}/n_next"] = np.asarray(n2).astype(np.float16)
        if (B, L) == cases[0]:
            for mname, mask in (("nomask", None), ("mask", mm)):
                r = mk.make_trunk(mx.float16)(p16, mx.array(z.float().numpy()), mask)
                out[f"trunk16_{mname}/{tag}"] = np.asarray(r).astype(np.float32)
            r = mk.make_trunk(mx.float16, use=())(p16, mx.array(z.float().numpy()), mm)
            out[f"trunk16_unfused_mask/{tag}"] = np.asarray(r).astype(np.float32)
            r = mt.make_trunk(mx.float32)(p32, mx.array(z.float().numpy()), mx.array(msk.float().numpy()))
            out[f"trunk32_mask/{tag}"] = np.asarray(r).astype(np.float32)

    meta = {"seed_weights": SEED_WEIGHTS, "c_z": c_z, "c": c, "hidden": HIDDEN, "ln_noise": 0.1,
            "mix_eps16": mix_eps16}
    out["meta"] = np.frombuffer(repr(meta).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, {os.path.getsize(args.out) / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
