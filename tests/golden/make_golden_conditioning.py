"""Generate ``conditioning_golden.npz`` by running two more of the reference's functions on the CPU.

Run in a container that has the reference checkout (read-only is fine)::

    python tests/golden/make_golden_conditioning.py --reference /path/to/esmfold2-mlx

Like ``make_golden.py`` it puts ``tests/golden/mlx_standin`` on ``sys.path`` as ``mlx.core`` and
imports the reference's modules unmodified from ``<reference>/src``:

* ``esmfold2_mlx.mlx_diffusion16.pair_biases`` (``mlx_diffusion16.py:81-87``): the diffusion
  head's per-fold pair conditioning in the fp16 ``pair16`` precision.  Its weights come from the
  reference's own copy helpers ``_ln`` / ``_lin`` / ``_transition_layer``
  (``mlx_diffusion.py:39-52``) applied to a seeded ``esmfold2_mlx_b200.synthetic.DiffusionHead``;
  the two statements that fold the token blocks' pair biases into one matrix
  (``mlx_diffusion.py:85-86``) and the ``pair16`` casts (``mlx_diffusion16.py:224-227``, through
  the reference's ``_cast``) sit inside larger functions that need the full Biohub module tree,
  so this script repeats those few lines.  ``mlx_diffusion.py`` imports two constants from
  Biohub's ``esm`` package (absent here); a module holding placeholder values is registered
  under that name before the import, and ``pair_biases`` does not read them.
  A second head (``pc2``) has widths the CUDA kernels take, for the GPU test against these
  outputs.
* ``esmfold2_mlx.var_6b_mlx_loop._step`` (``var_6b_mlx_loop.py:67-71``): the parcae recurrence
  ``z' = a * z + LN(z_init + refined) @ B^T`` in fp32, with an lm_encoder that returns its input
  (``refined`` is passed as ``lz``) and a folding trunk that returns its input, so the stored
  output is the recurrence alone.

The GPU never runs this and the test suite only reads the ``.npz``.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

# pair conditioning: c_trunk = c_rel = c_pair = 64, transition width 128, 3 token blocks x 4 heads
PC = dict(c_trunk=64, c_rel=64, c_pair=64, hidden=128, n_transitions=2, n_blocks=3, heads=4, seed=21)
PC_CASES = ((1, 12, 31), (2, 7, 32))  # (B, L, input seed)
# a second head at widths the CUDA kernels take (c_trunk + c_rel = 256, c_pair = 128, 32 bias
# channels), so the GPU path can be compared with the reference's outputs directly; its inputs
# hold fp16-representable values and are stored as fp16 (exact) to keep the file small
PC2 = dict(c_trunk=128, c_rel=128, c_pair=128, hidden=256, n_transitions=1, n_blocks=4, heads=8, seed=23)
PC2_CASES = ((1, 64, 33),)
PARCAE_C, PARCAE_CASES = 64, ((1, 9, 41), (2, 5, 42))
PARCAE_WIDE_CASES = ((128, 1, 20, 43),)  # (c, B, L, seed): a width tmu_parcae_step takes


def _register_esm_constants():
    """``mlx_diffusion.py:28`` imports ``CHAR_VOCAB_SIZE, MAX_CHARS`` from Biohub's ``esm``."""
    names = ["esm", "esm.models", "esm.models.esmfold2", "esm.models.esmfold2.layers"]
    for n in names:
        sys.modules.setdefault(n, types.ModuleType(n))
    layers = sys.modules["esm.models.esmfold2.layers"]
    layers.CHAR_VOCAB_SIZE = getattr(layers, "CHAR_VOCAB_SIZE", 0)
    layers.MAX_CHARS = getattr(layers, "MAX_CHARS", 0)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of abhi0raj/esmfold2-mlx")
    ap.add_argument("--out", default=os.path.join(HERE, "conditioning_golden.npz"))
    args = ap.parse_args()

    sys.path.insert(0, os.path.join(HERE, "mlx_standin"))
    sys.path.insert(0, os.path.join(args.reference, "src"))
    sys.path.insert(0, REPO)
    _register_esm_constants()
    import mlx.core as mx  # the stand-in
    from esmfold2_mlx import mlx_diffusion as base  # reference code, unmodified
    from esmfold2_mlx import mlx_diffusion16 as m16  # reference code, unmodified
    from esmfold2_mlx import var_6b_mlx_loop as loop  # reference code, unmodified

    from esmfold2_mlx_b200.synthetic import DiffusionHead

    out = {"meta": np.frombuffer(repr({"pc": PC, "pc2": PC2, "parcae_c": PARCAE_C}).encode(), dtype=np.uint8)}

    # ---------------- pair conditioning ----------------
    for name, cfg, cases in (("pc", PC, PC_CASES), ("pc2", PC2, PC2_CASES)):
        head = DiffusionHead(**cfg)
        for k, v in head.state_dict().items():
            out[f"{name}_w/" + k] = v.detach().numpy().astype(np.float32)
        cond, blocks = head.diffusion_module.conditioning, head.diffusion_module.token_transformer.attn_blocks
        with torch.no_grad():  # mlx_diffusion.py:85-86
            bias_w = torch.cat([b.pair_norm.weight[:, None] * b.pair_bias_proj.weight.T for b in blocks], -1)
            bias_b = torch.cat([b.pair_bias_proj(b.pair_norm.bias) for b in blocks], -1)
        pp = {"ln": base._ln(cond.z_input_norm), "proj": base._lin(cond.z_proj),
              "transitions": [base._transition_layer(b) for b in cond.z_transitions],
              "bias_w": base._mx(bias_w), "bias_b": base._mx(bias_b)}
        # pair16 (mlx_diffusion16.py:225-227)
        pp["proj"], pp["bias_w"], pp["bias_b"] = (pp[k].astype(m16.F16) for k in ("proj", "bias_w", "bias_b"))
        pp["transitions"] = [m16._cast(b, m16.F16, ("a", "b", "out")) for b in pp["transitions"]]
        for B, L, seed in cases:
            g = torch.Generator().manual_seed(seed)
            zt = 4.0 * torch.randn(B, L, L, cfg["c_trunk"], generator=g)
            rp = torch.randn(B, L, L, cfg["c_rel"], generator=g)
            tag = f"B{B}L{L}"
            if name == "pc2":
                zt, rp = zt.half().float(), rp.half().float()
                out[f"{name}/{tag}/z_trunk"], out[f"{name}/{tag}/rel_pos"] = zt.half().numpy(), rp.half().numpy()
            else:
                out[f"{name}/{tag}/z_trunk"], out[f"{name}/{tag}/rel_pos"] = zt.numpy(), rp.numpy()
            bias = m16.pair_biases(pp, mx.array(zt.numpy()), mx.array(rp.numpy()), cfg["heads"], m16.F16)
            out[f"{name}/{tag}/bias"] = np.asarray(bias)

    # ---------------- parcae step ----------------
    ident_lm = lambda params, lz, mask: lz  # noqa: E731
    ident_trunk = lambda params, z, mask: z  # noqa: E731
    for c, B, L, seed in [(PARCAE_C, *case) for case in PARCAE_CASES] + list(PARCAE_WIDE_CASES):
        g = torch.Generator().manual_seed(seed)
        t = {"z": torch.randn(B, L, L, c, generator=g), "z_init": torch.randn(B, L, L, c, generator=g),
             "refined": 3.0 * torch.randn(B, L, L, c, generator=g),
             "ln_w": 1.0 + 0.1 * torch.randn(c, generator=g), "ln_b": 0.1 * torch.randn(c, generator=g),
             "a": torch.rand(c, generator=g), "b_mat": torch.randn(c, c, generator=g) / c**0.5}
        tag = f"B{B}L{L}" if c == PARCAE_C else f"B{B}L{L}c{c}"
        for k, v in t.items():
            out[f"parcae/{tag}/{k}"] = v.numpy()
        m = {k: mx.array(v.numpy()) for k, v in t.items()}
        zn = loop._step(ident_lm, ident_trunk, None, None, m["ln_w"], m["ln_b"], m["a"], m["b_mat"].T,
                        m["refined"], m["z"], m["z_init"], None)
        out[f"parcae/{tag}/z_next"] = np.asarray(zn)

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, {os.path.getsize(args.out) / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
