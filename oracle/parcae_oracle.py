"""CPU oracle for the parcae step of the 6B recycling loop (TEST INFRASTRUCTURE ONLY).

Restates ``_step``'s recurrence (abhi0raj/esmfold2-mlx ``src/esmfold2_mlx/var_6b_mlx_loop.py:67-71``,
fp32 MLX in the reference):  z' = a * z + LN(z_init + refined; parcae_input_norm, eps 1e-5) @ B^T,
with ``bT = b_mat.T`` (``:169``).  ``dtype`` float32 follows the reference's arithmetic; float64
is the exact value both are measured against.  Parity pin: ``tests/golden/conditioning_golden.npz``
(``tests/golden/make_golden_conditioning.py`` runs the reference's ``_step`` unmodified over a
numpy stand-in for MLX, with identity lm_encoder and trunk), checked by
``tests/test_oracle_golden_conditioning.py`` to a few fp32 ulps; the reference's own tests need the
6B checkpoint, esm and MLX, all absent.
"""

from __future__ import annotations

import torch


def parcae_step(z, z_init, refined, ln_w, ln_b, a, b_mat, dtype=torch.float32) -> torch.Tensor:
    u = (z_init.to(dtype) + refined.to(dtype))
    mean = u.mean(-1, keepdim=True)
    d = u - mean
    var = (d * d).mean(-1, keepdim=True)
    inj = d * torch.rsqrt(var + 1e-5) * ln_w.to(dtype) + ln_b.to(dtype)
    return torch.as_tensor(a).to(dtype) * z.to(dtype) + inj @ b_mat.to(dtype).T
