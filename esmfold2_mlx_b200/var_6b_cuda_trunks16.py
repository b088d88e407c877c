"""Variant (6B release model): every folding-trunk stack on B200 in fp16.

The release model has four trunk stacks: the main trunk (24 blocks), ``lm_encoder`` (4), the
parcae coda (2) and the confidence head's trunk (4) (``src/esmfold2_mlx/var_6b_mlx_trunks16k.py:19-32``).
Each becomes a :class:`~esmfold2_mlx_b200.trunk.CUDAFoldingTrunk` with the same weights.
"""

import torch

from .trunk import CUDAFoldingTrunk

DEVICE = "cuda"  # where the weights live when apply() is given no device (the current CUDA device)


def _wrap(trunk, device):
    if not isinstance(trunk, CUDAFoldingTrunk):
        trunk = CUDAFoldingTrunk(trunk, dtype=torch.float16, device=device)
    return trunk


def apply(model, device=None):
    device = DEVICE if device is None else device
    model.folding_trunk = _wrap(model.folding_trunk, device)
    if getattr(model, "lm_encoder", None) is not None:
        model.lm_encoder = _wrap(model.lm_encoder, device)
    model.parcae_coda = _wrap(model.parcae_coda, device)
    model.confidence_head.folding_trunk = _wrap(model.confidence_head.folding_trunk, device)
