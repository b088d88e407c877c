"""Variant: the fp16 folding trunk on B200 with the sm_100a triangle-update kernels.

Same weights, fp16 scheme and 1/256 contraction pre-scale as the reference's ``mlx_trunk16k``
(``src/esmfold2_mlx/var_mlx_trunk16k.py:16-19``); ``model.folding_trunk`` becomes a
:class:`~esmfold2_mlx_b200.trunk.CUDAFoldingTrunk`.
"""

import torch

from .trunk import CUDAFoldingTrunk

DEVICE = "cuda"  # where the weights live when apply() is given no device (the current CUDA device)


def apply(model, device=None):
    model.folding_trunk = CUDAFoldingTrunk(model.folding_trunk, dtype=torch.float16,
                                           device=DEVICE if device is None else device)
