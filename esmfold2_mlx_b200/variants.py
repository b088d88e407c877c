"""Swap registry: ``apply_variants(model, names)`` imports ``esmfold2_mlx_b200.var_<name>`` and
calls its ``apply(model)``, in order (``src/esmfold2_mlx/variants.py:74-86``).

The B200 variants are ``cuda_trunk16`` (the experimental checkpoints' folding trunk) and
``6b_cuda_trunks16`` (all four trunk stacks of the 6B release model).  A maintainer who wants
the reference's own registry to find them adds thin ``var_cuda_trunk16.py`` /
``var_6b_cuda_trunks16.py`` modules there whose ``apply`` forwards to these.
"""

from __future__ import annotations

import importlib

DEFAULT_STACK = "cuda_trunk16"
DEFAULT_STACK_6B = "6b_cuda_trunks16"


def apply_variants(model, names):
    if isinstance(names, str):
        names = names.split(",")
    for name in [n for n in names if n]:
        try:
            module = importlib.import_module(f"{__package__}.var_{name}")
        except ModuleNotFoundError as e:
            if e.name != f"{__package__}.var_{name}":
                raise
            raise ValueError(f"unknown speed variant {name!r}") from None
        module.apply(model)
    return model
