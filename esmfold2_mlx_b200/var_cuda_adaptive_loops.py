"""Variant: adaptive recycling (``var_adaptive_loops.py``) with the convergence check on B200.

Apply after the trunk swap, e.g. ``apply_variants(model, "cuda_trunk16,cuda_adaptive_loops")``:
it wraps ``model.folding_trunk`` and stops running passes once the distogram's expected
distances stop moving (p95 of the change < 0.6 Å), computing them with the fused kernel K5.
"""

from .adaptive import apply  # noqa: F401
