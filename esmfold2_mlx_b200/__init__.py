"""B200 (sm_100a) triangle multiplicative update for ESMFold2's folding trunk.

A drop-in for the hot path of abhi0raj/esmfold2-mlx: ``apply_variants(model, "cuda_trunk16")``
swaps ``model.folding_trunk`` for :class:`CUDAFoldingTrunk`, whose triangle updates run as three
hand-written sm_100a kernels behind the C ABI in ``include/tmu.h`` (``lib/libtmu.so``).

Importing the package is cheap; the CUDA library loads on first use and raises if it is not built.
"""

__version__ = "0.1.0"

__all__ = ["CUDAFoldingTrunk", "apply_variants", "__version__"]


def __getattr__(name):
    if name == "CUDAFoldingTrunk":
        from .trunk import CUDAFoldingTrunk

        return CUDAFoldingTrunk
    if name == "apply_variants":
        from .variants import apply_variants

        return apply_variants
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
