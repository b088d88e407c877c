"""Numpy stand-in for the parts of MLX 0.32.3 the reference trunk calls (fixture generation only).

MLX is not installed in this image and cannot be.  ``tests/golden/make_golden*.py`` put this
directory on ``sys.path`` so the reference's unmodified ``mlx_trunk.py``, ``mlx_trunk_kernels.py``,
``mlx_diffusion16.py`` and ``var_6b_mlx_loop.py`` import it as ``mlx.core`` and run on the CPU.
Nothing else uses it.
"""
