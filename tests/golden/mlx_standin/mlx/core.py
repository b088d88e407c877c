"""``mlx.core`` restated over numpy, for running the reference trunk on the CPU (fixtures only).

Only what ``src/esmfold2_mlx/mlx_trunk.py``, ``mlx_trunk_kernels.py``, ``mlx_diffusion16.pair_biases``
and ``var_6b_mlx_loop._step`` call is provided.
Semantics follow MLX 0.32.3's documented behaviour for these primitives:

* arrays carry a dtype (float16 or float32); an op on float16 and float32 arrays returns float32,
  an op of an array with a Python scalar returns the array's dtype;
* fp16 element-wise ops (``+ - *``, ``sigmoid``) compute in fp32 and round once to fp16;
* ``matmul`` / ``addmm`` accumulate in fp32 and round once to the output dtype;
* ``fast.layer_norm`` computes fp32 statistics (mean, then centred variance) and rounds once;
  a ``None`` weight or bias means no scale or no shift;
* ``compile`` returns the function unchanged (it does not alter arithmetic), ``eval`` is a no-op.

``fast.metal_kernel`` returns an evaluator keyed by the kernel's ``name`` that restates the three
Metal kernels of ``mlx_trunk_kernels.py`` (fp32 arithmetic, one rounding per output):
``trunk_gate_cf`` (``:47-80``), ``trunk_ln_cf_to_cl`` (``:107-147``), ``trunk_resgate_ln``
(``:165-190``).  The Metal source strings themselves are not executed.
"""

from __future__ import annotations

import types

import numpy as np

float16 = np.dtype(np.float16)
float32 = np.dtype(np.float32)


def _np(x):
    return x._a if isinstance(x, array) else np.asarray(x)


def _dtype_of(*xs):
    dts = [x.dtype for x in xs if isinstance(x, array)]
    if not dts or float32 in dts:
        return float32
    return float16


class array:
    __array_priority__ = 100

    def __init__(self, a, dtype=None):
        a = _np(a)
        if dtype is None:
            dtype = a.dtype if a.dtype in (np.float16, np.float32) else float32
        self._a = np.asarray(a).astype(dtype)

    # -- metadata ---------------------------------------------------------------------
    @property
    def dtype(self):
        return self._a.dtype

    @property
    def shape(self):
        return tuple(self._a.shape)

    @property
    def size(self):
        return int(self._a.size)

    @property
    def ndim(self):
        return self._a.ndim

    def item(self):
        return self._a.item()

    def __array__(self, dtype=None, copy=None):
        return self._a if dtype is None else self._a.astype(dtype)

    # -- conversion / layout -------------------------------------------------------------
    def astype(self, dtype):
        return array(self._a.astype(np.float32).astype(dtype), dtype)

    def transpose(self, *axes):
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            axes = tuple(axes[0])
        return array(np.transpose(self._a, axes if axes else None), self.dtype)

    def swapaxes(self, a, b):
        return array(np.swapaxes(self._a, a, b), self.dtype)

    def reshape(self, *shape):
        return array(self._a.reshape(*shape), self.dtype)

    def __getitem__(self, idx):
        return array(self._a[idx], self.dtype)

    @property
    def T(self):
        return array(self._a.T, self.dtype)

    # -- arithmetic ----------------------------------------------------------------------
    def _bin(self, other, fn):
        dt = _dtype_of(self, other)
        r = fn(_np(self).astype(np.float32), _np(other).astype(np.float32))
        return array(r.astype(dt), dt)

    def __add__(self, o):
        return self._bin(o, np.add)

    __radd__ = __add__

    def __sub__(self, o):
        return self._bin(o, np.subtract)

    def __rsub__(self, o):
        return array(o)._bin(self, np.subtract)

    def __mul__(self, o):
        return self._bin(o, np.multiply)

    __rmul__ = __mul__

    def __truediv__(self, o):
        return self._bin(o, np.divide)

    def __neg__(self):
        return array(-self._a, self.dtype)

    def __matmul__(self, o):
        return matmul(self, o)

    def __abs__(self):
        return array(np.abs(self._a), self.dtype)


def matmul(a, b):
    dt = _dtype_of(a, b)
    r = np.matmul(_np(a).astype(np.float32), _np(b).astype(np.float32))
    return array(r.astype(dt), dt)


def addmm(c, a, b, alpha=1.0, beta=1.0):
    dt = _dtype_of(c, a, b)
    r = alpha * np.matmul(_np(a).astype(np.float32), _np(b).astype(np.float32)) + beta * _np(c).astype(np.float32)
    return array(r.astype(dt), dt)


def _sig32(x):
    return (1.0 / (1.0 + np.exp(-x.astype(np.float32)))).astype(np.float32)


def sigmoid(x):
    return array(_sig32(_np(x)).astype(x.dtype), x.dtype)


def split(x, n, axis=-1):
    return [array(p, x.dtype) for p in np.split(_np(x), n, axis=axis)]


def concatenate(xs, axis=0):
    dt = _dtype_of(*xs)
    return array(np.concatenate([_np(x).astype(dt) for x in xs], axis=axis), dt)


def linspace(start, stop, num=50, dtype=float32):
    return array(np.linspace(start, stop, num, dtype=np.float64).astype(np.float32).astype(dtype), dtype)


def zeros(shape, dtype=float32):
    return array(np.zeros(shape, dtype), dtype)


def eval(*args, **kw):  # noqa: A001 - mirrors mx.eval
    return None


def compile(fn, *a, **kw):  # noqa: A001 - mirrors mx.compile
    return fn


def _ln32(x, w, b, eps):
    x = x.astype(np.float32)
    mean = x.mean(-1, keepdims=True, dtype=np.float32)
    v = x - mean
    var = (v * v).mean(-1, keepdims=True, dtype=np.float32)
    inv = (1.0 / np.sqrt(var + np.float32(eps))).astype(np.float32)
    y = v * inv
    if w is not None:
        y = y * w.astype(np.float32)
    if b is not None:
        y = y + b.astype(np.float32)
    return y


def _layer_norm(x, w, b, eps):
    w = None if w is None else _np(w)
    b = None if b is None else _np(b)
    return array(_ln32(_np(x), w, b, eps).astype(x.dtype), x.dtype)


# --------------------------------------------------------------------------------------
# fast.metal_kernel: restated kernels of mlx_trunk_kernels.py
# --------------------------------------------------------------------------------------


def _kernel_gate_cf(inputs, tmpl, output_shapes, output_dtypes):
    proj, mask = (_np(t) for t in inputs)
    C = tmpl["C"]
    B, c, L, _ = output_shapes[0]
    p = proj.astype(np.float32).reshape(B, L * L, 4 * C)
    outs = []
    for lo in (0, C):
        s, g = p[..., lo:lo + C], p[..., 2 * C + lo:3 * C + lo]
        v = s / (1.0 + np.exp(-g))
        if tmpl["HAS_MASK"]:
            v = v * mask.astype(np.float32).reshape(B, L * L, 1)
        outs.append(array(v.transpose(0, 2, 1).reshape(B, C, L, L).astype(output_dtypes[0]), output_dtypes[0]))
    return outs


def _kernel_ln_cf_to_cl(inputs, tmpl, output_shapes, output_dtypes):
    x, w, b, eps = (_np(t) for t in inputs)
    xt = np.transpose(x.astype(np.float32), (0, 2, 3, 1))
    y = _ln32(xt, w, b, float(eps.reshape(-1)[0]))
    return [array(y.astype(output_dtypes[0]), output_dtypes[0])]


def _kernel_resgate_ln(inputs, tmpl, output_shapes, output_dtypes):
    z, m, g, w, b, eps = (_np(t) for t in inputs)
    dt = output_dtypes[0]
    zn = (z.astype(np.float32) + m.astype(np.float32) / (1.0 + np.exp(-g.astype(np.float32)))).astype(dt)
    n = _ln32(zn.astype(np.float32), w, b, float(eps.reshape(-1)[0]))
    return [array(zn, dt), array(n.astype(dt), dt)]


_KERNELS = {
    "trunk_gate_cf": _kernel_gate_cf,
    "trunk_ln_cf_to_cl": _kernel_ln_cf_to_cl,
    "trunk_resgate_ln": _kernel_resgate_ln,
}


def _metal_kernel(name, input_names, output_names, source, header="", **kw):
    impl = _KERNELS[name]

    def run(inputs, template, grid, threadgroup, output_shapes, output_dtypes, **kw2):
        tmpl = {k: v for k, v in template}
        return impl(inputs, tmpl, output_shapes, [np.dtype(d) for d in output_dtypes])

    return run


fast = types.SimpleNamespace(layer_norm=_layer_norm, metal_kernel=_metal_kernel)
