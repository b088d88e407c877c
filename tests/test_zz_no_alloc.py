"""The no-allocation entry point (tmu_trimul_noalloc) against the workspace one (tmu_trimul).

Some callers cannot allocate device memory when they run the update (a host framework that owns
all device memory, or code that must not trigger cudaMalloc's device-wide synchronisation).
tmu_trimul_noalloc serves them from a fixed scratch array inside the library.  This file checks,
through the C ABI, that two calls in a row -- different shapes, directions and masks, so the
second call reuses scratch the first one left behind -- give the same fp16 output as tmu_trimul
on the same inputs, within the parity tests' tolerance (4 fp16 ulps at the tensor's scale; the
kernels are the same, so equality is expected), and that sizes beyond the cap are refused.
At the released model's width (c_z = c = 256) the cap allows one fold up to L = 128, and the
wide kernels cannot write over their input, so an in-place call is refused.
It is collected last so that a failure here does not stop the rest of the suite.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from esmfold2_mlx_b200 import _lib, ops
from esmfold2_mlx_b200.synthetic import FoldingTrunk, pair_mask, pair_tensor

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ulp16(x: float) -> float:
    return 2.0 ** (math.floor(math.log2(max(abs(x), 2.0**-14))) - 10)


def _noalloc(lib, z, out, mask, w, outgoing, status):
    B, L = z.shape[0], z.shape[1]
    return lib.tmu_trimul_noalloc(ops._ptr(z), ops._ptr(out), ops._ptr(mask), ctypes.byref(w.struct), B, L, w.c_z,
                                  w.c, 1 if outgoing else 0, ops.MIX_EPS_FP16, ops._ptr(status),
                                  ops._stream_ptr(z.device))


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    lib = _lib.load()
    trunk = FoldingTrunk(1, 128, 128, hidden=256, seed=21, ln_noise=0.1)
    w_out = ops.TrimulWeights.from_module(trunk.blocks[0].tri_mul_out, DEV)
    w_in = ops.TrimulWeights.from_module(trunk.blocks[0].tri_mul_in, DEV)
    cases = [  # (L, B, n_pad, weights, outgoing)
        (150, 1, 12, w_out, True),
        (97, 2, 0, w_in, False),
    ]
    status = ops.new_status(DEV)
    for k, (L, B, n_pad, w, outgoing) in enumerate(cases):
        z = pair_tensor(B, L, 128, 40 + k).half().to(DEV)
        mask = pair_mask(B, L, n_pad).half().to(DEV) if n_pad else None
        ref = ops.trimul(z, mask, w, outgoing)  # tmu_trimul with a workspace
        out = torch.full_like(z, float("nan"))
        rc = _noalloc(lib, z, out, mask, w, outgoing, status)
        assert rc == 0, (_lib.STATUS_NAMES.get(rc), lib.tmu_last_error())
        code, site = ops.read_status(status)
        assert code == 0, f"device status {code} at {site:#x}"
        got, want = out.float().cpu(), ref.float().cpu()
        assert torch.isfinite(got).all()
        diff = float((got - want).abs().max())
        assert diff <= 4 * _ulp16(float(want.abs().max())), f"call {k}: max diff {diff}"


def test_noalloc_refuses_sizes_beyond_its_scratch():
    lib = _lib.load()
    trunk = FoldingTrunk(1, 128, 128, hidden=256, seed=22)
    w = ops.TrimulWeights.from_module(trunk.blocks[0].tri_mul_out, DEV)
    L = 179  # 128 * 179 * 184 * 2 bytes per buffer > TMU_NOALLOC_MAX_BUFFER_BYTES
    z = torch.zeros(1, L, L, 128, dtype=torch.float16, device=DEV)
    out = torch.empty_like(z)
    rc = _noalloc(lib, z, out, None, w, True, None)
    assert _lib.STATUS_NAMES[rc] == "TMU_ERR_UNSUPPORTED"
    assert b"static scratch" in lib.tmu_last_error()


def test_noalloc_wide_cz256_matches_and_refuses_in_place():
    """c_z = c = 256: two calls in a row against tmu_trimul, then an in-place call (z_out == z),
    which the wide kernels cannot do, refused with TMU_ERR_INVALID_ARGUMENT before any launch."""
    lib = _lib.load()
    trunk = FoldingTrunk(1, 256, 256, hidden=512, seed=23, ln_noise=0.1)
    status = ops.new_status(DEV)
    for k, (L, direction, n_pad) in enumerate(((60, "out", 5), (128, "in", 0))):
        w = ops.TrimulWeights.from_module(getattr(trunk.blocks[0], "tri_mul_" + direction), DEV)
        z = pair_tensor(1, L, 256, 50 + k).half().to(DEV)
        mask = pair_mask(1, L, n_pad).half().to(DEV) if n_pad else None
        ref = ops.trimul(z, mask, w, direction == "out")
        out = torch.full_like(z, float("nan"))
        rc = _noalloc(lib, z, out, mask, w, direction == "out", status)
        assert rc == 0, (_lib.STATUS_NAMES.get(rc), lib.tmu_last_error())
        code, site = ops.read_status(status)
        assert code == 0, f"device status {code} at {site:#x}"
        got, want = out.float().cpu(), ref.float().cpu()
        assert torch.isfinite(got).all()
        diff = float((got - want).abs().max())
        assert diff <= 4 * _ulp16(float(want.abs().max())), f"call {k}: max diff {diff}"
    rc = _noalloc(lib, z, z, None, w, False, status)
    assert _lib.STATUS_NAMES[rc] == "TMU_ERR_INVALID_ARGUMENT"
    z129 = torch.zeros(1, 129, 129, 256, dtype=torch.float16, device=DEV)  # 256 * 129 * 136 * 2 > 8 MiB
    rc = _noalloc(lib, z129, torch.empty_like(z129), None, w, True, None)
    assert _lib.STATUS_NAMES[rc] == "TMU_ERR_UNSUPPORTED"
