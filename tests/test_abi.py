"""CPU checks of the C-ABI library: it loads without a GPU, exports every symbol include/tmu.h
declares, and its host-only helpers agree with the Python side.  No kernel is launched."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from esmfold2_mlx_b200 import _lib, build, ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build.build()  # no-op when up to date; nvcc cross-compiles sm_100a without a GPU
    return _lib.load()


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "tmu.h")).read()
    return sorted(set(re.findall(r"\b(tmu_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported(lib):
    declared = _declared_symbols()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signatures out of sync with tmu.h"


def test_host_helpers(lib):
    assert lib.tmu_version().startswith(b"tmu-b200")
    assert lib.tmu_status_name(0) == b"TMU_OK"
    assert lib.tmu_status_name(6) == b"TMU_ERR_DEVICE_TIMEOUT"
    for code, name in _lib.STATUS_NAMES.items():
        assert lib.tmu_status_name(code).decode() == name
    for L in (1, 7, 8, 76, 146, 238, 3072):
        assert lib.tmu_row_pitch(L) == ops.row_pitch(L) and ops.row_pitch(L) % 8 == 0
    assert ops.proj_row_order(128) == ops.proj_row_order_py(128)
    assert sorted(ops.proj_row_order_py(128)) == list(range(512))
    assert lib.tmu_proj_row_order(100, (ctypes.c_int * 400)()) == 1


def test_workspace_size(lib):
    for B, L in ((1, 76), (64, 146), (1, 3072)):
        cm = B * 128 * L * ops.row_pitch(L) * 2
        cm = (cm + 255) // 256 * 256
        assert lib.tmu_workspace_bytes(B, L, 128, 128) == 256 + 3 * cm
    assert lib.tmu_workspace_bytes(0, 10, 128, 128) == 0


def test_argument_checks_need_no_gpu(lib):
    # shape / null checks run before any CUDA call
    W = ctypes.POINTER(_lib.TmuTrimulWeights)
    assert lib.tmu_trimul(None, None, None, W(), 1, 64, 192, 192, 1, 1e-5, None, 0, None) == 4  # unsupported c
    assert lib.tmu_trimul(None, None, None, W(), 1, 64, 256, 128, 1, 1e-5, None, 0, None) == 4  # c != c_z
    assert lib.tmu_trimul(None, None, None, W(), 0, 64, 128, 128, 1, 1e-5, None, 0, None) == 1
    assert lib.tmu_contract(None, None, None, 0, 64, 1, None, None) == 1
    assert lib.tmu_contract(None, None, None, 1, 9000, 1, None, None) == 4
    assert lib.tmu_reset_status(None, None) == 1
    old = lib.tmu_set_wait_timeout_ns(123)
    assert lib.tmu_set_wait_timeout_ns(old) == 123


def test_argument_checks_of_the_later_entry_points_need_no_gpu(lib):
    """tmu_transition, tmu_disto_expected, the slab and IPC helpers reject bad arguments before
    touching a device (codes: 1 invalid argument, 4 unsupported)."""
    TW = ctypes.POINTER(_lib.TmuTransitionWeights)
    tw = _lib.TmuTransitionWeights()
    assert lib.tmu_transition(None, None, TW(), 1, 64, 192, 512, 0, None, None) == 4  # c_z 192 not built
    assert lib.tmu_transition(None, None, TW(), 1, 64, 128, 100, 0, None, None) == 4  # hidden % 64
    assert lib.tmu_transition(None, None, TW(), 1, 64, 128, 512, 7, None, None) == 1  # activation
    assert lib.tmu_transition(None, None, ctypes.byref(tw), 1, 64, 128, 512, 0, None, None) == 1  # no weights
    assert lib.tmu_disto_expected(None, None, None, None, None, 1, 64, 128, 64, None, None) == 4  # 128 bins only
    assert lib.tmu_disto_expected(None, None, None, None, None, 1, 64, 192, 128, None, None) == 4
    assert lib.tmu_disto_expected(None, None, None, None, None, 1, 64, 128, 128, None, None) == 1
    # a column block of x needs a row pitch >= N and a multiple of 8
    assert lib.tmu_contract_ex(None, None, None, 1, 128, 256, 256, 128, 200, 0, None, None) == 1
    assert lib.tmu_contract_ex(None, None, None, 1, 128, 256, 256, 128, 260, 0, None, None) == 1
    assert lib.tmu_contract_ex(None, None, None, 1, 128, 256, 256, 128, 0, -1, None, None) == 1
    off = ctypes.c_ulonglong(0)
    assert lib.tmu_ipc_export(None, None, ctypes.byref(off)) == 1
    p = ctypes.c_void_p()
    assert lib.tmu_ipc_import(None, 0, ctypes.byref(p)) == 1
    assert lib.tmu_ipc_close(None) == 1
    assert lib.tmu_copy_async(None, None, 0, None) == 1


def test_pair_cond_argument_checks_need_no_gpu(lib):
    """tmu_pair_cond rejects unsupported widths and missing weights before touching a device."""
    PW = ctypes.POINTER(_lib.TmuPairCondWeights)
    pw = _lib.TmuPairCondWeights()
    args = lambda ct, cr, cp, h, nb, H: (None, None, PW(), 1, 16, ct, cr, cp, h, nb, H, None, None, 0, None, None)  # noqa: E731
    assert lib.tmu_pair_cond(*args(256, 128, 256, 512, 192, 16)) == 4  # c_trunk != c_rel
    assert lib.tmu_pair_cond(*args(256, 256, 192, 512, 192, 16)) == 4  # c_pair
    assert lib.tmu_pair_cond(*args(256, 256, 256, 512, 192, 16)) == 1  # no weights
    a = list(args(256, 256, 256, 512, 192, 16))
    a[2] = ctypes.byref(pw)
    assert lib.tmu_pair_cond(*a) == 1  # empty weight struct
    assert lib.tmu_pair_cond_workspace_bytes(1, 16, 512, 256, 2) == 3 * 16 * 16 * 256 * 2 + 16 * 16 * 512 * 2
    assert lib.tmu_pair_cond_workspace_bytes(1, 5, 256, 128, 0) == 6400 + 12800  # terms rounded up to 256 B
    assert lib.tmu_pair_cond_workspace_bytes(0, 16, 512, 256, 2) == 0


def test_pair_block_workspace_and_argument_checks_need_no_gpu(lib):
    """tmu_pair_block: the workspace is the tri-mul's plus, at c_z = 256, one pair buffer; bad
    arguments are rejected before anything is launched (codes: 1 invalid argument, 2 misaligned,
    3 workspace too small, 4 unsupported).  The pointers below are never dereferenced."""
    for B, L in ((1, 76), (2, 146)):
        assert lib.tmu_pair_block_workspace_bytes(B, L, 128, 128) == lib.tmu_workspace_bytes(B, L, 128, 128)
        pair = (B * L * L * 256 * 2 + 255) // 256 * 256
        assert lib.tmu_pair_block_workspace_bytes(B, L, 256, 256) == lib.tmu_workspace_bytes(B, L, 256, 256) + pair
    assert lib.tmu_pair_block_workspace_bytes(0, 10, 128, 128) == 0

    fake = lambda i: ctypes.c_void_p(0x100000 + 0x1000 * i)  # noqa: E731  16- and 256-byte aligned
    w = _lib.TmuTrimulWeights(*(fake(i) if i not in (3, 7, 9) else None for i in range(10)))  # no biases
    tw = _lib.TmuTransitionWeights(fake(20), fake(21), fake(22), fake(23))
    need = lib.tmu_pair_block_workspace_bytes(1, 64, 128, 128)

    def call(c=128, hidden=256, act=0, w_in=w, tw_=tw, ws=fake(30), nbytes=need, eps=1e-5):
        return lib.tmu_pair_block(fake(40), fake(41), None, ctypes.byref(w), ctypes.byref(w_in), ctypes.byref(tw_),
                                  1, 64, c, c, hidden, act, eps, ws, nbytes, None)

    assert call(c=192) == 4
    assert call(hidden=100) == 4
    assert call(act=5) == 1
    assert call(tw_=_lib.TmuTransitionWeights()) == 1
    assert call(w_in=_lib.TmuTrimulWeights()) == 1
    one_bias = _lib.TmuTrimulWeights(*(fake(i) if i not in (3, 9) else None for i in range(10)))  # b_emit only
    assert call(w_in=one_bias) == 1
    assert call(ws=None) == 1
    assert call(ws=ctypes.c_void_p(0x100010)) == 2
    assert call(nbytes=need - 1) == 3
    assert call(eps=0.0) == 1
