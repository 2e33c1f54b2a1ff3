"""The C ABI library loads and exports every entry point the header declares.

CPU only: no call here launches a kernel. Argument checks that fail before any
CUDA call are exercised because they define the error behaviour the Python
mirror maps to ValueError.
"""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "gptq_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gq_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from mlx_gptq_b200 import _lib

    return _lib.lib()


def test_header_declares_entry_points():
    names = _declared()
    assert "gq_hessian_bf16" in names and "gq_gptq_mxfp" in names and "gq_gptq_affine" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_the_header():
    from mlx_gptq_b200 import _lib

    assert set(_declared()) == set(_lib.SIGNATURES)


def test_status_strings(lib):
    assert lib.gq_abi_version() == 1
    assert lib.gq_status_string(0) == b"ok"
    assert b"positive definite" in lib.gq_status_string(2)


def test_argument_errors_without_gpu(lib):
    from mlx_gptq_b200 import _lib

    p = ctypes.c_void_p(16)
    st = lib.gq_pack_q(p, 2, 32, 3, p, None)  # 3-bit is not packable (packing.py:17-18)
    assert st == _lib.GQ_ERR_ARG
    assert b"cannot pack 3-bit" in lib.gq_last_error()
    st = lib.gq_rtn_mxfp(p, 0, 4, 48, 1, p, None, p, None, 0, None)  # 48 % 32 != 0
    assert st == _lib.GQ_ERR_ARG
    st = lib.gq_gptq_mxfp(p, 0, p, p, None, None, 1, 8, 64, 1, 7, p, None, p, None, 0, None, None, 0, None)
    assert st == _lib.GQ_ERR_ARG and b"algorithm" in lib.gq_last_error()
    st = lib.gq_gptq_affine(p, None, 0, p, 1, 8, 96, 4, 64, 128, 1, 1, p, p, p, None, None, 0, None, None)
    assert st == _lib.GQ_ERR_ARG  # 96 not divisible by 64


def test_python_errors_match_reference_types():
    import numpy as np
    from mlx_gptq_b200 import grid, packing

    with pytest.raises(ValueError):
        packing.pack_q(np.zeros((2, 32), np.uint8), 3)
    with pytest.raises(ValueError):
        grid.mode_defaults("int3")
    assert grid.mode_defaults("mxfp4") == (32, 4) and grid.mode_defaults("affine") == (64, 4)


def test_cpu_tensors_are_rejected_not_computed():
    import torch
    from mlx_gptq_b200 import solve_gptq

    W = torch.randn(1, 8, 64)
    H = torch.eye(64).unsqueeze(0)
    with pytest.raises(RuntimeError, match="CUDA"):
        solve_gptq(W, H, bits=4, group_size=32)


def test_hessian_tile_schedule_queries(lib, monkeypatch):
    """Host-only queries of the Hessian tile schedule: 256x256 tiles on or above the
    diagonal for the CTA-pair kernel (one per pair in a wave), 128x256 ones for the
    one-CTA kernel (one per CTA)."""
    for c in (64, 1088, 2048, 4096, 11008):
        t = -(-c // 256)
        monkeypatch.setenv("GQ_HESSIAN_KERNEL", "2sm")
        assert lib.gq_hessian_tile_count(c) == t * (t + 1) // 2
        assert lib.gq_hessian_concurrent_tiles(148) == 74
        monkeypatch.setenv("GQ_HESSIAN_KERNEL", "1sm")
        mt = -(-c // 128)
        assert lib.gq_hessian_tile_count(c) == sum(min(2 * tn + 2, mt) for tn in range(t))
        assert lib.gq_hessian_concurrent_tiles(148) == 148
    assert lib.gq_hessian_tile_count(0) == 0 and lib.gq_hessian_concurrent_tiles(0) == 0
    # the range form validates its range before touching the device
    import ctypes

    import numpy as np

    monkeypatch.setenv("GQ_HESSIAN_KERNEL", "2sm")
    h = np.zeros(64, np.float32)
    assert h.ctypes.data % 16 == 0
    st = lib.gq_hessian_bf16_range(None, 0, 4, 8, h.ctypes.data, 4, 1.0, 0.0, 0, 5, None, None)
    assert st == 1 and b"tile range" in lib.gq_last_error()  # GQ_ERR_ARG before any launch
    assert lib.gq_hessian_bf16_range(None, 0, 4, 8, h.ctypes.data, 4, 1.0, 0.0, 1, 1, None, None) == 0  # empty


def test_timed_out_status_word_raises(monkeypatch):
    """A bounded device wait that gave up leaves GQ_ERR_TIMEOUT in the device's status
    word; the solver entry points read it and raise instead of using a partial H.
    Host-side check with a CPU stand-in for the device word."""
    import torch

    from mlx_gptq_b200 import _lib

    word = torch.tensor([_lib.GQ_ERR_TIMEOUT], dtype=torch.int32)
    monkeypatch.setattr(_lib, "status_word", lambda device=None: word)
    with pytest.raises(_lib.GQError) as ei:
        _lib.raise_on_device_timeout("cpu")
    assert ei.value.status == _lib.GQ_ERR_TIMEOUT and "gave up" in str(ei.value)
    assert int(word.item()) == 0  # reported once, then cleared
    _lib.raise_on_device_timeout("cpu")  # a clear word raises nothing
