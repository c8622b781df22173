"""C-ABI checks that need no GPU: the library loads, exports exactly what
``include/picotron_b200.h`` declares, and rejects bad arguments before touching CUDA."""

from __future__ import annotations

import ctypes
import re
import subprocess
import threading
from pathlib import Path

import pytest

from picotron_b200 import _capi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "picotron_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^PT_API\s+[\w\s\*]+?\b(pt_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for required in ("pt_rmsnorm_fwd", "pt_rmsnorm_bwd", "pt_rmsnorm_dw_reduce",
                     "pt_swiglu_fwd", "pt_swiglu_bwd", "pt_rope_fwd", "pt_rope_bwd",
                     "pt_probe", "pt_last_error"):
        assert required in names


def test_library_loads_and_exports_every_declared_symbol():
    lib = _capi.library()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} not exported"
        assert name in _capi.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_capi.SIGNATURES) == set(declared_functions())
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_capi.LIBRARY_PATH)],
                        capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (pt_\w+)$", nm, flags=re.M))
    assert exported == set(declared_functions())


def test_abi_version_matches():
    assert _capi.library().pt_abi_version() == _capi.ABI_VERSION


def test_header_constants_match_binding():
    text = HEADER.read_text()
    for name in ("PT_OK", "PT_ERR_INVALID_ARGUMENT", "PT_ERR_UNSUPPORTED_DTYPE", "PT_ERR_SHAPE",
                 "PT_ERR_DEVICE", "PT_ERR_CUDA", "PT_FLOAT32", "PT_FLOAT16", "PT_BFLOAT16",
                 "PT_ROPE_INTERLEAVED", "PT_ROPE_ROTATE_HALF"):
        value = int(re.search(rf"\b{name}\s*=\s*(\d+)", text).group(1))
        assert getattr(_capi, name) == value, name


def _status(fn, *args):
    return fn(*args)


def test_rmsnorm_host_validation_without_gpu():
    lib = _capi.library()
    # negative rows
    assert lib.pt_rmsnorm_fwd(1, 8, 1, 1, 8, None, -1, 8, 0, 0, 1e-6, None) == _capi.PT_ERR_SHAPE
    assert "rows" in _capi.last_error()
    # zero hidden
    assert lib.pt_rmsnorm_fwd(1, 8, 1, 1, 8, None, 4, 0, 0, 0, 1e-6, None) == _capi.PT_ERR_SHAPE
    # rows == 0 is a no-op success
    assert lib.pt_rmsnorm_fwd(None, 8, None, None, 8, None, 0, 8, 0, 0, 1e-6, None) == _capi.PT_OK
    # negative eps
    assert (lib.pt_rmsnorm_fwd(1, 8, 1, 1, 8, None, 4, 8, 0, 0, -1.0, None)
            == _capi.PT_ERR_INVALID_ARGUMENT)
    # row stride smaller than hidden
    assert lib.pt_rmsnorm_fwd(1, 4, 1, 1, 8, None, 4, 8, 0, 0, 1e-6, None) == _capi.PT_ERR_SHAPE
    # null pointer
    assert (lib.pt_rmsnorm_fwd(None, 8, 1, 1, 8, None, 4, 8, 0, 0, 1e-6, None)
            == _capi.PT_ERR_INVALID_ARGUMENT)
    assert "x is NULL" in _capi.last_error()
    # backward: num_partials must be positive
    assert (lib.pt_rmsnorm_bwd(1, 8, 1, 8, 1, None, 1, 8, 1, 0, 4, 8, 0, 0, 1e-6, None)
            == _capi.PT_ERR_INVALID_ARGUMENT)
    assert (lib.pt_rmsnorm_dw_reduce(1, 0, 8, 1, 0, None) == _capi.PT_ERR_INVALID_ARGUMENT)
    n = ctypes.c_int(0)
    assert lib.pt_rmsnorm_bwd_num_partials(4, 8, 0, 0, None) == _capi.PT_ERR_INVALID_ARGUMENT


def test_swiglu_and_rope_host_validation_without_gpu():
    lib = _capi.library()
    assert lib.pt_swiglu_fwd(1, 1, 1, -5, 2, None) == _capi.PT_ERR_SHAPE
    assert lib.pt_swiglu_fwd(1, 1, 1, 8, 9, None) == _capi.PT_ERR_UNSUPPORTED_DTYPE
    assert lib.pt_swiglu_fwd(None, None, None, 0, 2, None) == _capi.PT_OK
    assert lib.pt_swiglu_bwd(1, 1, 1, 1, 1, 8, 7, None) == _capi.PT_ERR_UNSUPPORTED_DTYPE
    st = _capi._i64x4
    # odd head_dim
    assert (lib.pt_rope_fwd(1, st([0, 0, 0, 1]), 1, st([0, 0, 0, 1]), st([1, 1, 1, 7]), 1, 1, 4,
                            0, 2, 2, None) == _capi.PT_ERR_SHAPE)
    # unknown layout
    assert (lib.pt_rope_fwd(1, st([0, 0, 0, 1]), 1, st([0, 0, 0, 1]), st([1, 1, 1, 8]), 1, 1, 4,
                            5, 2, 2, None) == _capi.PT_ERR_INVALID_ARGUMENT)
    # non-unit head_dim stride
    assert (lib.pt_rope_bwd(1, st([0, 0, 0, 2]), 1, st([0, 0, 0, 1]), st([1, 1, 1, 8]), 1, 1, 4,
                            0, 2, 2, None) == _capi.PT_ERR_SHAPE)
    # table stride too small
    assert (lib.pt_rope_fwd(1, st([0, 0, 0, 1]), 1, st([0, 0, 0, 1]), st([1, 1, 1, 8]), 1, 1, 3,
                            0, 2, 2, None) == _capi.PT_ERR_SHAPE)
    # unsupported (states, table) dtype pair
    assert (lib.pt_rope_fwd(1, st([0, 0, 0, 1]), 1, st([0, 0, 0, 1]), st([1, 1, 1, 8]), 1, 1, 4,
                            0, 0, 2, None) != _capi.PT_OK)


def test_probe_without_device_reports_an_error():
    status, major, minor, sms = _capi.probe(0)
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        pytest.skip("a GPU is present; covered by the gpu tests")
    assert status == _capi.PT_ERR_DEVICE
    assert _capi.last_error()


def test_last_error_is_thread_local():
    lib = _capi.library()
    assert lib.pt_swiglu_fwd(1, 1, 1, -1, 2, None) == _capi.PT_ERR_SHAPE
    main_message = _capi.last_error()
    seen = {}

    def worker():
        seen["before"] = _capi.last_error()
        lib.pt_swiglu_fwd(1, 1, 1, 8, 42, None)
        seen["after"] = _capi.last_error()

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert seen["before"] == ""
    assert "dtype" in seen["after"]
    assert _capi.last_error() == main_message


def test_errors_raise_the_requested_exception_type():
    from picotron_b200.errors import TritonSwiGLUUnavailable

    with pytest.raises(TritonSwiGLUUnavailable, match="PT_ERR_SHAPE"):
        _capi.swiglu_fwd(1, 1, 1, -1, _capi.PT_BFLOAT16, 0, TritonSwiGLUUnavailable)
    with pytest.raises(_capi.PtError) as info:
        _capi.swiglu_fwd(1, 1, 1, -1, _capi.PT_BFLOAT16, 0)
    assert info.value.status == _capi.PT_ERR_SHAPE
