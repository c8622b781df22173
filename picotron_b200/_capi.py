"""ctypes binding of ``libpicotron_b200.so`` (declared in ``include/picotron_b200.h``).

This module is the only place Python touches the C ABI. Each wrapper takes raw device
addresses (ints), sizes, dtype codes and a stream handle (int), calls the C entry point
and raises :class:`PtError` (or the subclass the caller asks for) on a non-zero status
with the library's thread-local message. There is no fallback: if the shared library is
missing or does not load, :func:`library` raises :class:`LibraryUnavailable`.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().with_name("libpicotron_b200.so")

# enum pt_status
PT_OK = 0
PT_ERR_INVALID_ARGUMENT = 1
PT_ERR_UNSUPPORTED_DTYPE = 2
PT_ERR_SHAPE = 3
PT_ERR_DEVICE = 4
PT_ERR_CUDA = 5

STATUS_NAMES = {
    PT_OK: "PT_OK",
    PT_ERR_INVALID_ARGUMENT: "PT_ERR_INVALID_ARGUMENT",
    PT_ERR_UNSUPPORTED_DTYPE: "PT_ERR_UNSUPPORTED_DTYPE",
    PT_ERR_SHAPE: "PT_ERR_SHAPE",
    PT_ERR_DEVICE: "PT_ERR_DEVICE",
    PT_ERR_CUDA: "PT_ERR_CUDA",
}

# enum pt_dtype
PT_FLOAT32 = 0
PT_FLOAT16 = 1
PT_BFLOAT16 = 2

# enum pt_rope_layout
PT_ROPE_INTERLEAVED = 0
PT_ROPE_ROTATE_HALF = 1

ABI_VERSION = 1

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_float = ctypes.c_float
_c_ptr = ctypes.c_void_p
_c_i64_4 = ctypes.c_int64 * 4

# name -> (restype, argtypes). Mirrors include/picotron_b200.h one to one; the CPU test
# suite checks that every function declared there is exported and listed here.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "pt_abi_version": (_c_int, []),
    "pt_last_error": (ctypes.c_char_p, []),
    "pt_probe": (_c_int, [_c_int, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int),
                          ctypes.POINTER(_c_int)]),
    "pt_rmsnorm_fwd": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_ptr, _c_i64, _c_ptr, _c_i64, _c_i64,
                                _c_int, _c_int, _c_float, _c_ptr]),
    "pt_rmsnorm_bwd_num_partials": (_c_int, [_c_i64, _c_i64, _c_int, _c_int,
                                             ctypes.POINTER(_c_int)]),
    "pt_rmsnorm_bwd": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_i64,
                                _c_ptr, _c_int, _c_i64, _c_i64, _c_int, _c_int, _c_float,
                                _c_ptr]),
    "pt_rmsnorm_dw_reduce": (_c_int, [_c_ptr, _c_int, _c_i64, _c_ptr, _c_int, _c_ptr]),
    "pt_rmsnorm_bwd_fused_workspace": (_c_int, [_c_i64, _c_i64, _c_int, _c_int,
                                                ctypes.POINTER(_c_i64)]),
    "pt_rmsnorm_bwd_fused": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_ptr,
                                      _c_i64, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_int,
                                      _c_int, _c_float, _c_ptr]),
    "pt_add_rmsnorm_bwd_fused_workspace": (_c_int, [_c_i64, _c_i64, _c_int, _c_int,
                                                    ctypes.POINTER(_c_i64)]),
    "pt_add_rmsnorm_bwd_fused": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_i64,
                                          _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_ptr, _c_ptr,
                                          _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_float,
                                          _c_ptr]),
    "pt_swiglu_gemm_fwd": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_ptr, _c_i64, _c_ptr, _c_i64,
                                    _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_int,
                                    _c_ptr]),
    "pt_swiglu_gemm_bwd": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_i64,
                                    _c_ptr, _c_ptr, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64,
                                    _c_i64, _c_int, _c_ptr]),
    "pt_transpose_2d": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64, _c_int, _c_ptr]),
    "pt_cross_entropy_fwd": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr,
                                      _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_int,
                                      _c_ptr]),
    "pt_cross_entropy_bwd": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr,
                                      _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                      _c_i64, _c_i64, _c_int, _c_ptr]),
    "pt_adamw_step": (_c_int, [ctypes.POINTER(_c_ptr), ctypes.POINTER(_c_ptr),
                               ctypes.POINTER(_c_ptr), ctypes.POINTER(_c_ptr),
                               ctypes.POINTER(_c_i64), ctypes.POINTER(_c_i64),
                               ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                               _c_int, ctypes.c_double, ctypes.c_double, ctypes.c_double, _c_int,
                               _c_ptr]),
    "pt_rope_qk_fwd": (_c_int, [_c_ptr, _c_i64_4, _c_ptr, _c_i64_4, _c_i64_4, _c_ptr, _c_i64_4,
                                _c_ptr, _c_i64_4, _c_i64_4, _c_ptr, _c_ptr, _c_i64, _c_int,
                                _c_int, _c_int, _c_ptr]),
    "pt_rope_qk_bwd": (_c_int, [_c_ptr, _c_i64_4, _c_ptr, _c_i64_4, _c_i64_4, _c_ptr, _c_i64_4,
                                _c_ptr, _c_i64_4, _c_i64_4, _c_ptr, _c_ptr, _c_i64, _c_int,
                                _c_int, _c_int, _c_ptr]),
    "pt_add_rmsnorm_fwd": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_i64,
                                    _c_ptr, _c_i64, _c_ptr, _c_i64, _c_i64, _c_int, _c_int,
                                    _c_float, _c_ptr]),
    "pt_add_rmsnorm_bwd_num_partials": (_c_int, [_c_i64, _c_i64, _c_int, _c_int,
                                                 ctypes.POINTER(_c_int)]),
    "pt_add_rmsnorm_bwd": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr,
                                    _c_ptr, _c_ptr, _c_i64, _c_ptr, _c_int, _c_i64, _c_i64,
                                    _c_int, _c_int, _c_float, _c_ptr]),
    "pt_rmsnorm_bwd_noalloc": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_ptr,
                                        _c_i64, _c_ptr, _c_i64, _c_i64, _c_int, _c_int,
                                        _c_float, _c_ptr]),
    "pt_take_device_error": (_c_int, [ctypes.POINTER(_c_int)]),
    "pt_selftest_wait_timeout": (_c_int, [_c_i64, _c_ptr]),
    "pt_swiglu_fwd": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_i64, _c_int, _c_ptr]),
    "pt_swiglu_bwd": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_int, _c_ptr]),
    "pt_rope_fwd": (_c_int, [_c_ptr, _c_i64_4, _c_ptr, _c_i64_4, _c_i64_4, _c_ptr, _c_ptr,
                             _c_i64, _c_int, _c_int, _c_int, _c_ptr]),
    "pt_rope_bwd": (_c_int, [_c_ptr, _c_i64_4, _c_ptr, _c_i64_4, _c_i64_4, _c_ptr, _c_ptr,
                             _c_i64, _c_int, _c_int, _c_int, _c_ptr]),
}


class LibraryUnavailable(RuntimeError):
    """The compiled library is missing or cannot be loaded."""


class PtError(RuntimeError):
    """A C-ABI call returned a non-zero pt_status."""

    def __init__(self, function: str, status: int, message: str) -> None:
        self.function = function
        self.status = status
        self.message = message
        name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{function} failed with {name}: {message}")


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raise if it is not built or loadable."""

    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIBRARY_PATH.is_file():
            raise LibraryUnavailable(
                f"{LIBRARY_PATH.name} is not built; run `python -m picotron_b200.build`"
            )
        try:
            lib = ctypes.CDLL(str(LIBRARY_PATH))
        except OSError as error:
            raise LibraryUnavailable(f"cannot load {LIBRARY_PATH}: {error}") from error
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.pt_abi_version()
        if version != ABI_VERSION:
            raise LibraryUnavailable(
                f"{LIBRARY_PATH.name} has ABI version {version}; expected {ABI_VERSION}"
            )
        _lib = lib
        return lib


def is_available() -> bool:
    """True when the library loads (says nothing about a GPU being present)."""

    try:
        library()
    except LibraryUnavailable:
        return False
    return True


def last_error() -> str:
    return library().pt_last_error().decode("utf-8", "replace")


def _check(function: str, status: int, error_type: type[Exception] | None) -> None:
    if status == PT_OK:
        return
    message = last_error()
    error = PtError(function, status, message)
    if error_type is not None and error_type is not PtError:
        raise error_type(str(error)) from error
    raise error


def _i64x4(values) -> ctypes.Array:
    return _c_i64_4(*[int(v) for v in values])


# ------------------------------------------------------------------------- wrappers --


def probe(device: int) -> tuple[int, int, int, int]:
    """Return (status, cc_major, cc_minor, sm_count) for ``device`` without raising."""

    major, minor, sms = _c_int(0), _c_int(0), _c_int(0)
    status = library().pt_probe(int(device), ctypes.byref(major), ctypes.byref(minor),
                                ctypes.byref(sms))
    return status, major.value, minor.value, sms.value


def rmsnorm_fwd(x: int, x_row_stride: int, weight: int, y: int, y_row_stride: int,
                rstd: int | None, rows: int, hidden: int, x_dtype: int, w_dtype: int,
                eps: float, stream: int, error_type: type[Exception] | None = None) -> None:
    status = library().pt_rmsnorm_fwd(x, x_row_stride, weight, y, y_row_stride, rstd, rows,
                                      hidden, x_dtype, w_dtype, eps, stream)
    _check("pt_rmsnorm_fwd", status, error_type)


def rmsnorm_bwd_num_partials(rows: int, hidden: int, x_dtype: int, w_dtype: int,
                             error_type: type[Exception] | None = None) -> int:
    out = _c_int(0)
    status = library().pt_rmsnorm_bwd_num_partials(rows, hidden, x_dtype, w_dtype,
                                                   ctypes.byref(out))
    _check("pt_rmsnorm_bwd_num_partials", status, error_type)
    return out.value


def rmsnorm_bwd(dy: int, dy_row_stride: int, x: int, x_row_stride: int, weight: int,
                rstd: int | None, dx: int, dx_row_stride: int, dw_partials: int,
                num_partials: int, rows: int, hidden: int, x_dtype: int, w_dtype: int,
                eps: float, stream: int, error_type: type[Exception] | None = None) -> None:
    status = library().pt_rmsnorm_bwd(dy, dy_row_stride, x, x_row_stride, weight, rstd, dx,
                                      dx_row_stride, dw_partials, num_partials, rows, hidden,
                                      x_dtype, w_dtype, eps, stream)
    _check("pt_rmsnorm_bwd", status, error_type)


def rmsnorm_dw_reduce(dw_partials: int, num_partials: int, hidden: int, dw: int,
                      dw_dtype: int, stream: int,
                      error_type: type[Exception] | None = None) -> None:
    status = library().pt_rmsnorm_dw_reduce(dw_partials, num_partials, hidden, dw, dw_dtype,
                                            stream)
    _check("pt_rmsnorm_dw_reduce", status, error_type)


def rmsnorm_bwd_fused_workspace(rows: int, hidden: int, x_dtype: int, w_dtype: int,
                                error_type: type[Exception] | None = None) -> int:
    """Floats of workspace that pt_rmsnorm_bwd_fused needs."""

    out = _c_i64(0)
    status = library().pt_rmsnorm_bwd_fused_workspace(rows, hidden, x_dtype, w_dtype,
                                                      ctypes.byref(out))
    _check("pt_rmsnorm_bwd_fused_workspace", status, error_type)
    return out.value


def rmsnorm_bwd_fused(dy: int, dy_row_stride: int, x: int, x_row_stride: int, weight: int,
                      rstd: int | None, dx: int, dx_row_stride: int, dw: int, workspace: int,
                      workspace_floats: int, rows: int, hidden: int, x_dtype: int,
                      w_dtype: int, eps: float, stream: int,
                      error_type: type[Exception] | None = None) -> None:
    """RMSNorm backward with the dweight reduction in the same launch (pt_rmsnorm_bwd_fused)."""

    status = library().pt_rmsnorm_bwd_fused(dy, dy_row_stride, x, x_row_stride, weight, rstd,
                                            dx, dx_row_stride, dw, workspace, workspace_floats,
                                            rows, hidden, x_dtype, w_dtype, eps, stream)
    _check("pt_rmsnorm_bwd_fused", status, error_type)


def add_rmsnorm_bwd_fused_workspace(rows: int, hidden: int, x_dtype: int, w_dtype: int,
                                    error_type: type[Exception] | None = None) -> int:
    """Floats of workspace that pt_add_rmsnorm_bwd_fused needs."""

    out = _c_i64(0)
    status = library().pt_add_rmsnorm_bwd_fused_workspace(rows, hidden, x_dtype, w_dtype,
                                                          ctypes.byref(out))
    _check("pt_add_rmsnorm_bwd_fused_workspace", status, error_type)
    return out.value


def add_rmsnorm_bwd_fused(dy: int, dy_row_stride: int, dh: int | None, dh_row_stride: int,
                          h: int, h_row_stride: int, weight: int, rstd: int | None, dx: int,
                          dx_row_stride: int, dw: int, workspace: int, workspace_floats: int,
                          rows: int, hidden: int, x_dtype: int, w_dtype: int, eps: float,
                          stream: int, error_type: type[Exception] | None = None) -> None:
    """Fused residual add + RMSNorm backward with the dweight reduction in the same launch
    (pt_add_rmsnorm_bwd_fused)."""

    status = library().pt_add_rmsnorm_bwd_fused(dy, dy_row_stride, dh, dh_row_stride, h,
                                                h_row_stride, weight, rstd, dx, dx_row_stride,
                                                dw, workspace, workspace_floats, rows, hidden,
                                                x_dtype, w_dtype, eps, stream)
    _check("pt_add_rmsnorm_bwd_fused", status, error_type)


def rmsnorm_bwd_noalloc(dy: int, dy_row_stride: int, x: int, x_row_stride: int, weight: int,
                        rstd: int | None, dx: int, dx_row_stride: int, dw: int, rows: int,
                        hidden: int, x_dtype: int, w_dtype: int, eps: float, stream: int,
                        error_type: type[Exception] | None = None) -> None:
    """RMSNorm backward that allocates nothing (see pt_rmsnorm_bwd_noalloc)."""

    status = library().pt_rmsnorm_bwd_noalloc(dy, dy_row_stride, x, x_row_stride, weight, rstd,
                                              dx, dx_row_stride, dw, rows, hidden, x_dtype,
                                              w_dtype, eps, stream)
    _check("pt_rmsnorm_bwd_noalloc", status, error_type)


def add_rmsnorm_fwd(residual: int, residual_row_stride: int, branch: int,
                    branch_row_stride: int, weight: int, h_out: int, h_row_stride: int,
                    y: int, y_row_stride: int, rstd: int | None, rows: int, hidden: int,
                    x_dtype: int, w_dtype: int, eps: float, stream: int,
                    error_type: type[Exception] | None = None) -> None:
    """Fused residual add + RMSNorm forward (see pt_add_rmsnorm_fwd)."""

    status = library().pt_add_rmsnorm_fwd(residual, residual_row_stride, branch,
                                          branch_row_stride, weight, h_out, h_row_stride, y,
                                          y_row_stride, rstd, rows, hidden, x_dtype, w_dtype,
                                          eps, stream)
    _check("pt_add_rmsnorm_fwd", status, error_type)


def add_rmsnorm_bwd_num_partials(rows: int, hidden: int, x_dtype: int, w_dtype: int,
                                 error_type: type[Exception] | None = None) -> int:
    out = _c_int(0)
    status = library().pt_add_rmsnorm_bwd_num_partials(rows, hidden, x_dtype, w_dtype,
                                                       ctypes.byref(out))
    _check("pt_add_rmsnorm_bwd_num_partials", status, error_type)
    return out.value


def add_rmsnorm_bwd(dy: int, dy_row_stride: int, dh: int | None, dh_row_stride: int, h: int,
                    h_row_stride: int, weight: int, rstd: int | None, dx: int,
                    dx_row_stride: int, dw_partials: int, num_partials: int, rows: int,
                    hidden: int, x_dtype: int, w_dtype: int, eps: float, stream: int,
                    error_type: type[Exception] | None = None) -> None:
    """Fused residual add + RMSNorm backward (see pt_add_rmsnorm_bwd)."""

    status = library().pt_add_rmsnorm_bwd(dy, dy_row_stride, dh, dh_row_stride, h,
                                          h_row_stride, weight, rstd, dx, dx_row_stride,
                                          dw_partials, num_partials, rows, hidden, x_dtype,
                                          w_dtype, eps, stream)
    _check("pt_add_rmsnorm_bwd", status, error_type)


def swiglu_gemm_fwd(x: int, x_row_stride: int, w_gate: int, w_up: int, w_row_stride: int,
                    act: int, act_row_stride: int, gate_out: int | None, up_out: int | None,
                    pre_row_stride: int, m: int, n: int, k: int, dtype: int, stream: int,
                    error_type: type[Exception] | None = None) -> None:
    """Fused gate/up GEMM + SwiGLU activation on the tensor cores (pt_swiglu_gemm_fwd)."""

    status = library().pt_swiglu_gemm_fwd(x, x_row_stride, w_gate, w_up, w_row_stride, act,
                                          act_row_stride, gate_out, up_out, pre_row_stride, m,
                                          n, k, dtype, stream)
    _check("pt_swiglu_gemm_fwd", status, error_type)


def swiglu_gemm_bwd(dy: int, dy_row_stride: int, w_down_t: int, w_row_stride: int, gate: int,
                    up: int, pre_row_stride: int, dgate: int, dup: int, grad_row_stride: int,
                    dact_out: int | None, dact_row_stride: int, m: int, n: int, k: int,
                    dtype: int, stream: int, error_type: type[Exception] | None = None) -> None:
    """The down projection's input gradient with the SwiGLU backward in its epilogue
    (pt_swiglu_gemm_bwd)."""

    status = library().pt_swiglu_gemm_bwd(dy, dy_row_stride, w_down_t, w_row_stride, gate, up,
                                          pre_row_stride, dgate, dup, grad_row_stride, dact_out,
                                          dact_row_stride, m, n, k, dtype, stream)
    _check("pt_swiglu_gemm_bwd", status, error_type)


def transpose_2d(src: int, src_row_stride: int, dst: int, dst_row_stride: int, rows: int,
                 cols: int, dtype: int, stream: int,
                 error_type: type[Exception] | None = None) -> None:
    """dst = src transposed (pt_transpose_2d)."""

    status = library().pt_transpose_2d(src, src_row_stride, dst, dst_row_stride, rows, cols,
                                       dtype, stream)
    _check("pt_transpose_2d", status, error_type)


def cross_entropy_fwd(logits: int, vocab: int, outer: int, inner: int, logits_strides,
                      targets: int, targets_strides, ignore_index: int, row_loss: int,
                      row_lse: int, mean_out: int, dtype: int, stream: int,
                      error_type: type[Exception] | None = None) -> None:
    """Per-row loss / lse and the mean cross-entropy (see pt_cross_entropy_fwd)."""

    status = library().pt_cross_entropy_fwd(logits, vocab, outer, inner, logits_strides[0],
                                            logits_strides[1], targets, targets_strides[0],
                                            targets_strides[1], ignore_index, row_loss, row_lse,
                                            mean_out, dtype, stream)
    _check("pt_cross_entropy_fwd", status, error_type)


def cross_entropy_bwd(logits: int, vocab: int, outer: int, inner: int, logits_strides,
                      targets: int, targets_strides, ignore_index: int, row_lse: int,
                      mean_out: int, grad_loss: int | None, dlogits: int, dlogits_strides,
                      dtype: int, stream: int,
                      error_type: type[Exception] | None = None) -> None:
    """Logits gradient of the mean cross-entropy (see pt_cross_entropy_bwd)."""

    status = library().pt_cross_entropy_bwd(logits, vocab, outer, inner, logits_strides[0],
                                            logits_strides[1], targets, targets_strides[0],
                                            targets_strides[1], ignore_index, row_lse, mean_out,
                                            grad_loss, dlogits, dlogits_strides[0],
                                            dlogits_strides[1], dtype, stream)
    _check("pt_cross_entropy_bwd", status, error_type)


def adamw_step(params, grads, exp_avgs, exp_avg_sqs, numels, steps, lrs, weight_decays,
               beta1: float, beta2: float, eps: float, maximize: bool, stream: int,
               error_type: type[Exception] | None = None) -> None:
    """One fused AdamW step over lists of device addresses (see pt_adamw_step)."""

    n = len(params)
    ptrs = lambda xs: (_c_ptr * n)(*[int(x) for x in xs])  # noqa: E731
    status = library().pt_adamw_step(
        ptrs(params), ptrs(grads), ptrs(exp_avgs), ptrs(exp_avg_sqs),
        (_c_i64 * n)(*[int(x) for x in numels]), (_c_i64 * n)(*[int(x) for x in steps]),
        (ctypes.c_double * n)(*[float(x) for x in lrs]),
        (ctypes.c_double * n)(*[float(x) for x in weight_decays]), n, float(beta1),
        float(beta2), float(eps), int(bool(maximize)), stream)
    _check("pt_adamw_step", status, error_type)


def rope_qk(direction: str, q: int, q_strides, q_out: int, q_out_strides, q_sizes, k: int,
            k_strides, k_out: int, k_out_strides, k_sizes, cosine: int, sine: int,
            table_row_stride: int, layout: int, dtype: int, table_dtype: int, stream: int,
            error_type: type[Exception] | None = None) -> None:
    """Query and key in one launch; ``direction`` is "fwd" or "bwd" (see pt_rope_qk_fwd)."""

    fn = library().pt_rope_qk_fwd if direction == "fwd" else library().pt_rope_qk_bwd
    status = fn(q, _i64x4(q_strides), q_out, _i64x4(q_out_strides), _i64x4(q_sizes), k,
                _i64x4(k_strides), k_out, _i64x4(k_out_strides), _i64x4(k_sizes), cosine, sine,
                table_row_stride, layout, dtype, table_dtype, stream)
    _check("pt_rope_qk_" + direction, status, error_type)


def selftest_wait_timeout(limit_cycles: int, stream: int) -> None:
    """Launch the bounded-wait self-test (see pt_selftest_wait_timeout)."""

    _check("pt_selftest_wait_timeout",
           library().pt_selftest_wait_timeout(limit_cycles, stream), None)


def take_device_error() -> int:
    """Read and clear the device-side error word of the current device (synchronous)."""

    code = _c_int(0)
    _check("pt_take_device_error", library().pt_take_device_error(ctypes.byref(code)), None)
    return code.value


def swiglu_fwd(gate: int, up: int, out: int, n: int, dtype: int, stream: int,
               error_type: type[Exception] | None = None) -> None:
    status = library().pt_swiglu_fwd(gate, up, out, n, dtype, stream)
    _check("pt_swiglu_fwd", status, error_type)


def swiglu_bwd(dout: int, gate: int, up: int, dgate: int, dup: int, n: int, dtype: int,
               stream: int, error_type: type[Exception] | None = None) -> None:
    status = library().pt_swiglu_bwd(dout, gate, up, dgate, dup, n, dtype, stream)
    _check("pt_swiglu_bwd", status, error_type)


def rope(direction: str, x: int, x_strides, out: int, out_strides, sizes, cosine: int,
         sine: int, table_row_stride: int, layout: int, dtype: int, table_dtype: int,
         stream: int, error_type: type[Exception] | None = None) -> None:
    """``direction`` is "fwd" (rotate by +angle) or "bwd" (rotate by -angle)."""

    name = {"fwd": "pt_rope_fwd", "bwd": "pt_rope_bwd"}[direction]
    fn = getattr(library(), name)
    status = fn(x, _i64x4(x_strides), out, _i64x4(out_strides), _i64x4(sizes), cosine, sine,
                table_row_stride, layout, dtype, table_dtype, stream)
    _check(name, status, error_type)
