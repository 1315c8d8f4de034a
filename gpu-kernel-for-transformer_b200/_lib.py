"""ctypes binding of the C-ABI library ``lib/libtfx_b200.so`` (include/tfx.h).

The library is the product: every op of the forward is a hand-written
sm_100a kernel behind an ``extern "C"`` entry point. This module only loads
it, declares the signatures, and maps status codes to Python exceptions with
the reference wrappers' conventions: shape/argument problems raise
``ValueError`` (triton_fused_norm.py:149-155, triton_fused_ffn.py:230-241),
everything else ``RuntimeError``. There is no fallback: if the library is
missing, every op raises.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

PKG_DIR = pathlib.Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "lib" / "libtfx_b200.so"

TFX_OK = 0
TFX_ERR_INVALID_ARGUMENT = -1
TFX_ERR_UNSUPPORTED = -2
TFX_ERR_MISALIGNED = -3
TFX_ERR_WORKSPACE = -4
TFX_ERR_CUDA = -5
TFX_ERR_DEVICE = -6

TFX_DTYPE_F16 = 0
TFX_DTYPE_F32 = 1

TFX_DEV_TIMEOUT_FULL = 1
TFX_DEV_TIMEOUT_EMPTY = 2
TFX_DEV_TIMEOUT_ACCUM = 3
TFX_DEV_TIMEOUT_ACCUM_FREE = 4
TFX_DEV_TIMEOUT_OTHER = 5

TFX_PATH_AUTO = 0
TFX_PATH_CHAIN = 1

TFX_EPI_BIAS = 0
TFX_EPI_BIAS_GELU = 1
TFX_EPI_BIAS_RESIDUAL = 2

# Every symbol include/tfx.h declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
SIGNATURES = {
    "tfx_version": (_I, []),
    "tfx_status_string": (ctypes.c_char_p, [_I]),
    "tfx_last_error_message": (ctypes.c_char_p, []),
    "tfx_layer_norm": (_I, [_P, _P, _P, _P, _I, _I64, _I, _F, _I, _P]),
    "tfx_residual_layer_norm": (_I, [_P, _P, _P, _P, _P, _P, _I, _I64, _I, _F, _I, _P]),
    "tfx_linear": (_I, [_P, _P, _P, _P, _P, _I64, _I, _I, _I, _P]),
    "tfx_attention": (_I, [_P, _P, _P, _I64, _P, _I64, _I, _I, _I, _I, _F, _I, _P, _P]),
    "tfx_attention_masked": (_I, [_P, _P, _P, _I64, _P, _I64, _I, _I, _I, _I, _F, _I, _P, _P]),
    "tfx_attention_vt_ld": (_I64, [_I]),
    "tfx_transpose_v": (_I, [_P, _I64, _P, _I, _I, _I, _P]),
    "tfx_attention_vt": (_I, [_P, _P, _P, _I64, _P, _I64, _I, _I, _I, _I, _F, _I, _P, _P]),
    "tfx_forward_workspace_bytes": (_I64, [_P, _I, _I]),
    "tfx_forward": (_I, [_P, _P, _P, _I, _I, _P, _P, ctypes.c_size_t, _P]),
    "tfx_forward_masked": (_I, [_P, _P, _P, _I, _I, _P, _P, ctypes.c_size_t, _P]),
    "tfx_forward_static": (_I, [_P, _P, _P, _I, _I, _P, _P]),
    "tfx_forward_kv_workspace_bytes": (_I64, [_P, _I, _I]),
    "tfx_forward_kv": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, ctypes.c_size_t, _P]),
    "tfx_read_device_error": (_I, [ctypes.POINTER(_I)]),
    "tfx_selftest_bounded_wait": (_I, [_I64, _P]),
}


class TfxLayer(ctypes.Structure):
    """Mirror of ``tfx_layer`` (include/tfx.h)."""

    _fields_ = [
        (name, ctypes.c_void_p)
        for name in (
            "norm1_weight", "norm1_bias", "qkv_weight", "qkv_bias", "out_weight", "out_bias",
            "norm2_weight", "norm2_bias", "ffn_in_weight", "ffn_in_bias", "ffn_out_weight",
            "ffn_out_bias",
        )
    ]


class TfxModel(ctypes.Structure):
    """Mirror of ``tfx_model`` (include/tfx.h)."""

    _fields_ = [
        ("d_model", ctypes.c_int),
        ("num_heads", ctypes.c_int),
        ("ffn_dim", ctypes.c_int),
        ("num_layers", ctypes.c_int),
        ("causal", ctypes.c_int),
        ("eps", ctypes.c_float),
        ("layers", ctypes.POINTER(TfxLayer)),
        ("final_norm_weight", ctypes.c_void_p),
        ("final_norm_bias", ctypes.c_void_p),
        ("path", ctypes.c_int),
    ]


_lib = None
_lock = threading.Lock()


class LibraryNotBuilt(RuntimeError):
    pass


def load(path: pathlib.Path | str | None = None) -> ctypes.CDLL:
    """Load the library once (RTLD_LOCAL) and declare its signatures."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = pathlib.Path(path) if path else LIB_PATH
        if not p.exists():
            raise LibraryNotBuilt(
                f"{p} is missing: build it with `python {PKG_DIR.name}/build.py` "
                "(this package has no CPU or PyTorch fallback)"
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(status: int, what: str) -> None:
    """Raise the reference-style exception for a non-zero status."""
    if status == TFX_OK:
        return
    lib = load()
    detail = lib.tfx_last_error_message().decode(errors="replace")
    kind = lib.tfx_status_string(status).decode(errors="replace")
    msg = f"{what}: {kind}" + (f" ({detail})" if detail else "")
    if status in (TFX_ERR_INVALID_ARGUMENT, TFX_ERR_UNSUPPORTED, TFX_ERR_MISALIGNED,
                  TFX_ERR_WORKSPACE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def read_device_error() -> int:
    """Read-and-clear the current device's kernel timeout word (synchronises)."""
    code = ctypes.c_int(0)
    check(load().tfx_read_device_error(ctypes.byref(code)), "tfx_read_device_error")
    return code.value
