"""Loading of the two in-tree native artefacts.

``lib()`` returns the C ABI (``libfa_sm100.so``) through ctypes, with every
function of ``include/fa_sm100.h`` typed.  ``ext()`` imports the PyTorch
extension module ``flash_attention_cuda``.  Neither has a fallback: if an
artefact is missing the call raises, naming the build command.
"""

from __future__ import annotations

import ctypes
import importlib.util
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libfa_sm100.so"
EXT_PATH = PKG / "flash_attention_cuda.so"

# Every exported symbol declared in include/fa_sm100.h: name -> (restype, argtypes)
_i64, _vp, _int, _f32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_float
ABI = {
    "fa_fwd_sm100": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _f32, _vp]),
    "fa_fwd_sm100_varlen": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _f32, _vp]),
    "fa_fwd_sm100_noalloc": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _f32, _vp]),
    "fa_fwd_sm100_lse": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _f32, _vp]),
    "fa_bwd_sm100_varlen": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                   _i64, _int, _f32, _vp]),
    "fa_bwd_sm100": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int,
                            _f32, _vp]),
    "fa_last_error": (ctypes.c_char_p, []),
    "fa_read_status": (_int, [_vp, ctypes.POINTER(ctypes.c_uint), _int]),
    "fa_set_wait_limit_ns": (None, [ctypes.c_ulonglong]),
    "fa_selftest_wait_timeout": (_int, [ctypes.c_ulonglong, _vp]),
    "fa_smem_bytes": (_int, []),
    "fa_fwd_sm100_debug": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _f32, _vp, _vp]),
    "fa_set_max_splits": (None, [_int]),
    "fa_release_workspaces": (_int, []),
}

_lib = None
_ext = None

_BUILD_HINT = "build it with `python -m flash_attention_2_lab_b200.build`"


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing; {_BUILD_HINT}")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in ABI.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def ext():
    global _ext
    if _ext is None:
        if not EXT_PATH.exists():
            raise ImportError(f"{EXT_PATH} is missing; {_BUILD_HINT}")
        import torch  # noqa: F401  (loads libtorch / libc10 before the extension)

        name = "flash_attention_cuda"
        if name in sys.modules and getattr(sys.modules[name], "__file__", None) == str(EXT_PATH):
            _ext = sys.modules[name]
        else:
            spec = importlib.util.spec_from_file_location(name, EXT_PATH)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            sys.modules[name] = mod
            _ext = mod
    return _ext


def last_error() -> str:
    return lib().fa_last_error().decode(errors="replace")


def check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(f"fa_sm100 call failed ({rc}): {last_error()}")
