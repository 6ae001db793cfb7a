"""ctypes binding of include/glt_graft.h.

Loads the in-tree ``libglt_b200.so``.  There is no fallback: if the library
is missing the import fails loudly (build it with ``python -m glt_b200.build``).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libglt_b200.so")

GLT_OK = 0
STATUS_NAMES = {
    0: "GLT_OK", 1: "GLT_EINVAL", 2: "GLT_ECUDA", 3: "GLT_ENCCL", 4: "GLT_EIO",
    5: "GLT_ETIMEOUT", 6: "GLT_ESTATE", 7: "GLT_ENOMEM",
}


class GltError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} not found: the CUDA library is required (python -m glt_b200.build)"
        )
    return C.CDLL(LIB_PATH)


lib = _load()

_vp, _i32, _i64, _f32, _u32 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint

# (name, restype, argtypes) for every exported symbol; tests check that each
# declaration of include/glt_graft.h appears here and in the library.
SIGNATURES: dict[str, tuple] = {
    "glt_last_error": (C.c_char_p, []),
    "glt_version": (C.c_char_p, []),
    "glt_device_error": (_i32, [C.POINTER(_u32)]),
    "glt_gemm": (_i32, [_vp, _i64, _i32, _vp, _i64, _i32, _vp, _i64, _i32,
                        _i32, _i32, _i32, _f32, _f32, _vp]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def last_error() -> str:
    return lib.glt_last_error().decode(errors="replace")


def check(status: int) -> None:
    if status != GLT_OK:
        raise GltError(status, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib, name)(*args))
