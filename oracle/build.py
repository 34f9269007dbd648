"""Builds and loads the C part of the oracle (TEST INFRASTRUCTURE ONLY)."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
LIB = ORACLE / "_build" / "liboracle.so"
_lib = None


def build() -> Path:
    src = ORACLE / "c" / "fp8_e4m3.c"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ORACLE)], check=True)
    return LIB


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIB))
        lib.oracle_float_to_e4m3.restype = ctypes.c_uint8
        lib.oracle_float_to_e4m3.argtypes = [ctypes.c_float]
        lib.oracle_e4m3_to_float.restype = ctypes.c_float
        lib.oracle_e4m3_to_float.argtypes = [ctypes.c_uint8]
        lib.oracle_quantize_rows.restype = None
        lib.oracle_quantize_rows.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_void_p, ctypes.c_void_p]
        _lib = lib
    return _lib
