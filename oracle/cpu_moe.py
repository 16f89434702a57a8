"""ctypes binding of oracle/build/libcpumoe.so (cpu_moe.cpp): TEST INFRASTRUCTURE.

The C++ CPU restatement of the layer: a second checker for the numpy oracle and the CPU
baseline bench.py times on the host cores. Build: ``make -C oracle``.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "build", "libcpumoe.so")
_lib = None


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run `make -C oracle`")
        lib = ctypes.CDLL(LIB_PATH)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        lib.cpu_moe_layer.restype = i32
        lib.cpu_moe_layer.argtypes = [vp, i64, i32, i32] + [vp] * 6 + [i32] + [vp] * 6 + \
            [vp, vp, i32, f32, i32, vp]
        lib.cpu_moe_max_threads.restype = i32
        lib.cpu_moe_has_avx512.restype = i32
        _lib = lib
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _bank_arrays(bank: dict):
    names = ("gate_up_packed", "gate_up_scale", "gate_up_global", "down_packed", "down_scale",
             "down_global")
    out = []
    for n in names:
        a = np.ascontiguousarray(bank[n])
        if a.dtype == np.float16:
            a = a.view(np.uint16)
        out.append(a)
    return out


def moe_layer(x_bits: np.ndarray, bank: dict, topk_w: np.ndarray, topk_ids: np.ndarray,
              shared: dict | None = None, limit: float = float("inf"), nthreads: int = 0):
    """x_bits: uint16 bf16 bits [T, H]; bank/shared: dicts of numpy arrays (Nvfp4Bank.numpy());
    returns uint16 bf16 bits [T, H]."""
    lib = load()
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    T, H = x_bits.shape
    b = _bank_arrays(bank)
    E, I = b[0].shape[0], b[0].shape[1] // 2
    s = _bank_arrays(shared) if shared is not None else [None] * 6
    w = np.ascontiguousarray(topk_w, dtype=np.float32)
    ids = np.ascontiguousarray(topk_ids, dtype=np.int32)
    out = np.empty((T, H), np.uint16)
    st = lib.cpu_moe_layer(_p(x_bits), T, H, I, *[_p(a) for a in b], E, *[_p(a) for a in s],
                           _p(w), _p(ids), ids.shape[1] if ids.ndim == 2 else 1, float(limit),
                           int(nthreads), _p(out))
    if st != 0:
        raise ValueError(f"cpu_moe_layer failed ({st})")
    return out


def max_threads() -> int:
    return int(load().cpu_moe_max_threads())


def has_avx512() -> bool:
    return bool(load().cpu_moe_has_avx512())
