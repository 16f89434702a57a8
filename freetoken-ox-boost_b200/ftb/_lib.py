"""ctypes binding of ``libftb.so`` (the sm_100a CUDA library; C ABI in ``include/ftb.h``).

The library is loaded from this package directory only. There is no fallback: if it is
missing or fails to load, every op raises ``FtbLibraryError``.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# FTB_LIBRARY names another build of the same library (same C ABI) to load instead.
LIB_PATH = os.environ.get("FTB_LIBRARY") or os.path.join(_HERE, "libftb.so")

FTB_OK = 0
FTB_ERR_SHAPE = 1
FTB_ERR_ALIGN = 2
FTB_ERR_WORKSPACE = 3
FTB_ERR_CUDA = 4
FTB_ERR_ARG = 5
FTB_ERR_TIMEOUT = 6
FTB_ERR_NOT_BUILT = 7

FTB_ROUTE_SOFTMAX = 0
FTB_ROUTE_SIGMOID = 1
FTB_ROUTE_SQRTSOFTPLUS = 2

STATUS_BAD_ID = 1
STATUS_F16_OVERFLOW = 2  # reserved: no longer raised (out-of-range rows of h are rescaled)
STATUS_TIMEOUT = 4

EP_HANDLE_BYTES = 64
PHASE_SHARED = 1   # FTB_PHASE_SHARED: this split-decode phase computes the shared expert
PHASE_COMBINE = 2  # FTB_PHASE_COMBINE: it ends with the combine of every route

# Every symbol include/ftb.h declares, with (restype, argtypes).
_vp, _i32, _i64, _f32, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t


class Nvfp4BankStruct(ctypes.Structure):
    """``ftb_nvfp4_bank``: device pointers of the six banks + the expert count."""
    _fields_ = [
        ("gate_up_packed", _vp),
        ("gate_up_scale", _vp),
        ("gate_up_global", _vp),
        ("down_packed", _vp),
        ("down_scale", _vp),
        ("down_global", _vp),
        ("num_experts", _i64),
    ]


_BP = ctypes.POINTER(Nvfp4BankStruct)

FTB_ACT_SILU = 0
FTB_ACT_SWIGLU_CLAMP = 1
FTB_ACT_SWIGLUOAI = 2
FTB_PATH_DECODE = 0
FTB_PATH_PREFILL = 1
FTB_PATH_PREFILL_FP4 = 2
FTB_HQUANT_NONE = 0
FTB_HQUANT_FP8_BLOCK128 = 1


class MoeArgsStruct(ctypes.Structure):
    """``ftb_moe_args``: one layer call (every option of the reference's drivers)."""
    _fields_ = [
        ("x", _vp), ("bank", _BP), ("shared", _BP), ("topk_w", _vp), ("topk_ids", _vp),
        ("T", _i64), ("H", _i32), ("I", _i32), ("top_k", _i32),
        ("activation", _i32), ("act_alpha", _f32), ("act_limit", _f32),
        ("weight_on_input", _i32), ("path", _i32), ("route_mask", _vp), ("phase", _i32),
        ("out", _vp), ("workspace", _vp), ("workspace_bytes", _sz),
        ("ic1", _vp), ("h", _vp), ("ic3", _vp), ("shared_ic1", _vp), ("shared_h", _vp),
        ("shared_out", _vp), ("h_quant", _i32),
    ]

SIGNATURES = {
    "ftb_status_string": (ctypes.c_char_p, [_i32]),
    "ftb_version": (_i32, []),
    "ftb_last_cuda_error": (ctypes.c_char_p, []),
    "ftb_route_topk": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _f32, _i32, _vp, _vp, _vp]),
    "ftb_route_ranked": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _f32, _i32, _vp, _vp, _vp, _vp,
                                _vp]),
    "ftb_router_gemv": (_i32, [_vp, _vp, _i64, _i32, _i32, _vp, _vp]),
    "ftb_moe_align_workspace_bytes": (_sz, [_i64, _i32, _i32]),
    "ftb_moe_align": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ftb_moe_decode_workspace_bytes": (_sz, [_i64, _i32, _i32, _i32, _i32, _i32]),
    "ftb_moe_decode": (_i32, [_vp, _BP, _BP, _vp, _vp, _i64, _i32, _i32, _i32, _f32, _vp, _vp,
                              _sz, _vp]),
    "ftb_moe_prefill_fp4_workspace_bytes": (_sz, [_i64, _i32, _i32, _i32, _i32, _i32]),
    "ftb_quant_nvfp4": (_i32, [_vp, _i32, _i64, _i32, _vp, _vp, _vp, _vp]),
    "ftb_moe_layer": (_i32, [ctypes.POINTER(MoeArgsStruct), _vp]),
    "ftb_moe_decode_plan": (_i32, [_i64, _i32, _i32, _i32, _i32, _i32, _vp]),
    "ftb_moe_decode_debug": (_i32, [_vp, _BP, _BP, _vp, _vp, _i64, _i32, _i32, _i32, _f32, _vp,
                                    _vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ftb_moe_combine": (_i32, [_vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp]),
    "ftb_moe_decode_phase": (_i32, [_vp, _BP, _BP, _vp, _vp, _vp, _i32, _i64, _i32, _i32, _i32,
                                    _f32, _vp, _vp, _sz, _vp]),
    "ftb_moe_prefill_workspace_bytes": (_sz, [_i64, _i32, _i32, _i32, _i32, _i32]),
    "ftb_moe_prefill": (_i32, [_vp, _BP, _BP, _vp, _vp, _i64, _i32, _i32, _i32, _f32, _vp, _vp,
                               _sz, _vp]),
    "ftb_moe_prefill_debug": (_i32, [_vp, _BP, _BP, _vp, _vp, _i64, _i32, _i32, _i32, _f32, _vp,
                                     _vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ftb_moe_decode_noalloc": (_i32, [_vp, _BP, _BP, _vp, _vp, _i64, _i32, _i32, _i32, _f32,
                                      _vp, _vp]),
    "ftb_ep_region_bytes": (_sz, [_i32, _i64, _i32, _i32]),
    "ftb_ep_create": (_i32, [_i32, _i32, _i64, _i32, _i32, _i32, _i32, _i32,
                             ctypes.POINTER(_vp)]),
    "ftb_ep_handle": (_i32, [_vp, _vp]),
    "ftb_ep_open": (_i32, [_vp, _vp]),
    "ftb_ep_set_wait_ns": (_i32, [_vp, _i64]),
    "ftb_ep_set_trace": (_i32, [_vp, _vp]),
    "ftb_ep_forward": (_i32, [_vp, _vp, _vp, _vp, _BP, _BP, _f32, _vp, _vp]),
    "ftb_ep_forward_act": (_i32, [_vp, _vp, _vp, _vp, _BP, _BP, _i32, _f32, _f32, _i32, _vp,
                                  _vp]),
    "ftb_ep_forward_tokens": (_i32, [_vp, _i64, _vp, _vp, _vp, _BP, _BP, _i32, _f32, _f32, _i32,
                                     _vp, _vp]),
    "ftb_ep_status": (_i32, [_vp, _i32, _vp]),
    "ftb_ep_destroy": (_i32, [_vp]),
    "ftb_profile_begin": (_i32, []),
    "ftb_profile_end": (_i32, [_vp, _vp, _i32]),
}

KERNEL_NAMES = {0: "sort_stage", 1: "gate_up_gemv", 2: "down_gemv", 3: "combine", 4: "route_topk",
                5: "ep_publish", 6: "ep_combine", 7: "permute_rows", 8: "quant_h"}


class FtbLibraryError(RuntimeError):
    pass


class FtbError(RuntimeError):
    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        super().__init__(f"{fn} failed: status {status} ({status_string(status)}){detail}")


_lock = threading.Lock()
_lib = None


def load(path: str = LIB_PATH):
    """Load libftb.so once; raise if it is absent (no CPU or Python fallback exists)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise FtbLibraryError(
                f"{path} is not built; build it with `make -C freetoken-ox-boost_b200/csrc` "
                "or `python -c 'import __graft_entry__ as g; g.build()'`")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def status_string(status: int) -> str:
    try:
        return load().ftb_status_string(int(status)).decode()
    except FtbLibraryError:
        return "?"


def check(fn: str, status: int) -> None:
    if status != FTB_OK:
        detail = ""
        if status == FTB_ERR_CUDA:
            detail = ": " + load().ftb_last_cuda_error().decode()
        raise FtbError(fn, status, detail)
