"""ftb_moe_decode_noalloc: the decode layer for callers that cannot allocate device memory
(a runtime that owns every allocation, an FFI host without a device allocator, a process that
must not allocate after start-up). It takes its workspace from the library's own fixed
device scratch array instead of a caller buffer. This file is collected last on purpose.

The entry point is called through the C ABI on two calls in a row (different batch sizes,
so the second call runs on the first call's leftover scratch) and must match the existing
workspace entry point, ftb_moe_decode, within the parity tolerance used by the other tests.
"""
import ctypes

import pytest
import torch

import ftb
from ftb import _lib
from tests.moe_cases import build_case, compare, to_f32

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda:0"


def _noalloc(case, limit=float("inf")):
    bank = case["bank"].to(DEV)
    sh = case["shared"].to(DEV) if case["shared"] is not None else None
    x = case["inp"].x.to(DEV)
    w = torch.from_numpy(case["w"]).to(DEV)
    ids = torch.from_numpy(case["ids"]).to(DEV)
    T, H = x.shape
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    b = bank.struct()
    s = sh.struct() if sh is not None else None
    st = _lib.load().ftb_moe_decode_noalloc(
        ctypes.c_void_p(x.data_ptr()), ctypes.byref(b), ctypes.byref(s) if s is not None else None,
        ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(ids.data_ptr()), T, H, bank.inter,
        ids.shape[1], limit, ctypes.c_void_p(out.data_ptr()),
        torch.cuda.current_stream().cuda_stream)
    _lib.check("ftb_moe_decode_noalloc", st)
    # the existing entry point (caller workspace) on the same inputs
    ref = ftb.moe_decode(x, bank, w, ids, shared=sh, act_limit=limit)
    torch.cuda.synchronize()
    return out, ref


def test_noalloc_matches_workspace_entry_point_twice():
    first = build_case(8, 256, 256, 17, 2, seed=41)
    second = build_case(8, 256, 256, 3, 2, seed=42)
    for case in (first, second):
        out, ref = _noalloc(case)
        rel, _ = compare(to_f32(out), to_f32(ref))
        assert rel <= TOL, rel


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    b = _lib.Nvfp4BankStruct(16, 16, 16, 16, 16, 16, 256)
    # config-1 shape at T=4096 needs far more than the 16 MiB scratch
    st = lib.ftb_moe_decode_noalloc(None, ctypes.byref(b), None, None, None, 4096, 4096, 1536, 8,
                                    float("inf"), None, None)
    assert st == _lib.FTB_ERR_WORKSPACE
