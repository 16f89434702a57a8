"""ftb_moe_decode_noalloc: the decode layer for callers that cannot allocate device memory.

Who needs it: code that runs inside a runtime owning every device allocation (a serving
engine's caching allocator that this call site cannot reach), a foreign-language host (Go,
Java, Rust over FFI) with no device-allocator binding, or a process that must not allocate
after start-up (allocation can fail, fragment memory or synchronise the device). Such callers
cannot pass the workspace ftb_moe_decode() asks for, so this entry point takes it from the
library's own fixed device scratch array.

The test calls it through the C ABI on two calls in a row (different shapes, so the second
call runs on the first call's leftover scratch) and requires outputs bit-identical to the
workspace entry point, ftb_moe_decode, which runs the same kernels on the same inputs. This
file is collected last on purpose; it passes alone in a fresh process and after the others.
"""
import ctypes

import pytest
import torch

import ftb
from ftb import _lib
from tests.moe_cases import build_case

pytestmark = pytest.mark.gpu
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
    cases = [build_case(8, 256, 256, 17, 2, seed=41),         # shared expert, 128-row tiles
             build_case(64, 2048, 768, 1, 8, seed=42, shared=False)]  # config 0, 96-row tiles
    for case in cases:
        out, ref = _noalloc(case)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    b = _lib.Nvfp4BankStruct(16, 16, 16, 16, 16, 16, 256)
    # config-1 shape at T=4096 needs far more than the 16 MiB scratch
    st = lib.ftb_moe_decode_noalloc(None, ctypes.byref(b), None, None, None, 4096, 4096, 1536, 8,
                                    float("inf"), None, None)
    assert st == _lib.FTB_ERR_WORKSPACE
