"""The C ABI library: it loads without a GPU, exports every symbol include/ftb.h declares,
and its host-only queries answer (no kernel is launched here)."""
import os
import re

import pytest

from ftb import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"^FTB_API\s+[\w\s\*]+?\b(ftb_\w+)\s*\(", text, re.M))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "ftb_moe_decode" in names and "ftb_route_topk" in names and len(names) >= 10


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports_symbol(name):
    lib = _lib.load()
    assert hasattr(lib, name)
    assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.ftb_version() >= 1
    for s in range(8):
        assert lib.ftb_status_string(s)
    assert lib.ftb_status_string(0) == b"ok"


def test_workspace_queries_host_only():
    lib = _lib.load()
    small = lib.ftb_moe_decode_workspace_bytes(4, 2048, 768, 64, 8, 0)
    big = lib.ftb_moe_decode_workspace_bytes(64, 4096, 1536, 256, 8, 1)
    assert 0 < small < big
    assert small % 256 == 0 and big % 256 == 0
    assert lib.ftb_moe_align_workspace_bytes(4096, 8, 256) >= 4096 * 8 * 4


def test_bad_shapes_rejected_before_any_launch():
    lib = _lib.load()
    # top_k > 32 and E > 1024 are rejected on the host
    assert lib.ftb_route_topk(None, 4, 64, 33, 0, None, 1.0, 1, None, None, None) == _lib.FTB_ERR_SHAPE
    assert lib.ftb_route_topk(None, 4, 2048, 8, 0, None, 1.0, 1, None, None, None) == _lib.FTB_ERR_SHAPE
    assert lib.ftb_route_topk(None, 4, 64, 8, 7, None, 1.0, 1, None, None, None) == _lib.FTB_ERR_ARG
    # H and I must be multiples of 256 (TMA row strides of the scale banks)
    b = _lib.Nvfp4BankStruct(16, 16, 16, 16, 16, 16, 8)
    import ctypes
    for h, i in ((100, 256), (384, 256), (256, 128), (256, 384)):
        st = lib.ftb_moe_decode(None, ctypes.byref(b), None, None, None, 4, h, i, 2, 1.0, None,
                                None, 0, None)
        assert st == _lib.FTB_ERR_SHAPE, (h, i)
    # T == 0 is a no-op
    st = lib.ftb_moe_decode(None, ctypes.byref(b), None, None, None, 0, 256, 256, 2, 1.0, None,
                            None, 0, None)
    assert st == _lib.FTB_OK


def test_ep_host_checks():
    """Expert-parallel group: region size is a host-only query, and bad group arguments are
    rejected before any device call."""
    import ctypes

    lib = _lib.load()
    T, H, K, W = 64, 4096, 8, 2
    want = 256 + 256 + T * H * 2 + T * K * 4 + T * K * 4 + W * T * K * H * 2
    assert lib.ftb_ep_region_bytes(W, T, H, K) == want
    h = ctypes.c_void_p()
    assert lib.ftb_ep_create(0, 9, T, H, 1536, 256, K, 1, ctypes.byref(h)) == _lib.FTB_ERR_ARG
    assert lib.ftb_ep_create(2, 2, T, H, 1536, 256, K, 1, ctypes.byref(h)) == _lib.FTB_ERR_ARG
    assert lib.ftb_ep_create(0, 3, T, H, 1536, 256, K, 1, ctypes.byref(h)) == _lib.FTB_ERR_SHAPE
    assert lib.ftb_ep_create(0, 2, T, 100, 1536, 256, K, 1, ctypes.byref(h)) == _lib.FTB_ERR_SHAPE
    assert not h.value
    assert lib.ftb_ep_destroy(None) == _lib.FTB_OK
    assert lib.ftb_ep_forward(None, None, None, None, None, None, 0.0, None, None) == _lib.FTB_ERR_ARG
