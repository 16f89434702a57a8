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
    # flags, ids, w, staged rows (f16) and their scales for W*T slots, own route outputs
    want = 256 + 256 + T * K * 4 + T * K * 4 + W * T * H * 2 + 512 + T * K * H * 2
    assert lib.ftb_ep_region_bytes(W, T, H, K) == want
    h = ctypes.c_void_p()
    assert lib.ftb_ep_create(0, 9, T, H, 1536, 256, K, 1, ctypes.byref(h)) == _lib.FTB_ERR_ARG
    assert lib.ftb_ep_create(2, 2, T, H, 1536, 256, K, 1, ctypes.byref(h)) == _lib.FTB_ERR_ARG
    assert lib.ftb_ep_create(0, 3, T, H, 1536, 256, K, 1, ctypes.byref(h)) == _lib.FTB_ERR_SHAPE
    assert lib.ftb_ep_create(0, 2, T, 100, 1536, 256, K, 1, ctypes.byref(h)) == _lib.FTB_ERR_SHAPE
    assert not h.value
    assert lib.ftb_ep_destroy(None) == _lib.FTB_OK
    assert lib.ftb_ep_forward(None, None, None, None, None, None, 0.0, None, None) == _lib.FTB_ERR_ARG


def _plan(T, H, I, E, K, shared):
    import ctypes

    plan = (ctypes.c_int32 * 2)()
    st = _lib.load().ftb_moe_decode_plan(T, H, I, E, K, 1 if shared else 0, plan)
    return st, (plan[0], plan[1])


def test_smoke_shape_is_accepted_by_the_library():
    """__graft_entry__.smoke() calls the decode layer at SMOKE_SHAPE: the library's host-side
    shape rules (the same check ftb_moe_decode applies) must accept it."""
    import __graft_entry__ as g

    S = g.SMOKE_SHAPE
    st, plan = _plan(S["T"], S["H"], S["I"], S["E"], S["K"], S["shared"])
    assert st == _lib.FTB_OK, _lib.status_string(st)
    assert plan[0] in (96, 128) and plan[1] == 128


@pytest.mark.parametrize("T,want", [(1, (96, 128)), (4, (128, 128)), (16, (128, 128)),
                                    (64, (128, 128))])
def test_decode_plan_config1(T, want):
    """Tile rows of the config-1 decode (H4096 I1536 E256 top-8 + shared) on 148 SMs: the
    GPU parity tests at these T assert the same plan, so each launched variant is tested."""
    st, plan = _plan(T, 4096, 1536, 256, 8, True)
    assert st == _lib.FTB_OK and plan == want


def test_decode_plan_config0_t1_uses_96_row_tiles():
    st, plan = _plan(1, 2048, 768, 64, 8, False)
    assert st == _lib.FTB_OK and plan == (96, 128)


def test_decode_plan_rejects_what_decode_rejects():
    assert _plan(4, 256, 128, 8, 2, True)[0] == _lib.FTB_ERR_SHAPE
    assert _plan(4, 256, 256, 8, 33, True)[0] == _lib.FTB_ERR_SHAPE
    assert _plan(4, 256, 256, 2048, 8, True)[0] == _lib.FTB_ERR_SHAPE


# Largest config-1 token count (with a shared expert) whose decode workspace fits the
# allocation-free entry point's 16 MiB scratch.
NOALLOC_MAX_T_CONFIG1 = 122


def test_noalloc_scratch_limit_host_only():
    """The allocation-free decode uses a 16 MiB static scratch: at the config-1 shape with a
    shared expert it fits up to NOALLOC_MAX_T_CONFIG1 tokens (the figure include/ftb.h states)
    and not one more; bigger calls, and shapes the layer rejects, are refused on the host
    before any device call."""
    import ctypes

    lib = _lib.load()
    limit = 16 << 20
    fits = [T for T in range(1, 400)
            if lib.ftb_moe_decode_workspace_bytes(T, 4096, 1536, 256, 8, 1) <= limit]
    assert max(fits) == NOALLOC_MAX_T_CONFIG1
    header = open(os.path.join(ROOT, "include", "ftb.h")).read()
    assert f"T <= {NOALLOC_MAX_T_CONFIG1})" in header
    b = _lib.Nvfp4BankStruct(16, 16, 16, 16, 16, 16, 256)
    inf = float("inf")
    sh = _lib.Nvfp4BankStruct(16, 16, 16, 16, 16, 16, 1)
    assert lib.ftb_moe_decode_noalloc(None, ctypes.byref(b), ctypes.byref(sh), None, None,
                                      NOALLOC_MAX_T_CONFIG1 + 1, 4096, 1536, 8, inf, None,
                                      None) == _lib.FTB_ERR_WORKSPACE
    assert lib.ftb_moe_decode_noalloc(None, ctypes.byref(b), None, None, None, 4, 4096, 1536,
                                      33, inf, None, None) == _lib.FTB_ERR_SHAPE
    assert lib.ftb_moe_decode_noalloc(None, ctypes.byref(b), None, None, None, 1 << 40, 4096,
                                      1536, 8, inf, None, None) == _lib.FTB_ERR_SHAPE
    big = _lib.Nvfp4BankStruct(16, 16, 16, 16, 16, 16, 4096)
    assert lib.ftb_moe_decode_noalloc(None, ctypes.byref(big), None, None, None, 4, 4096, 1536,
                                      8, inf, None, None) == _lib.FTB_ERR_SHAPE
