"""GPU parity of the layer options the reference's drivers take beyond the default silu path,
and of activations beyond the f16 range of the tensor-core operand. Every case runs the
decode GEMVs and the tensor-core prefill against the CPU oracle.

* ``activation="swigluoai"`` with ``act_alpha`` / ``act_limit``
  (patches/moe_fused_nvfp4.patch:12-14, 47-48);
* ``apply_router_weight_on_input=True``: the routed weight scales ic1 instead of ic3
  (patches/moe_fused_nvfp4.patch:138,145; experts_resident.py:72-83);
* a token whose activation h reaches |h| ~ 1e6: the reference keeps h in bf16
  (kernel_triton_dsv4_fused_moe.patch:22-36); the kernels' f16 operand rows are rescaled by a
  power of two inside the call, so the result matches with status 0.
Tolerance: max|d| / max|ref| <= 1e-2 per compared tensor (north star).
"""
import numpy as np
import pytest
import torch

import ftb
from ftb import synth
from tests.moe_cases import build_case, compare, oracle_layer, to_f32

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda:0"
PATHS = {"decode": ftb.moe_decode, "prefill": ftb.moe_prefill}


def _run(path, case, **kw):
    bank = case["bank"].to(DEV)
    sh = case["shared"].to(DEV) if case["shared"] is not None else None
    x = case["inp"].x.to(DEV)
    w = torch.from_numpy(case["w"]).to(DEV)
    ids = torch.from_numpy(case["ids"]).to(DEV)
    out, it = PATHS[path](x, bank, w, ids, shared=sh, debug=True, **kw)
    torch.cuda.synchronize()
    return out, it


def _check(out, it, ref, names=("ic1", "h", "ic3")):
    assert it["status"] == 0, it["status"]
    for name in names:
        rel, _ = compare(to_f32(it[name]), ref[name])
        assert rel <= TOL, (name, rel)
    rel, _ = compare(to_f32(out), ref["out"])
    assert rel <= TOL, ("out", rel)


@pytest.mark.parametrize("path", ["decode", "prefill"])
@pytest.mark.parametrize("alpha,limit", [(1.702, 7.0), (1.0, 0.8)])
def test_swigluoai(path, alpha, limit):
    case = build_case(8, 256, 256, 24, 2, seed=61)
    ref = oracle_layer(case, limit, act="swigluoai", alpha=alpha)
    out, it = _run(path, case, activation="swigluoai", act_alpha=alpha, act_limit=limit)
    _check(out, it, ref, ("ic1", "h", "ic3", "shared_h", "shared_out"))


@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_router_weight_on_input(path):
    case = build_case(8, 256, 256, 20, 2, seed=62)
    ref = oracle_layer(case, w_on_input=True)
    out, it = _run(path, case, apply_router_weight_on_input=True)
    _check(out, it, ref, ("ic1", "h", "ic3", "shared_h", "shared_out"))
    # it differs from the default placement of the weight (ic1 carries it now)
    plain = oracle_layer(case)
    assert compare(to_f32(it["ic1"]), plain["ic1"])[0] > 0.05


def _big_token_case(T, hot, scale, seed, shared=True):
    case = build_case(8, 256, 256, T, 2, seed=seed, shared=shared)
    x = case["inp"].x.clone()
    x[hot] = (x[hot].float() * scale).to(torch.bfloat16)  # power of two: exact in bf16
    case["inp"] = synth.Inputs(x, case["inp"].logits)
    return case


@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_h_beyond_f16_range_one_token(path):
    """One token at 4096x scale: its routes' h reaches ~1e6 (far beyond f16's 65504)."""
    case = _big_token_case(9, [4], 4096.0, 63)
    ref = oracle_layer(case)
    assert np.abs(ref["h"][4]).max() > 1e5 and np.abs(ref["shared_h"][4]).max() > 1e5
    out, it = _run(path, case)
    _check(out, it, ref, ("ic1", "h", "ic3", "shared_h", "shared_out"))
    # the other tokens' outputs are unaffected (compare them on their own scale)
    keep = [t for t in range(9) if t != 4]
    rel, _ = compare(to_f32(out)[keep], ref["out"][keep])
    assert rel <= TOL, rel


@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_h_beyond_f16_range_many_rows(path):
    """Every token large (all rows rescaled, one clamp-free and one clamped activation);
    each token compared on its own scale."""
    case = _big_token_case(40, list(range(40)), 2048.0, 64)
    ref = oracle_layer(case)
    out, it = _run(path, case)
    assert it["status"] == 0
    got = to_f32(out)
    for t in range(40):
        rel, _ = compare(got[t], ref["out"][t])
        assert rel <= TOL, (t, rel)
    # swiglu_clamp keeps h small: nothing to rescale, still exact
    ref_c = oracle_layer(case, 7.0)
    out_c, it_c = _run(path, case, activation="swiglu_clamp", act_limit=7.0)
    _check(out_c, it_c, ref_c)


def test_h_rescale_in_split_decode():
    """The split (hit/miss) decode over a large token equals the single-phase decode."""
    E, H, I, K, T = 16, 256, 256, 4, 6
    bank = synth.make_bank(E, H, I, seed=5, device=DEV)
    inp = synth.make_inputs(T, H, E, seed=9, device=DEV)
    x = inp.x.clone()
    x[2] = (x[2].float() * 4096.0).to(torch.bfloat16)
    w, ids = ftb.fused_topk(x, inp.logits, K, True)
    ref = ftb.moe_decode(x, bank, w, ids)
    miss = torch.zeros(T, K, dtype=torch.bool, device=DEV)
    miss[2, ::2] = True
    miss[4, 1] = True
    out = ftb.fused_experts_decode_nvfp4_split(x, *bank.tensors(), w, ids, miss, None)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
