"""GPU parity of the libftb decode path against the CPU oracle (through the C ABI).

Tolerances (written here, from the north star): router ids and the permutation are
bit-exact; layer outputs and every bf16 intermediate are within max|d|/max|ref| <= 1e-2 of
the oracle (the GPU sums fp32 products in another order, so a few bf16 roundings flip).
"""
import numpy as np
import pytest
import torch

import ftb
from ftb import synth
from oracle import moe_oracle as m
from tests.moe_cases import build_case, compare, oracle_layer, to_f32

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda:0"


def run_gpu(case, limit=float("inf"), debug=True, activation=None):
    bank = case["bank"].to(DEV)
    sh = case["shared"].to(DEV) if case["shared"] is not None else None
    x = case["inp"].x.to(DEV)
    w = torch.from_numpy(case["w"]).to(DEV)
    ids = torch.from_numpy(case["ids"]).to(DEV)
    act = activation or ("silu" if limit == float("inf") else "swiglu_clamp")
    return ftb.moe_decode(x, bank, w, ids, activation=act, act_limit=limit, shared=sh,
                          debug=debug)


@pytest.mark.parametrize("T", [1, 3, 17])
def test_decode_small_with_shared(T):
    case = build_case(8, 256, 256, T, 2, seed=T)
    ref = oracle_layer(case)
    out, it = run_gpu(case)
    torch.cuda.synchronize()
    assert it["status"] == 0
    for name, key in [("ic1", "ic1"), ("h", "h"), ("ic3", "ic3"), ("shared_h", "shared_h"),
                      ("shared_out", "shared_out")]:
        rel, _ = compare(to_f32(it[key]), ref[key])
        assert rel <= TOL, f"{name}: {rel}"
    rel, frac = compare(to_f32(out), ref["out"])
    assert rel <= TOL and frac < 0.05, (rel, frac)


def test_decode_cfg0_full_router_gemv():
    """T=4, H=2048, I=768, 64 experts, top-8, router GEMV x.G^T."""
    case = build_case(64, 2048, 768, 4, 8, seed=0, shared=False, router_gemv=True)
    G = case["inp"].router_w.to(DEV)
    x = case["inp"].x.to(DEV)
    logits = ftb.router_logits(x, G)
    ref_logits = m.router_logits(case["inp"].x.float().numpy(), case["inp"].router_w.numpy())
    assert np.abs(to_f32(logits) - ref_logits).max() <= 1e-5 * np.abs(ref_logits).max()
    w, ids = ftb.fused_topk(x, logits, 8, True)
    ow, oids = m.topk_softmax(to_f32(logits), 8, True)
    assert np.array_equal(ids.cpu().numpy(), oids)
    assert np.abs(w.cpu().numpy() - ow).max() <= 1e-6
    case["ids"], case["w"] = oids, ow
    ref = oracle_layer(case)
    out, it = run_gpu(case)
    rel, frac = compare(to_f32(out), ref["out"])
    assert rel <= TOL and frac < 0.05, (rel, frac)
    f64 = m.moe_layer_f64(case["inp"].x.float().numpy(), case["bank"].numpy(), ow, oids)
    assert m.max_abs_rel(to_f32(out), f64) <= TOL


def test_decode_cfg0_t1_96_row_tiles():
    """Config 0 at T=1 (8 routes of 64 experts, 2I = 1536): the gate_up GEMV runs its 96-row
    work tiles (k_gemv_tma<0,1,6>); every intermediate against the oracle."""
    from ftb.fused_nvfp4 import decode_plan

    assert decode_plan(1, 2048, 768, 64, 8, False) == (96, 128)
    case = build_case(64, 2048, 768, 1, 8, seed=5, shared=False)
    ref = oracle_layer(case)
    out, it = run_gpu(case)
    torch.cuda.synchronize()
    assert it["status"] == 0
    for key in ("ic1", "h", "ic3"):
        rel, _ = compare(to_f32(it[key]), ref[key])
        assert rel <= TOL, (key, rel)
    rel, frac = compare(to_f32(out), ref["out"])
    assert rel <= TOL and frac < 0.05, (rel, frac)


def test_decode_swiglu_clamp():
    case = build_case(8, 256, 256, 5, 2, seed=7)
    ref = oracle_layer(case, limit=0.75)
    out, it = run_gpu(case, limit=0.75)
    assert compare(to_f32(it["h"]), ref["h"])[0] <= TOL
    assert compare(to_f32(out), ref["out"])[0] <= TOL


def test_decode_hot_expert_many_routes():
    """One expert hit by 40 routes (> 16, several route groups per tile)."""
    T, K, E = 40, 2, 8
    ids = np.stack([np.full(T, 3), np.arange(T) % E], 1).astype(np.int32)
    ids[:, 1] = np.where(ids[:, 1] == 3, 4, ids[:, 1])
    case = build_case(E, 256, 256, T, K, seed=5, ids=ids)
    ref = oracle_layer(case)
    out, _ = run_gpu(case)
    assert compare(to_f32(out), ref["out"])[0] <= TOL


def test_batch_invariance_bitwise():
    """A token's output bits do not depend on the rest of the batch."""
    case = build_case(8, 256, 256, 9, 2, seed=9)
    full, _ = run_gpu(case)
    sub = dict(case)
    sub["inp"] = synth.Inputs(case["inp"].x[2:5].clone(), case["inp"].logits[2:5].clone())
    sub["w"], sub["ids"] = case["w"][2:5], case["ids"][2:5]
    part, _ = run_gpu(sub)
    assert torch.equal(full[2:5].view(torch.int16), part.view(torch.int16))


def test_bad_ids_flagged_and_skipped():
    case = build_case(8, 256, 256, 3, 2, seed=4, shared=False)
    case["ids"] = case["ids"].copy()
    case["ids"][1, 1] = 99
    out, it = run_gpu(case)
    assert it["status"] & 1
    ok = case["ids"].copy()
    w = case["w"].copy()
    w[1, 1] = 0.0
    ok[1, 1] = 0
    ref = m.moe_layer(case["inp"].x.float().numpy(), case["bank"].numpy(), w, ok)
    assert compare(to_f32(out), ref["out"])[0] <= TOL


def test_empty_batch():
    case = build_case(8, 256, 256, 1, 2, seed=1)
    bank = case["bank"].to(DEV)
    x = torch.empty(0, 256, dtype=torch.bfloat16, device=DEV)
    out = ftb.moe_decode(x, bank, torch.empty(0, 2, device=DEV),
                         torch.empty(0, 2, dtype=torch.int32, device=DEV))
    assert out.shape == (0, 256)


def test_moe_align_matches_oracle():
    g = torch.Generator().manual_seed(3)
    T, K, E, bm = 300, 8, 64, 16
    ids = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
    sorted_ids, expert_ids, ntpp = ftb.moe_align_block_size(ids.to(DEV), bm, E)
    osorted, oexp, ontpp, _, _ = m.moe_align(ids.numpy(), E, bm)
    n = int(ntpp.item())
    assert n == ontpp
    assert np.array_equal(sorted_ids[:n].cpu().numpy(), osorted)
    assert np.array_equal(expert_ids[:n // bm].cpu().numpy(), oexp)
    assert bool((sorted_ids[n:] == T * K).all()) and bool((expert_ids[n // bm:] == -1).all())


def test_sigmoid_router_golden_on_gpu():
    import glob
    import os

    for path in sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden",
                                              "route_sigmoid_*.npz"))):
        d = np.load(path)
        lg = torch.from_numpy(d["logits"]).to(DEV)
        w, ids = ftb.fused_route(lg, torch.from_numpy(d["bias"]).to(DEV), int(d["top_k"]),
                                 bool(d["renorm"]), float(d["scaling"]))
        assert np.array_equal(ids.cpu().numpy(), d["ids"]), path
        ref = d["w"]
        got = w.cpu().numpy()
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(got), fin)
        assert np.abs(got[fin] - ref[fin]).max() <= 2e-6 * max(1.0, np.abs(ref[fin]).max())


def _golden(pattern):
    import glob
    import os

    return sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", pattern)))


@pytest.mark.parametrize("path", _golden("route_sqrtsoftplus_*.npz"))
def test_sqrtsoftplus_router_golden_on_gpu(path):
    d = np.load(path)
    w, ids = ftb.fused_route(torch.from_numpy(d["logits"]).to(DEV),
                             torch.from_numpy(d["bias"]).to(DEV), int(d["top_k"]),
                             bool(d["renorm"]), float(d["scaling"]), act="sqrtsoftplus")
    assert np.array_equal(ids.cpu().numpy(), d["ids"])
    got, ref = w.cpu().numpy(), d["w"]
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), fin)
    assert np.abs(got[fin] - ref[fin]).max(initial=0) <= 2e-6 * max(1.0, np.abs(ref[fin]).max())


@pytest.mark.parametrize("path", _golden("route_ranked_*.npz"))
def test_ranked_router_golden_on_gpu(path):
    d = np.load(path)
    w, ids, rid, rsc = ftb.fused_route_ranked(torch.from_numpy(d["logits"]).to(DEV),
                                              torch.from_numpy(d["bias"]).to(DEV),
                                              int(d["top_k"]), bool(d["renorm"]),
                                              float(d["scaling"]), n_rank=int(d["n_rank"]))
    assert np.array_equal(ids.cpu().numpy(), d["ids"])
    assert np.array_equal(rid.cpu().numpy(), d["rank_ids"])
    for got, ref in ((w.cpu().numpy(), d["w"]), (rsc.cpu().numpy(), d["rank_scores"])):
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(got), fin)
        assert np.abs(got[fin] - ref[fin]).max(initial=0) <= 2e-6 * max(1.0, np.abs(ref[fin]).max())


def test_softmax_router_ties_on_gpu():
    lg = torch.zeros(2, 256)
    lg[0, ::3] = 1.0
    lg[1] = torch.arange(256) % 7
    w, ids = ftb.fused_topk(None, lg.to(DEV), 8, True)
    ow, oids = m.topk_softmax(lg.numpy(), 8, True)
    assert np.array_equal(ids.cpu().numpy(), oids)
    assert np.abs(w.cpu().numpy() - ow).max() <= 1e-6
