"""GPU parity of the tensor-core prefill path (ftb_moe_prefill).

Small shapes against the CPU oracle (every bf16 intermediate and the output): routes per
expert from a handful to > 256, so experts span one or two segments and the MMA's N ranges
from 16 to 256. BASELINE config 2 (T=4096, H=4096, I=1536, 256 experts, top-8, shared
expert) against the torch fp32 restatement of the oracle's arithmetic (the numpy oracle
takes minutes at that size). Tolerance: max|d| / max|ref| <= 1e-2 (north star).
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


def run_prefill(case, debug=True):
    bank = case["bank"].to(DEV)
    sh = case["shared"].to(DEV) if case["shared"] is not None else None
    x = case["inp"].x.to(DEV)
    w = torch.from_numpy(case["w"]).to(DEV)
    ids = torch.from_numpy(case["ids"]).to(DEV)
    return ftb.moe_prefill(x, bank, w, ids, shared=sh, debug=debug)


@pytest.mark.parametrize("E,T,K", [(8, 64, 2), (4, 300, 2), (4, 600, 2)])
def test_prefill_small_vs_oracle(E, T, K):
    case = build_case(E, 256, 256, T, K, seed=E * 1000 + T)
    ref = oracle_layer(case)
    out, it = run_prefill(case)
    torch.cuda.synchronize()
    assert it["status"] == 0
    for name in ("ic1", "h", "ic3", "shared_h", "shared_out"):
        rel, _ = compare(to_f32(it[name]), ref[name])
        assert rel <= TOL, (name, rel)
    rel, _ = compare(to_f32(out), ref["out"])
    assert rel <= TOL, rel
    counts = np.bincount(case["ids"].reshape(-1), minlength=E)
    if T == 600:
        assert counts.max() > 256  # an expert spans two segments


def test_prefill_matches_decode_closely():
    """The two paths sum the same exact products in different orders."""
    case = build_case(8, 512, 256, 96, 2, seed=77)
    bank = case["bank"].to(DEV)
    sh = case["shared"].to(DEV)
    x = case["inp"].x.to(DEV)
    w = torch.from_numpy(case["w"]).to(DEV)
    ids = torch.from_numpy(case["ids"]).to(DEV)
    a = ftb.moe_prefill(x, bank, w, ids, shared=sh)
    b = ftb.moe_decode(x, bank, w, ids, shared=sh)
    torch.cuda.synchronize()
    rel = float((a.float() - b.float()).abs().max() / b.float().abs().max())
    assert rel <= TOL


def test_config2_prefill_vs_fp32_restatement():
    from tests.test_gpu_decode_large import _max_abs_rel, _reference

    import tests.test_gpu_decode_large as big
    E, H, I, K, T = big.E, big.H, big.I, big.K, 4096
    bank = synth.make_bank(E, H, I, seed=31, device=DEV)
    shared = synth.make_shared(H, I, seed=31, device=DEV)
    inp = synth.make_inputs(T, H, E, seed=31, device=DEV)
    w, ids = ftb.fused_topk(inp.x, inp.logits, K, True)
    out, it = ftb.moe_prefill(inp.x, bank, w, ids, shared=shared, debug=True)
    ref = _reference(inp.x, bank, shared, w, ids)
    torch.cuda.synchronize()
    assert it["status"] == 0
    for name in ("ic1", "h", "ic3", "shared_h", "shared_out"):
        assert _max_abs_rel(it[name], ref[name]) <= TOL, name
    assert _max_abs_rel(out, ref["out"]) <= TOL
