"""Decode GEMVs whose segments hold many routes: the activation rows of a segment are loaded by
TMA boxes (gate_up from the x rows gathered into segment order when the call expects >= 12
routes per distinct expert, down from h from 4), for every segment of the launch, the small
ones included. Against the oracle (oracle/moe_oracle.py) with the
north star's tolerance, max|d| / max|ref| <= 1e-2, for every intermediate and the output;
and bit for bit against the same routes computed one token at a time (T = 1: one route per
segment, per-route copies only), since a route's result does not depend on its segment.
"""
import numpy as np
import pytest
import torch

import ftb
from tests.moe_cases import build_case, compare, oracle_layer, to_f32

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda:0"


@pytest.mark.parametrize("E,H,I,T,K", [(16, 1024, 512, 64, 8), (24, 512, 1024, 48, 6)])
def test_boxed_segments_match_oracle(E, H, I, T, K):
    from ftb.fused_nvfp4 import decode_plan

    case = build_case(E, H, I, T, K, seed=60 + E)
    assert decode_plan(T, H, I, E, K, True) == (128, 128)
    counts = np.bincount(case["ids"].ravel(), minlength=E)
    assert (counts >= 6).any()  # boxed segments (and the shared expert's 16-route segments)
    bank = case["bank"].to(DEV)
    sh = case["shared"].to(DEV)
    x = case["inp"].x.to(DEV)
    w = torch.from_numpy(case["w"]).to(DEV)
    ids = torch.from_numpy(case["ids"]).to(DEV)
    out, it = ftb.moe_decode(x, bank, w, ids, shared=sh, debug=True)
    torch.cuda.synchronize()
    assert it["status"] == 0
    ref = oracle_layer(case)
    for name in ("ic1", "h", "ic3", "shared_ic1", "shared_h", "shared_out"):
        rel, _ = compare(to_f32(it[name]), ref[name])
        assert rel <= TOL, (name, rel)
    assert compare(to_f32(out), ref["out"])[0] <= TOL
    # the same routes one token per call: per-route copies, one route per segment
    for t in (0, T // 2, T - 1):
        o1, it1 = ftb.moe_decode(x[t:t + 1].contiguous(), bank, w[t:t + 1].contiguous(),
                                 ids[t:t + 1].contiguous(), shared=sh, debug=True)
        torch.cuda.synchronize()
        assert torch.equal(it1["ic3"][0].view(torch.int16), it["ic3"][t].view(torch.int16)), t
        assert torch.equal(o1.view(torch.int16), out[t:t + 1].view(torch.int16)), t
