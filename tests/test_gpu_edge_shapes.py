"""The layer at the edges of its shape rules, decode and prefill, against the oracle
(oracle/moe_oracle.py) with the north star's tolerance (max|d| / max|ref| <= 1e-2 for every
bf16 intermediate and the output):

* one route per token (top_k = 1), and a single expert (E = 1, every route on it);
* the largest top_k (32) and the largest expert count (E = 1024) the library accepts;
* a token count that is not a multiple of anything (T = 37) with the shared expert.
"""
import pytest
import torch

import ftb
from tests.moe_cases import build_case, compare, oracle_layer, to_f32

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda:0"
PATHS = {"decode": ftb.moe_decode, "prefill": ftb.moe_prefill}


def _run(path, case):
    bank = case["bank"].to(DEV)
    sh = case["shared"].to(DEV) if case["shared"] is not None else None
    out, it = PATHS[path](case["inp"].x.to(DEV), bank, torch.from_numpy(case["w"]).to(DEV),
                          torch.from_numpy(case["ids"]).to(DEV), shared=sh, debug=True)
    torch.cuda.synchronize()
    return out, it


@pytest.mark.parametrize("path", ["decode", "prefill"])
@pytest.mark.parametrize("E,T,K,shared", [
    (8, 5, 1, True),       # top_k = 1
    (1, 6, 1, True),       # one expert
    (64, 3, 32, False),    # the largest top_k
    (1024, 8, 8, True),    # the largest expert count
    (16, 37, 4, True),     # an odd token count
])
def test_edge_shapes_match_oracle(path, E, T, K, shared):
    case = build_case(E, 256, 256, T, K, seed=E + T + K, shared=shared)
    ref = oracle_layer(case)
    out, it = _run(path, case)
    assert it["status"] == 0
    names = ["ic1", "h", "ic3"] + (["shared_h", "shared_out"] if shared else [])
    for name in names:
        rel, _ = compare(to_f32(it[name]), ref[name])
        assert rel <= TOL, (name, rel)
    rel, _ = compare(to_f32(out), ref["out"])
    assert rel <= TOL, ("out", rel)
