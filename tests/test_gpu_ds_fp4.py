"""ds_fp4 layers on the GPU (``fused_experts_ds_fp4``): a ds_fp4 bank converted to the NVFP4
bank, the decode GEMVs and the tensor-core GEMMs with the FP8 round trip of h
(FTB_HQUANT_FP8_BLOCK128), against the oracle's layer with ``h_quant="fp8_block128"`` on the
same weights (the conversion is exact: tests/test_ds_fp4.py).

Tolerance max|d|/max|ref| <= 1e-2 for ic1, h, ic3 and out; h is also required to match the
oracle bit for bit in all but a few elements (the kernel's sigmoid is a fast exp, so an
activation one fp32 ulp from an FP8 rounding boundary may round the other way).
"""
import numpy as np
import pytest
import torch

import ftb
from ftb import synth
from ftb.ds_fp4 import nvfp4_from_ds_fp4
from oracle import moe_oracle as m
from tests.moe_cases import compare, to_f32

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda:0"


def _case(E, H, I, T, K, seed, shared=True):
    ds = synth.make_ds_fp4_bank(E, H, I, seed=seed)
    bank, rep = nvfp4_from_ds_fp4(ds)
    assert rep.flushed_blocks == 0
    sh = None
    if shared:
        sh, _ = nvfp4_from_ds_fp4(synth.make_ds_fp4_bank(1, H, I, seed=seed + 1))
    inp = synth.make_inputs(T, H, E, seed=seed)
    w, ids = m.topk_softmax(inp.logits.numpy(), K, True)
    return bank, sh, inp.x, w.astype(np.float32), ids


@pytest.mark.parametrize("E,H,I,T,K,prefill,limit", [
    (8, 512, 512, 5, 2, False, 0.0),
    (8, 512, 512, 5, 2, False, 7.0),
    (16, 1024, 768, 33, 4, False, 0.0),
    (8, 512, 512, 300, 2, True, 0.0),
    (8, 512, 768, 260, 4, True, 7.0),
])
def test_ds_fp4_layer_matches_oracle(E, H, I, T, K, prefill, limit):
    bank, sh, x, w, ids = _case(E, H, I, T, K, seed=40 + T)
    out, it = ftb.fused_experts_ds_fp4(x.to(DEV), bank.to(DEV), torch.from_numpy(w).to(DEV),
                                       torch.from_numpy(ids).to(DEV), limit,
                                       shared=sh.to(DEV), prefill=prefill, debug=True)
    torch.cuda.synchronize()
    assert it["status"] == 0
    ref = m.moe_layer(x.float().numpy(), bank.numpy(), w, ids, sh.numpy(),
                      limit if limit > 0 else float("inf"), h_quant="fp8_block128")
    for name in ("ic1", "h", "ic3", "shared_h", "shared_out", "out"):
        rel, frac = compare(to_f32(it[name] if name != "out" else out), ref[name])
        assert rel <= TOL, (name, rel)
        if name in ("h", "shared_h"):
            assert frac <= 1e-3, (name, frac)


def test_ds_fp4_large_activation_rows():
    """Rows whose activation reaches ~1e6 (beyond fp16): the round trip's per-row shift keeps
    them exact, with status 0."""
    E, H, I, T, K = 8, 512, 512, 6, 2
    bank, sh, x, w, ids = _case(E, H, I, T, K, seed=77)
    x = x.clone()
    x[2] *= 1000.0  # ic1 ~ 1000x: h ~ 1e5..1e6
    out, it = ftb.fused_experts_ds_fp4(x.to(DEV), bank.to(DEV), torch.from_numpy(w).to(DEV),
                                       torch.from_numpy(ids).to(DEV), 0.0,
                                       shared=sh.to(DEV), debug=True)
    torch.cuda.synchronize()
    assert it["status"] == 0
    ref = m.moe_layer(x.float().numpy(), bank.numpy(), w, ids, sh.numpy(), float("inf"),
                      h_quant="fp8_block128")
    assert np.abs(ref["h"]).max() > 65504.0
    for name in ("h", "ic3", "out"):
        rel, _ = compare(to_f32(it[name] if name != "out" else out), ref[name])
        assert rel <= TOL, (name, rel)
