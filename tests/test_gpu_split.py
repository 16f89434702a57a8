"""Split (hit/miss) decode: two phases over complementary route masks, as the reference's
fused_experts_decode_nvfp4_split (patches/moe_fused_nvfp4.patch:189-272), must equal the
single-phase decode bit for bit (the phases write disjoint route rows; one combine)."""
import pytest
import torch

import ftb
from ftb import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,with_shared,frac", [(5, False, 0.3), (16, True, 0.5), (64, True, 0.1)])
def test_split_equals_single_phase(T, with_shared, frac):
    E, H, I, K = 32, 512, 256, 8
    dev = "cuda"
    bank = synth.make_bank(E, H, I, seed=3, device=dev)
    shared = synth.make_shared(H, I, seed=3, device=dev) if with_shared else None
    inp = synth.make_inputs(T, H, E, seed=11, device=dev)
    w, ids = ftb.fused_topk(inp.x, inp.logits, K, True)
    ref = ftb.moe_decode(inp.x, bank, w, ids, shared=shared)
    g = torch.Generator(device="cpu").manual_seed(T)
    miss = (torch.rand(T, K, generator=g) < frac).to(dev)
    ev = torch.cuda.Event()
    ev.record()
    out = ftb.fused_experts_decode_nvfp4_split(inp.x, *bank.tensors(), w, ids, miss, ev,
                                               shared=shared)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    # the (hit, miss) int8 pair form of the mask gives the same result
    hit8, miss8 = (~miss).to(torch.int8).flatten(), miss.to(torch.int8).flatten()
    out2 = ftb.fused_experts_decode_nvfp4_split(inp.x, *bank.tensors(), w, ids, (hit8, miss8),
                                                None, shared=shared)
    assert torch.equal(out2.view(torch.int16), ref.view(torch.int16))


def test_split_all_hits_and_all_misses():
    E, H, I, K, T = 16, 256, 256, 4, 8
    bank = synth.make_bank(E, H, I, seed=2, device="cuda")
    inp = synth.make_inputs(T, H, E, seed=4, device="cuda")
    w, ids = ftb.fused_topk(inp.x, inp.logits, K, True)
    ref = ftb.moe_decode(inp.x, bank, w, ids)
    for miss in (torch.zeros(T, K, dtype=torch.bool), torch.ones(T, K, dtype=torch.bool)):
        out = ftb.fused_experts_decode_nvfp4_split(inp.x, *bank.tensors(), w, ids, miss.cuda(),
                                                   None)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
