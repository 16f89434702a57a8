"""A layer loaded through the ModelOpt NVFP4 checkpoint path (ftb.checkpoint.bank_from_modelopt,
the stacking of overlay/freetoken/models/glm5_next/weight.py:187-210) runs on the GPU and
matches the CPU oracle, with per-projection global scales (weight_scale_2) other than 1.0 so
the per-row fp16 globals the loader builds are exercised. Tolerance: max|d| / max|ref| <= 1e-2.
"""
import pytest
import torch

import ftb
from ftb import checkpoint, synth
from tests.moe_cases import compare, oracle_layer, to_f32

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda:0"
PREFIX = "model.language_model.layers.7.mlp"


@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_layer_loaded_from_modelopt_checkpoint(path):
    E, H, I, T, K = 8, 512, 256, 24, 2
    src = synth.make_bank(E, H, I, seed=71)
    g = torch.Generator().manual_seed(72)
    scales = 2.0 ** torch.randint(-3, 3, (E, 3), generator=g).float()  # gate, up, down
    sd = checkpoint.bank_to_modelopt(src, PREFIX, global_scales=scales)
    bank = checkpoint.bank_from_modelopt(sd.__getitem__, PREFIX, E)
    for e in range(E):  # the loader's fp16 per-row globals carry the checkpoint scales
        assert torch.all(bank.gate_up_global[e, :I].float() == scales[e, 0])
        assert torch.all(bank.gate_up_global[e, I:].float() == scales[e, 1])
        assert torch.all(bank.down_global[e].float() == scales[e, 2])
    inp = synth.make_inputs(T, H, E, seed=73)
    from oracle import moe_oracle as m

    w, ids = m.topk_softmax(inp.logits.numpy(), K, True)
    case = dict(bank=bank, shared=None, inp=inp, w=w, ids=ids, K=K)
    ref = oracle_layer(case)
    fn = ftb.moe_decode if path == "decode" else ftb.moe_prefill
    out, it = fn(inp.x.to(DEV), bank.to(DEV), torch.from_numpy(w).to(DEV),
                 torch.from_numpy(ids).to(DEV), debug=True)
    torch.cuda.synchronize()
    assert it["status"] == 0
    for name in ("ic1", "h", "ic3"):
        assert compare(to_f32(it[name]), ref[name])[0] <= TOL, name
    assert compare(to_f32(out), ref["out"])[0] <= TOL
