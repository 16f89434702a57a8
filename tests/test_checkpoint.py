"""ModelOpt NVFP4 checkpoint -> native banks (ftb.checkpoint), CPU only.

The key layout and stacking follow the reference's GLM-5.3 loader
(overlay/freetoken/models/glm5_next/weight.py:43-46, :187-210)."""
import pytest
import torch

from ftb import checkpoint, synth
from ftb.banks import FP8

PREFIX = "model.language_model.layers.3.mlp"


def _bank():
    return synth.make_bank(4, 256, 256, seed=5)


def test_round_trip_bit_exact():
    bank = _bank()
    sd = checkpoint.bank_to_modelopt(bank, PREFIX)
    assert len(sd) == 4 * 3 * 3
    got = checkpoint.bank_from_modelopt(sd.__getitem__, PREFIX, 4)
    # scales come back as float8_e4m3fn (the checkpoint's dtype); compare their bits
    for a, b in zip(bank.tensors(), got.tensors()):
        assert a.shape == b.shape
        assert torch.equal(a.view(torch.uint8) if a.dtype == FP8 else a,
                           b.view(torch.uint8) if b.dtype == FP8 else b)
    assert got.gate_up_scale.dtype == FP8 and got.down_scale.dtype == FP8


def test_reference_stacking_order():
    # gate rows first, then up rows; the per-projection global expanded per row in fp16
    bank = _bank()
    sd = checkpoint.bank_to_modelopt(bank, PREFIX)
    sd[f"{PREFIX}.experts.1.up_proj.weight_scale_2"] = torch.tensor(0.25)
    sd[f"{PREFIX}.experts.2.gate_proj.weight"] = torch.full_like(
        sd[f"{PREFIX}.experts.2.gate_proj.weight"], 0x21)
    got = checkpoint.bank_from_modelopt(sd.__getitem__, PREFIX, 4)
    I = bank.inter
    assert torch.all(got.gate_up_global[1, I:] == 0.25)
    assert torch.all(got.gate_up_packed[2, :I] == 0x21)
    assert torch.equal(got.gate_up_packed[2, I:], bank.gate_up_packed[2, I:])


def test_uint8_scale_bits_accepted():
    bank = _bank()
    sd = checkpoint.bank_to_modelopt(bank, PREFIX)
    sd = {k: (v.view(torch.uint8) if v.dtype == FP8 else v) for k, v in sd.items()}
    got = checkpoint.bank_from_modelopt(sd.__getitem__, PREFIX, 4)
    assert got.gate_up_scale.dtype == FP8


def test_layer_discovery_and_errors():
    bank = _bank()
    sd = checkpoint.bank_to_modelopt(bank, PREFIX)
    sd.update(checkpoint.bank_to_modelopt(synth.make_bank(2, 256, 256, seed=1),
                                          "model.language_model.layers.7.mlp"))
    sd["model.language_model.layers.3.mlp.gate.weight"] = torch.zeros(4, 256)
    assert checkpoint.moe_layers_in(sd) == {PREFIX: 4, "model.language_model.layers.7.mlp": 2}
    del sd[f"{PREFIX}.experts.3.down_proj.weight_scale"]
    with pytest.raises(ValueError, match="missing"):
        checkpoint.moe_layers_in(sd)
    bad = checkpoint.bank_to_modelopt(bank, PREFIX)
    bad[f"{PREFIX}.experts.0.gate_proj.weight"] = bad[f"{PREFIX}.experts.0.gate_proj.weight"][:8]
    with pytest.raises(ValueError, match="disagree"):
        checkpoint.bank_from_modelopt(bad.__getitem__, PREFIX, 4)
    bad = checkpoint.bank_to_modelopt(bank, PREFIX)
    bad[f"{PREFIX}.experts.0.down_proj.weight"] = bad[f"{PREFIX}.experts.0.down_proj.weight"].float()
    with pytest.raises(ValueError):
        checkpoint.bank_from_modelopt(bad.__getitem__, PREFIX, 4)


def test_split_phase_masks():
    # the split decode's mask forms (ftb.fused_nvfp4._phase_masks, host logic only)
    from ftb.fused_nvfp4 import _phase_masks
    miss = torch.tensor([[True, False], [False, False], [True, True]])
    a, b = _phase_masks(miss, 6, torch.device("cpu"))
    assert a.dtype == torch.int8 and a.tolist() == [0, 1, 1, 1, 0, 0]
    assert b.tolist() == [1, 0, 0, 0, 1, 1]
    hit8, miss8 = a.clone(), b.clone()
    a2, b2 = _phase_masks((hit8, miss8), 6, torch.device("cpu"))
    assert torch.equal(a2, a) and torch.equal(b2, b)
    with pytest.raises(ValueError, match="T\\*top_k"):
        _phase_masks(miss, 8, torch.device("cpu"))
    with pytest.raises(ValueError):
        _phase_masks((hit8,), 6, torch.device("cpu"))
