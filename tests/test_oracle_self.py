"""Self-consistency of the oracle: GEMV vs exact float64 dequantisation, the permutation's
definition, the softmax router's tie/NaN rules, and the full layer vs float64."""
import numpy as np
import torch

from ftb import synth
from oracle import moe_oracle as m


def test_gemv_matches_float64_dequant():
    rng = np.random.default_rng(1)
    N, K = 48, 512
    packed = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    scale = torch.from_numpy(np.abs(rng.standard_normal((N, K // 16)) * 0.01).astype(np.float32)) \
        .to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    a = m.bf16_round(rng.standard_normal((5, K)).astype(np.float32))
    got = m.nvfp4_gemv(a, packed, scale)
    ref = a.astype(np.float64) @ m.dequant_rows(packed, scale).astype(np.float64).T
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


def test_moe_align_definition():
    rng = np.random.default_rng(2)
    T, K, E, bm = 37, 4, 16, 8
    ids = rng.integers(0, E, (T, K)).astype(np.int32)
    ids[3] = [5, 5, 5, 5]  # repeated expert within a token
    sorted_ids, expert_ids, ntpp, offsets, order = m.moe_align(ids, E, bm)
    flat = ids.reshape(-1)
    R = flat.size
    assert ntpp % bm == 0 and ntpp == len(sorted_ids)
    real = sorted_ids[sorted_ids < R]
    assert sorted(real.tolist()) == list(range(R))  # a permutation
    for b, e in enumerate(expert_ids):
        blk = sorted_ids[b * bm:(b + 1) * bm]
        blk = blk[blk < R]
        assert np.all(flat[blk] == e)
        assert np.all(np.diff(blk) > 0)  # stable: increasing route index
    assert np.array_equal(np.diff(offsets), np.bincount(flat, minlength=E))
    assert np.array_equal(order, np.argsort(flat, kind="stable"))


def test_topk_softmax_ties_and_nan():
    lg = np.zeros((2, 8), np.float32)
    lg[0] = [1, 3, 3, 2, 3, 0, -1, 2]
    lg[1] = [np.nan, 1, 1, np.nan, 0, 0, 0, 0]
    w, ids = m.topk_softmax(lg, 4, True)
    assert ids[0].tolist() == [1, 2, 4, 3]  # equal logits -> lower index first
    assert ids[1].tolist()[:2] == [1, 2]
    assert abs(float(w[0].sum()) - 1.0) < 1e-6


def test_layer_close_to_float64():
    E, H, I, T, K = 8, 256, 128, 5, 2
    bank = synth.make_bank(E, H, I, seed=3).numpy()
    shared = synth.make_shared(H, I, seed=3).numpy()
    inp = synth.make_inputs(T, H, E, seed=3)
    x = inp.x.float().numpy()
    w, ids = m.topk_softmax(inp.logits.numpy(), K, True)
    out = m.moe_layer(x, bank, w, ids, shared)["out"]
    ref = m.moe_layer_f64(x, bank, w, ids, shared)
    assert m.max_abs_rel(out, ref) < 1e-2
