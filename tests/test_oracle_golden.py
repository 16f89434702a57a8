"""The CPU oracle against golden vectors produced by the reference's own Triton kernels
(run under Triton's CPU interpreter by tests/golden/make_golden.py)."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import moe_oracle as m

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_e2m1_table_matches_reference_decode():
    t = np.load(os.path.join(GOLDEN, "e2m1_table.npz"))
    assert np.array_equal(t["f32"], m.E2M1_LUT)
    assert np.array_equal(m.bf16_from_bits(t["bf16_bits"]), m.E2M1_LUT)
    # -0.0 for code 8, like the reference's sign-bit construction
    assert np.signbit(m.E2M1_LUT[8])


def test_e4m3_table_matches_torch_all_bytes():
    b = torch.arange(256, dtype=torch.uint8)
    ref = b.view(torch.float8_e4m3fn).float().numpy()
    got = m.E4M3_TABLE
    assert np.array_equal(np.isnan(ref), np.isnan(got))
    ok = ~np.isnan(ref)
    assert np.array_equal(ref[ok].view(np.uint32), got[ok].view(np.uint32))


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(50000) * 10, rng.standard_normal(1000) * 1e-38,
                        [0.0, -0.0, np.inf, -np.inf, 3.3895e38]]).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(m.bf16_round(x).view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "route_sigmoid_*.npz"))))
def test_sigmoid_router_bit_exact(path):
    d = np.load(path)
    w, ids = m.fused_route_sigmoid(d["logits"], d["bias"], int(d["top_k"]), bool(d["renorm"]),
                                   float(d["scaling"]))
    assert np.array_equal(ids, d["ids"])
    assert np.array_equal(w.view(np.uint32), d["w"].view(np.uint32))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "route_sqrtsoftplus_*.npz"))))
def test_sqrtsoftplus_router_matches_reference(path):
    """The sqrt(softplus) score mode: ids bit-exact; weights within 2 ulp-scale (the
    interpreter's exp/log are numpy's, the oracle's too, but the fused form rounds twice)."""
    d = np.load(path)
    w, ids = m.fused_route_sigmoid(d["logits"], d["bias"], int(d["top_k"]), bool(d["renorm"]),
                                   float(d["scaling"]), act="sqrtsoftplus")
    assert np.array_equal(ids, d["ids"])
    fin = np.isfinite(d["w"])
    assert np.array_equal(np.isfinite(w), fin)
    assert np.abs(w[fin] - d["w"][fin]).max(initial=0) <= 2e-6 * max(1.0, np.abs(d["w"][fin]).max())


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "route_ranked_*.npz"))))
def test_ranked_router_bit_exact(path):
    d = np.load(path)
    w, ids, rid, rsc = m.fused_route_sigmoid(d["logits"], d["bias"], int(d["top_k"]),
                                             bool(d["renorm"]), float(d["scaling"]),
                                             n_rank=int(d["n_rank"]))
    assert np.array_equal(ids, d["ids"]) and np.array_equal(rid, d["rank_ids"])
    assert np.array_equal(rsc.view(np.uint32), d["rank_scores"].view(np.uint32))
    assert np.array_equal(w.view(np.uint32), d["w"].view(np.uint32))
    assert np.array_equal(rid[:, :int(d["top_k"])], ids)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "down_swiglu_*.npz"))))
def test_down_gemv_swiglu_bit_exact(path):
    """SwiGLU + down GEMV + global + routed weight, in the reference kernel's op order.
    The interpreter casts to bf16 by truncation, so the replay uses ``bf16_trunc``."""
    d = np.load(path)
    gu = m.bf16_from_bits(d["gate_up_bits"])
    I = gu.shape[1] // 2
    h = m.swiglu(gu[:, :I], gu[:, I:], float(d["limit"]), rnd=m.bf16_trunc)
    ids = d["topk_ids"].reshape(-1)
    w = d["topk_w"].reshape(-1)
    glob_ = d["down_global_bits"].view(np.float16).astype(np.float32)
    ref = m.bf16_from_bits(d["ic3_bits"]).reshape(len(ids), -1)
    out = np.zeros_like(ref)
    for r, e in enumerate(ids):
        acc = m.nvfp4_gemv(h[r:r + 1], d["down_packed"][e], d["down_scale"][e])
        out[r] = m.bf16_trunc(acc[0] * glob_[e] * w[r])
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
