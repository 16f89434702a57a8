"""The opt-in FP4 prefill (FTB_PATH_PREFILL_FP4, tcgen05 kind::mxf4nvf4) on the GPU.

It quantises x and h to NVFP4, so it is checked against a host restatement of that arithmetic
(tests/fp4_emul.py), not against the reference's bf16-activation oracle:
  * the quantiser: codes, E4M3 scales and globals bit-exact;
  * the layer: ic1 against the emulated gate_up GEMM on the quantised x, ic3 against the
    emulated down GEMM on the quantised h the kernel produced, out against the fixed-order
    combine of the kernel's own ic3; tolerance max|d|/max|ref| <= 1e-2 (fp32 summation order).
Its distance from the reference's arithmetic (the parity oracle) is measured and bounded
loosely: this path is not parity-preserving by design.
"""
import numpy as np
import pytest
import torch

import ftb
from oracle import moe_oracle as m
from tests import fp4_emul as q4
from tests.moe_cases import build_case, compare, oracle_layer, to_f32

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda:0"


@pytest.mark.parametrize("K,dtype", [(512, torch.bfloat16), (1536, torch.float16),
                                     (4096, torch.bfloat16)])
def test_quantiser_bit_exact(K, dtype):
    g = torch.Generator().manual_seed(K)
    x = torch.randn(37, K, generator=g) * torch.logspace(-3, 3, 37)[:, None]
    x[3] = 0.0
    x[5, :40] = 0.0  # zero blocks inside a row
    x[7, 17] = 3.0e4  # one large element: most blocks of the row quantise to small codes
    x = x.to(dtype)
    q, sf, gl = ftb.quant_nvfp4(x.to(DEV))
    torch.cuda.synchronize()
    codes, s8, ge = q4.quantise(x.float())
    assert torch.equal(gl.cpu(), ge)
    assert torch.equal(sf.cpu(), s8)
    assert torch.equal(q.cpu(), q4.pack(codes))


def _emulate(case, it, shared):
    """Per route: ic1 from the quantised x, ic3 from the quantised kernel h; shared likewise."""
    bank = case["bank"]
    x = case["inp"].x.float()
    T, H = x.shape
    I = bank.inter
    ids, w = case["ids"], case["w"]
    codes, s8, gx = q4.quantise(x)
    xd = q4.dequant_unscaled(codes, s8)
    h = it["h"].float().cpu()
    ic1 = torch.zeros(T, ids.shape[1], 2 * I)
    ic3 = torch.zeros(T, ids.shape[1], H)
    for e in np.unique(ids):
        tt, kk = np.nonzero(ids == e)
        tt, kk = torch.from_numpy(tt), torch.from_numpy(kk)
        wgu = q4.weights(bank.gate_up_packed[e], bank.gate_up_scale[e])
        acc = (xd[tt] @ wgu.T) * gx[tt, None]
        ic1[tt, kk] = (acc * bank.gate_up_global[e].float()[None]).to(torch.bfloat16).float()
        hc, hs, hg = q4.quantise(h[tt, kk])
        wdn = q4.weights(bank.down_packed[e], bank.down_scale[e])
        acc3 = ((q4.dequant_unscaled(hc, hs) @ wdn.T) * hg[:, None]) * bank.down_global[e].float()
        rw = torch.from_numpy(w[tt.numpy(), kk.numpy()]).float()
        ic3[tt, kk] = (acc3 * rw[:, None]).to(torch.bfloat16).float()
    out = {"ic1": ic1, "ic3": ic3}
    if shared is not None:
        wgu = q4.weights(shared.gate_up_packed[0], shared.gate_up_scale[0])
        acc = (xd @ wgu.T) * gx[:, None]
        out["shared_ic1"] = (acc * shared.gate_up_global[0].float()[None]).to(
            torch.bfloat16).float()
        hc, hs, hg = q4.quantise(it["shared_h"].float().cpu())
        wdn = q4.weights(shared.down_packed[0], shared.down_scale[0])
        acc3 = ((q4.dequant_unscaled(hc, hs) @ wdn.T) * hg[:, None]) * shared.down_global[0].float()
        out["shared_out"] = acc3.to(torch.bfloat16).float()
    return out


@pytest.mark.parametrize("E,T,K,shared", [(8, 200, 2, True), (4, 600, 2, False)])
def test_fp4_prefill_vs_emulation(E, T, K, shared):
    torch.backends.cuda.matmul.allow_tf32 = False
    case = build_case(E, 512, 512, T, K, seed=90 + T, shared=shared)
    bank = case["bank"].to(DEV)
    sh = case["shared"].to(DEV) if shared else None
    x = case["inp"].x.to(DEV)
    w = torch.from_numpy(case["w"]).to(DEV)
    ids = torch.from_numpy(case["ids"]).to(DEV)
    out, it = ftb.moe_prefill_fp4(x, bank, w, ids, shared=sh, debug=True)
    torch.cuda.synchronize()
    assert it["status"] == 0
    ref = _emulate(case, it, case["shared"])
    for name, t in ref.items():
        rel = m.max_abs_rel(to_f32(it[name]), t.numpy())
        assert rel <= TOL, (name, rel)
    # out = the fixed-order combine of the kernel's own ic3 (+ shared)
    s = it["ic3"].float().sum(1).to(torch.bfloat16).float()
    if shared:
        s = (s + it["shared_out"].float()).to(torch.bfloat16).float()
    assert m.max_abs_rel(to_f32(out), s.cpu().numpy()) <= TOL
    # distance from the reference's bf16-activation arithmetic (not a parity claim)
    err = compare(to_f32(out), oracle_layer(case)["out"])[0]
    print(f"fp4 prefill max|d|/max|ref| vs parity oracle: {err:.3f}")
    assert err < 0.35


@pytest.mark.parametrize("E", [256, 32])
def test_fp4_prefill_config2_shape_close_to_parity_path(E):
    """BASELINE config-2 shape (H=4096, I=1536, top-8, shared expert; 16 and 6 k stages): with
    256 experts all 4D tile coordinates of a full bank; with 32 experts the segments of config 2
    at T=4096 (128 routes per expert) on a bank of 340 MB. The FP4 path stays within the NVFP4
    activation error of the parity path, with status 0 (the first call is a warm-up)."""
    from ftb import synth

    H, I, K, T = 4096, 1536, 8, 512
    bank = synth.make_bank(E, H, I, seed=33, device=DEV)
    shared = synth.make_shared(H, I, seed=33, device=DEV)
    inp = synth.make_inputs(T, H, E, seed=33, device=DEV)
    w, ids = ftb.fused_topk(inp.x, inp.logits, K, True)
    ref = ftb.moe_prefill(inp.x, bank, w, ids, shared=shared)
    ftb.moe_prefill_fp4(inp.x, bank, w, ids, shared=shared)
    got, it = ftb.moe_prefill_fp4(inp.x, bank, w, ids, shared=shared, debug=True)
    torch.cuda.synchronize()
    assert it["status"] == 0
    err = float((got.float() - ref.float()).abs().max() / ref.float().abs().max())
    print(f"fp4 prefill at config-2 shape, max|d|/max|ref| vs parity path: {err:.3f}")
    assert err < 0.35
