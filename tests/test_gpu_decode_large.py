"""GPU parity at the BASELINE config-1 shape (H=4096, I=1536, 256 experts, top-8, shared
expert) at every config-1 token count, T in {1, 4, 16, 64}. Each T asserts the decode GEMVs'
work-tile plan, so every tile variant the library can launch at this shape is checked here:
96-row gate_up tiles at T=1, 128-row tiles (8 activation rows per stage) at T=4, 128-row tiles
(16 rows per stage) at T=16 and 64, with segments of one and of two n-tiles of routes at T=64.
Activation boxes (segments of >= 6 routes, gathered x rows) are covered by
test_gpu_decode_boxes.py.

The reference here is a torch fp32 restatement, on the GPU, of the CPU oracle's arithmetic
(oracle/moe_oracle.py expert_forward / moe_layer: exact NVFP4 dequantisation, fp32 dot
products, the same bf16 roundings in the same places) - the numpy oracle itself would take
minutes at this size. Only the fp32 summation order differs from both the oracle and the
kernels, so the tolerance is the north star's: max|d| / max|ref| <= 1e-2 for the layer
output and every bf16 intermediate.
"""
import pytest
import torch

import ftb
from ftb import synth

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda:0"
E, H, I, K = 256, 4096, 1536, 8

_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                      -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def _bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def _dequant(packed: torch.Tensor, scale_u8: torch.Tensor) -> torch.Tensor:
    """[N, K/2] u8 codes (low nibble = even k) and [N, K/16] E4M3 bits -> [N, K] fp32."""
    lut = _E2M1.to(packed.device)
    codes = torch.stack([packed & 15, packed >> 4], dim=-1).reshape(packed.shape[0], -1)
    w = lut[codes.long()]
    s = scale_u8.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
    return w * s


def _expert(x: torch.Tensor, bank, e: int, route_w=None):
    """oracle expert_forward in torch fp32: ic1 = bf16(acc * global), h = bf16(silu(g) * u),
    ic3 = bf16(acc * global [* w])."""
    wgu = _dequant(bank.gate_up_packed[e], bank.gate_up_scale[e])
    acc1 = x @ wgu.T
    ic1 = _bf16(acc1 * bank.gate_up_global[e].float()[None, :])
    g, u = ic1[:, :I], ic1[:, I:]
    h = _bf16((g * torch.sigmoid(g)) * u)
    wdn = _dequant(bank.down_packed[e], bank.down_scale[e])
    acc3 = (h @ wdn.T) * bank.down_global[e].float()[None, :]
    if route_w is not None:
        acc3 = acc3 * route_w[:, None]
    return ic1, h, _bf16(acc3)


def _reference(x, bank, shared, w, ids):
    T = x.shape[0]
    xf = x.float()
    ic1 = torch.zeros(T, K, 2 * I, device=x.device)
    h = torch.zeros(T, K, I, device=x.device)
    ic3 = torch.zeros(T, K, H, device=x.device)
    for e in torch.unique(ids).tolist():
        tt, kk = torch.nonzero(ids == e, as_tuple=True)
        a, b, c = _expert(xf[tt], bank, e, w[tt, kk])
        ic1[tt, kk], h[tt, kk], ic3[tt, kk] = a, b, c
    s = ic3[:, 0].clone()
    for k in range(1, K):
        s = s + ic3[:, k]
    routed = _bf16(s)
    s1, sh, s3 = _expert(xf, shared, 0)
    return dict(ic1=ic1, h=h, ic3=ic3, shared_h=sh, shared_out=s3, out=_bf16(routed + s3))


def _max_abs_rel(got: torch.Tensor, ref: torch.Tensor) -> float:
    return float((got.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def layer():
    bank = synth.make_bank(E, H, I, seed=21, device=DEV)
    shared = synth.make_shared(H, I, seed=21, device=DEV)
    return bank, shared


PLANS = {1: (96, 128), 4: (128, 128), 16: (128, 128), 64: (128, 128)}


@pytest.mark.parametrize("T", [1, 4, 16, 64])
def test_config1_decode_matches_fp32_restatement(layer, T):
    from ftb.fused_nvfp4 import decode_plan

    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert decode_plan(T, H, I, E, K, True) == PLANS[T]
    bank, shared = layer
    inp = synth.make_inputs(T, H, E, seed=300 + T, device=DEV)
    logits = inp.logits.clone()
    if T == 64:
        logits[:, 5:8] += 4.0  # three hot experts: segments of 16 routes (two n-tiles)
    w, ids = ftb.fused_topk(inp.x, logits, K, True)
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    out, it = ftb.moe_decode(inp.x, bank, w, ids, shared=shared, debug=True)
    ref = _reference(inp.x, bank, shared, w, ids)
    torch.cuda.synchronize()
    assert it["status"] == 0
    for name in ("ic1", "h", "ic3", "shared_h", "shared_out"):
        assert _max_abs_rel(it[name], ref[name]) <= TOL, name
    assert _max_abs_rel(out, ref["out"]) <= TOL
    if T == 64:
        # segments of one n-tile (<= 8 routes) and of two (9..16 routes) both occur
        assert int((counts > 8).sum()) >= 3 and int(((counts > 0) & (counts <= 8)).sum()) > 0
