"""Host restatement (torch, any device) of the FP4 prefill's activation quantisation and of its
GEMMs on dequantised operands: the checker for the opt-in FTB_PATH_PREFILL_FP4 path.

quantise (per row): g = amax / 2688 (1 for an all-zero row); per 16-element block
s = e4m3_rn_satfinite((amax_b / g) / 6); code = e2m1_rn_satfinite(v * (1 / (s * g))), 0 where
s == 0 - each step one fp32 operation rounded to nearest even, as the kernel does it.
"""
from __future__ import annotations

import torch

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def e2m1_rn(y: torch.Tensor) -> torch.Tensor:
    """fp32 -> e2m1 code (0..15), round to nearest even (ties to the code with mantissa bit 0),
    saturating at 6; the sign bit follows the sign of y (-0 included)."""
    a = y.abs()
    mag = torch.full_like(a, 7, dtype=torch.int64)
    for code, hi, incl in ((0, 0.25, True), (1, 0.75, False), (2, 1.25, True), (3, 1.75, False),
                           (4, 2.5, True), (5, 3.5, False), (6, 5.0, True)):
        below = (a <= hi) if incl else (a < hi)
        mag = torch.where((mag == 7) & below, torch.full_like(mag, code), mag)
    sign = torch.signbit(y).to(torch.int64)
    return (mag | (sign << 3)).to(torch.uint8)


def quantise(v: torch.Tensor):
    """v [rows, K] fp32 -> (codes uint8 [rows, K], scale bytes uint8 [rows, K/16], g [rows])."""
    v = v.float()
    rows, K = v.shape
    vb = v.view(rows, K // 16, 16)
    amax_b = vb.abs().amax(-1)
    amax = amax_b.amax(-1)
    g = amax / 2688.0
    g = torch.where((g > 0) & torch.isfinite(g), g, torch.ones_like(g))
    s = (amax_b / g[:, None]) / 6.0
    s8 = s.clamp(max=448.0).to(torch.float8_e4m3fn)
    sv = s8.float()
    inv = 1.0 / (sv * g[:, None])
    y = vb * inv[..., None]
    codes = e2m1_rn(y)
    codes = torch.where((sv > 0)[..., None], codes, torch.zeros_like(codes))
    return codes.view(rows, K), s8.view(torch.uint8), g


def pack(codes: torch.Tensor) -> torch.Tensor:
    """[rows, K] codes -> [rows, K/2] bytes, low nibble = even element."""
    c = codes.to(torch.int32)
    return (c[:, 0::2] | (c[:, 1::2] << 4)).to(torch.uint8)


def dequant_unscaled(codes: torch.Tensor, s8: torch.Tensor) -> torch.Tensor:
    """codes [rows, K] and scale bytes [rows, K/16] -> code * scale (without the global), fp32."""
    lut = E2M1.to(codes.device)
    vals = lut[codes.long()]
    s = s8.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
    return vals * s


def weights(packed: torch.Tensor, scale_u8: torch.Tensor) -> torch.Tensor:
    """Bank rows [N, K/2] codes and [N, K/16] E4M3 bits -> e2m1 * scale fp32 [N, K]."""
    codes = torch.stack([packed & 15, packed >> 4], dim=-1).reshape(packed.shape[0], -1)
    return dequant_unscaled(codes, scale_u8.view(torch.uint8))
