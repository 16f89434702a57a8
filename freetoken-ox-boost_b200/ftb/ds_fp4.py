"""ds_fp4 MoE layers (the DeepSeek-V4 expert format) on the NVFP4 kernels.

The reference's ds_fp4 layer (``freetoken.moe.fused_ds_fp4``, patches/moe_fused_ds_fp4.patch)
keeps each expert's weights as e2m1 codes (two per byte, gate rows 0..I-1 then up rows
I..2I-1 of gate_up) with one e8m0 scale per 32 consecutive elements of a row (a power of two,
2^(s - 127); byte 255 is NaN), and no per-row global. Its decode (``:119-141``) is: the gate_up
GEMV to bf16, ``fused_swiglu(gate_up, swiglu_limit, quant=True)`` (the activation rounded
through FP8 per 128 elements, patches/kernel_triton_dsv4_fused_moe.patch:25-35), the down GEMV
times the routed weight to bf16, and the sum over k; its prefill runs the same steps on grouped
GEMMs (``:220-242``).

Here a ds_fp4 bank is converted ONCE, exactly, into the native NVFP4 bank
(``nvfp4_from_ds_fp4``): a row whose e8m0 scales have the largest exponent m gets the global
2^(m - 8) (fp16, exact for m - 8 in [-24, 15]) and every 16-element block the E4M3 scale
2^(s - 127 - (m - 8)) (exact for exponents in [-9, 8], i.e. block scales down to 2^-17 of the
row's largest), so code * scale * global is the same real number as code * 2^(s - 127). The
layer then runs the NVFP4 decode GEMVs / tensor-core GEMMs with ``h_quant="fp8_block128"``.
Blocks whose scale lies more than 17 binades below their row's largest cannot be held exactly;
the conversion counts them and (``strict=True``) refuses, or flushes them to scale 0.

The cost of one bank format: an E4M3 byte per 16 weights instead of an e8m0 byte per 32
(+1/32 byte per weight, ~6% more bytes streamed by the HBM-bound decode).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .banks import Nvfp4Bank

E8M0 = getattr(torch, "float8_e8m0fnu", None)
_E4M3_MIN_EXP, _E4M3_MAX_EXP = -9, 8     # 2^k exactly representable in E4M3 (fn)
_F16_MIN_EXP, _F16_MAX_EXP = -24, 15     # 2^c exactly representable in fp16


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.dtype != torch.uint8 else t


@dataclass
class DsFp4Bank:
    """One ds_fp4 layer's routed experts (position == expert id)."""
    gate_up_packed: torch.Tensor  # [E, 2I, H/2] uint8 e2m1 codes (low nibble = even element)
    gate_up_scale: torch.Tensor   # [E, 2I, H/32] e8m0 (float8_e8m0fnu or uint8 bits)
    down_packed: torch.Tensor     # [E, H, I/2] uint8
    down_scale: torch.Tensor      # [E, H, I/32] e8m0

    @property
    def num_experts(self) -> int:
        return self.gate_up_packed.shape[0]

    @property
    def hidden(self) -> int:
        return self.down_packed.shape[1]

    @property
    def inter(self) -> int:
        return self.gate_up_packed.shape[1] // 2

    def validate(self) -> None:
        E, H, I = self.num_experts, self.hidden, self.inter
        want = {"gate_up_packed": (E, 2 * I, H // 2), "gate_up_scale": (E, 2 * I, H // 32),
                "down_packed": (E, H, I // 2), "down_scale": (E, H, I // 32)}
        for name, shape in want.items():
            t = getattr(self, name)
            if tuple(t.shape) != shape:
                raise ValueError(f"{name}: shape {tuple(t.shape)} != {shape}")
            if t.element_size() != 1:
                raise ValueError(f"{name}: one-byte elements expected, got {t.dtype}")
        if H % 32 or I % 32:
            raise ValueError("hidden and inter must be multiples of 32")


@dataclass
class ConversionReport:
    rows: int               # weight rows converted (gate_up and down, all experts)
    flushed_blocks: int     # 32-element blocks whose scale fell out of the exact range (now 0)
    global_exp_min: int     # range of the per-row global exponents c (global = 2^c)
    global_exp_max: int


def _convert(packed: torch.Tensor, scale: torch.Tensor, strict: bool):
    """One projection: e8m0 per 32 -> (E4M3 bits per 16, fp16 global per row, counts)."""
    s = _u8(scale).to(torch.int32)                      # [E, N, K/32]
    if bool((s == 255).any()):
        raise ValueError("e8m0 scale byte 255 (NaN) in the bank")
    c = s.amax(-1) - 127 - _E4M3_MAX_EXP                # [E, N]: global 2^c
    lo, hi = int(c.min()), int(c.max())
    if lo < _F16_MIN_EXP or hi > _F16_MAX_EXP:
        raise ValueError(f"row scale exponents {lo + 8}..{hi + 8} do not fit an fp16 global "
                         f"2^c with c in [{_F16_MIN_EXP}, {_F16_MAX_EXP}]")
    k = s - 127 - c[..., None]                          # block exponent vs the global, <= 8
    flush = k < _E4M3_MIN_EXP
    n_flush = int(flush.sum())
    if strict and n_flush:
        raise ValueError(f"{n_flush} blocks have scales more than 17 binades below their row's "
                         "largest; pass strict=False to flush them to 0")
    k = k.clamp(min=_E4M3_MIN_EXP)
    normal = (k + 7) << 3                               # E4M3 exponent field, mantissa 0
    sub = torch.ones_like(k) << (k - _E4M3_MIN_EXP).clamp(max=2)  # 2^-9, 2^-8, 2^-7
    bits = torch.where(k >= -6, normal, sub)
    bits = torch.where(flush, torch.zeros_like(bits), bits).to(torch.uint8)
    sf = bits.repeat_interleave(2, dim=-1).contiguous()  # one per 16 elements
    glob = torch.ldexp(torch.ones(c.shape, dtype=torch.float32, device=c.device),
                       c.to(torch.float32)).to(torch.float16)
    return packed.contiguous(), sf, glob, n_flush, lo, hi


def nvfp4_from_ds_fp4(bank: DsFp4Bank, strict: bool = True):
    """A ds_fp4 bank as the native NVFP4 bank holding the same weights (see the module
    docstring), and a ConversionReport. Runs on the bank's device."""
    bank.validate()
    gp, gs, gg, f1, l1, h1 = _convert(bank.gate_up_packed, bank.gate_up_scale, strict)
    dp, ds, dg, f2, l2, h2 = _convert(bank.down_packed, bank.down_scale, strict)
    out = Nvfp4Bank(gp, gs, gg, dp, ds, dg)
    out.validate()
    rep = ConversionReport(rows=bank.num_experts * (2 * bank.inter + bank.hidden),
                           flushed_blocks=f1 + f2, global_exp_min=min(l1, l2),
                           global_exp_max=max(h1, h2))
    return out, rep


def ds_fp4_dequant(packed: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """[..., N, K/2] codes and [..., N, K/32] e8m0 -> fp32 [..., N, K] (code * 2^(s - 127)):
    the ds_fp4 weight values, for checks."""
    lut = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], device=packed.device)
    codes = torch.stack([packed & 15, packed >> 4], dim=-1).flatten(-2).long()
    e = _u8(scale).to(torch.float32) - 127.0
    return lut[codes] * torch.exp2(e).repeat_interleave(32, dim=-1)


def fused_experts_ds_fp4(hidden_states: torch.Tensor, bank: Nvfp4Bank,
                         topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                         swiglu_limit: float = 0.0, *, shared: Nvfp4Bank | None = None,
                         out: torch.Tensor | None = None, prefill: bool | None = None,
                         debug: bool = False, check_status: bool = False):
    """The ds_fp4 MoE layer on a converted bank (``nvfp4_from_ds_fp4``): gate_up -> bf16,
    SwiGLU (clamped at swiglu_limit when it is > 0, as ``HAS_LIMIT=limit > 0``) with the FP8
    round trip per 128 elements, down x routed weight -> bf16, sum over k in order.
    ``prefill`` None picks the tensor-core GEMMs from PREFILL_MIN_TOKENS tokens."""
    from .fused_nvfp4 import PREFILL_MIN_TOKENS, moe_decode, moe_prefill

    L = float(swiglu_limit)
    clamp = L > 0 and L != float("inf")
    if prefill is None:
        prefill = hidden_states.shape[0] >= PREFILL_MIN_TOKENS
    fn = moe_prefill if prefill else moe_decode
    return fn(hidden_states, bank, topk_weights, topk_ids,
              activation="swiglu_clamp" if clamp else "silu",
              act_limit=L if clamp else float("inf"), shared=shared, out=out, debug=debug,
              check_status=check_status, h_quant="fp8_block128")
