"""Seeded synthetic NVFP4 MoE layers and inputs for the BASELINE configs (no checkpoints here).

Encoding of every weight matrix (configs 0-4):
  * E2M1 codes uniform over the 16 values, independent per element: uniform bytes (two
    independent uniform nibbles), low nibble = even k;
  * one FP8-E4M3 scale per 16-element block = e4m3(absmax / 6) of an underlying
    W ~ N(0, 0.02) block (round to nearest even, as ``Tensor.to(float8_e4m3fn)``);
  * global scale 1.0 stored as fp16 per row (the resident-layer layout, ModelOpt
    ``weight_scale_2`` expanded per row: overlay/freetoken/models/glm5_next/weight.py:194-204).
Activations x ~ N(0, 1) in bf16; router logits ~ N(0, 1) fp32 (configs 1-4) or
x.float() @ G.T with G ~ N(0, 0.02) fp32 [E, H] (config 0).

Generators: ``torch.Generator`` on the target device. Banks use ``seed``, the shared expert
``seed + 1``, activations/logits/router weights ``seed + 2 + stream``. Device and host draws
differ (different generator algorithms), so parity tests generate on the host and copy.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .banks import Nvfp4Bank

CONFIGS = {
    0: dict(hidden=2048, inter=768, experts=64, top_k=8, shared=False, tokens=(4,)),
    1: dict(hidden=4096, inter=1536, experts=256, top_k=8, shared=True, tokens=(1, 4, 16, 64)),
    2: dict(hidden=4096, inter=1536, experts=256, top_k=8, shared=True, tokens=(4096,)),
    3: dict(hidden=4096, inter=1536, experts=256, top_k=8, shared=True, tokens=(64,)),
    4: dict(hidden=4096, inter=1536, experts=256, top_k=8, shared=True, tokens=(256,), layers=60),
}


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def nvfp4_matrix(rows: int, cols: int, gen: torch.Generator, device, w_std: float = 0.02):
    """(packed u8 [rows, cols/2], scale u8 [rows, cols/16], global fp16 [rows])."""
    packed = torch.randint(0, 256, (rows, cols // 2), dtype=torch.uint8, device=device,
                           generator=gen)
    w = torch.randn(rows, cols // 16, 16, device=device, generator=gen) * w_std
    scale = (w.abs().amax(dim=-1) / 6.0).to(torch.float8_e4m3fn).view(torch.uint8)
    glob = torch.ones(rows, dtype=torch.float16, device=device)
    return packed, scale.contiguous(), glob


def make_bank(num_experts: int, hidden: int, inter: int, *, seed: int = 0, device="cpu",
              w_std: float = 0.02) -> Nvfp4Bank:
    """A layer's six native banks, experts drawn in order (gate_up then down per expert)."""
    E, H, I = num_experts, hidden, inter
    gen = _gen(device, seed)
    gu_p = torch.empty(E, 2 * I, H // 2, dtype=torch.uint8, device=device)
    gu_s = torch.empty(E, 2 * I, H // 16, dtype=torch.uint8, device=device)
    gu_g = torch.empty(E, 2 * I, dtype=torch.float16, device=device)
    dn_p = torch.empty(E, H, I // 2, dtype=torch.uint8, device=device)
    dn_s = torch.empty(E, H, I // 16, dtype=torch.uint8, device=device)
    dn_g = torch.empty(E, H, dtype=torch.float16, device=device)
    for e in range(E):
        gu_p[e], gu_s[e], gu_g[e] = nvfp4_matrix(2 * I, H, gen, device, w_std)
        dn_p[e], dn_s[e], dn_g[e] = nvfp4_matrix(H, I, gen, device, w_std)
    return Nvfp4Bank(gu_p, gu_s, gu_g, dn_p, dn_s, dn_g)


def make_shared(hidden: int, inter: int, *, seed: int = 0, device="cpu") -> Nvfp4Bank:
    return make_bank(1, hidden, inter, seed=seed + 1, device=device)


@dataclass
class Inputs:
    x: torch.Tensor            # [T, H] bf16
    logits: torch.Tensor       # [T, E] fp32
    router_w: torch.Tensor | None = None  # [E, H] fp32 (config 0)


def make_inputs(tokens: int, hidden: int, experts: int, *, seed: int = 0, stream: int = 0,
                device="cpu", router_gemv: bool = False, zipf_s: float | None = None) -> Inputs:
    gen = _gen(device, seed + 2 + stream)
    x = torch.randn(tokens, hidden, device=device, generator=gen).to(torch.bfloat16)
    if router_gemv:
        G = torch.randn(experts, hidden, device=device, generator=gen) * 0.02
        logits = x.float() @ G.t()
        return Inputs(x, logits.contiguous(), G.contiguous())
    logits = torch.randn(tokens, experts, device=device, generator=gen)
    if zipf_s is not None:
        # expert popularity p_e ~ rank_e^-s, ranks from a permutation seeded by `seed` alone
        # (a property of the layer: the same on every stream / rank), added as log p
        perm = torch.randperm(experts, device=device, generator=_gen(device, seed + 7919))
        ranks = torch.empty(experts, device=device)
        ranks[perm] = torch.arange(1, experts + 1, device=device, dtype=torch.float32)
        logp = -zipf_s * torch.log(ranks)
        logp = logp - torch.logsumexp(logp, 0)
        logits = logits + logp[None, :]
    return Inputs(x, logits.contiguous(), None)


def ds_fp4_matrix(rows: int, cols: int, gen: torch.Generator, device, w_std: float = 0.02):
    """(packed u8 [rows, cols/2], e8m0 scale u8 [rows, cols/32]): uniform codes as in
    ``nvfp4_matrix``; one e8m0 scale per 32-element block = 2^ceil(log2(absmax / 6)) of an
    underlying W ~ N(0, w_std) block (the MXFP4 power-of-two rule)."""
    packed = torch.randint(0, 256, (rows, cols // 2), dtype=torch.uint8, device=device,
                           generator=gen)
    w = torch.randn(rows, cols // 32, 32, device=device, generator=gen) * w_std
    e = torch.ceil(torch.log2(w.abs().amax(dim=-1) / 6.0)).clamp(-127, 127)
    return packed, (e + 127).to(torch.uint8).contiguous()


def make_ds_fp4_bank(num_experts: int, hidden: int, inter: int, *, seed: int = 0, device="cpu",
                     w_std: float = 0.02):
    """A ds_fp4 layer's routed experts (``ds_fp4.DsFp4Bank``), experts drawn in order."""
    from .ds_fp4 import DsFp4Bank

    E, H, I = num_experts, hidden, inter
    gen = _gen(device, seed)
    gu_p = torch.empty(E, 2 * I, H // 2, dtype=torch.uint8, device=device)
    gu_s = torch.empty(E, 2 * I, H // 32, dtype=torch.uint8, device=device)
    dn_p = torch.empty(E, H, I // 2, dtype=torch.uint8, device=device)
    dn_s = torch.empty(E, H, I // 32, dtype=torch.uint8, device=device)
    for e in range(E):
        gu_p[e], gu_s[e] = ds_fp4_matrix(2 * I, H, gen, device, w_std)
        dn_p[e], dn_s[e] = ds_fp4_matrix(H, I, gen, device, w_std)
    return DsFp4Bank(gu_p, gu_s, dn_p, dn_s)
