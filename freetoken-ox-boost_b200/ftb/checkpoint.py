"""ModelOpt NVFP4 checkpoint tensors -> the six native expert banks of one MoE layer.

The reference loads a GLM-5.3 ModelOpt NVFP4 checkpoint whose routed experts are stored per
expert and projection, ``{prefix}.experts.{e}.{gate_proj|up_proj|down_proj}.{kind}`` with
kind ``weight`` (packed e2m1, uint8 ``[rows, K/2]``, low nibble = even k), ``weight_scale``
(e4m3 ``[rows, K/16]``) and ``weight_scale_2`` (one fp32 per projection)
(overlay/freetoken/models/glm5_next/weight.py:43-46). Its resident-layer path stacks them
into the six banks (weight.py:187-210): gate_up = gate rows then up rows of each expert,
the per-projection global cast to fp16 and expanded to one value per output row. These
functions build the same banks; the kernels read that native layout directly, so no repack
follows.
"""
from __future__ import annotations

import re
from typing import Callable, Iterable

import torch

from .banks import FP8, Nvfp4Bank

_PROJS = ("gate_proj", "up_proj", "down_proj")
_KINDS = ("weight", "weight_scale", "weight_scale_2")
EXPERT_KEY_RE = re.compile(
    r"^(?P<prefix>.+)\.experts\.(?P<expert>\d+)\."
    r"(?P<proj>gate_proj|up_proj|down_proj)\.(?P<kind>weight|weight_scale|weight_scale_2)$")


def _scale_bits(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == FP8:
        return t
    if t.dtype == torch.uint8:
        return t.view(FP8)
    raise ValueError(f"weight_scale must be float8_e4m3fn or its uint8 bits, got {t.dtype}")


def bank_from_modelopt(get: Callable[[str], torch.Tensor], prefix: str, num_experts: int,
                       device=None) -> Nvfp4Bank:
    """Banks of experts 0..num_experts-1 of one layer.

    ``get(name)`` returns a checkpoint tensor (a safetensors reader's ``get_tensor``, a dict's
    ``__getitem__``); ``prefix`` is the layer's MLP prefix, e.g.
    ``"model.language_model.layers.3.mlp"``. Raises ``ValueError`` on shape or dtype
    mismatches between experts or projections."""
    E = num_experts
    if E < 1:
        raise ValueError("num_experts must be >= 1")

    def stack(proj, kind):
        ts = [get(f"{prefix}.experts.{e}.{proj}.{kind}") for e in range(E)]
        shapes = {tuple(t.shape) for t in ts}
        if len(shapes) != 1:
            raise ValueError(f"{prefix} {proj}.{kind}: experts disagree on shape {sorted(shapes)}")
        if kind == "weight":
            if ts[0].dtype != torch.uint8:
                raise ValueError(f"{proj}.weight must be packed uint8, got {ts[0].dtype}")
        else:
            ts = [_scale_bits(t) for t in ts]
        out = torch.stack(ts)
        return out.to(device) if device is not None else out

    def glob(proj, rows):
        gs = []
        for e in range(E):
            g = get(f"{prefix}.experts.{e}.{proj}.weight_scale_2")
            if g.numel() != 1:
                raise ValueError(f"{proj}.weight_scale_2 must hold one value, got {tuple(g.shape)}")
            gs.append(g.reshape(1).to(torch.float16).expand(rows))
        out = torch.stack(gs).contiguous()
        return out.to(device) if device is not None else out

    gp, up = stack("gate_proj", "weight"), stack("up_proj", "weight")
    gs, us = stack("gate_proj", "weight_scale"), stack("up_proj", "weight_scale")
    if gp.shape != up.shape or gs.shape != us.shape:
        raise ValueError("gate_proj and up_proj differ in shape")
    inter = gp.shape[1]
    dp, ds = stack("down_proj", "weight"), stack("down_proj", "weight_scale")
    hidden = dp.shape[1]
    bank = Nvfp4Bank(torch.cat([gp, up], dim=1).contiguous(),
                     torch.cat([gs, us], dim=1).contiguous(),
                     torch.cat([glob("gate_proj", inter), glob("up_proj", inter)], dim=1),
                     dp.contiguous(), ds.contiguous(), glob("down_proj", hidden))
    bank.validate()
    return bank


def moe_layers_in(names: Iterable[str]) -> dict:
    """{MLP prefix: number of experts} for every routed-expert block found in ``names``
    (expert ids must run 0..n-1 with every projection and kind present)."""
    seen: dict = {}
    for n in names:
        m = EXPERT_KEY_RE.match(n)
        if m:
            seen.setdefault(m["prefix"], set()).add((int(m["expert"]), m["proj"], m["kind"]))
    out = {}
    for prefix, keys in seen.items():
        n = 1 + max(e for e, _, _ in keys)
        want = {(e, p, k) for e in range(n) for p in _PROJS for k in _KINDS}
        missing = want - keys
        if missing:
            e, p, k = sorted(missing)[0]
            raise ValueError(f"{prefix}: missing {len(missing)} expert tensors, e.g. "
                             f"experts.{e}.{p}.{k}")
        out[prefix] = n
    return out


def bank_to_modelopt(bank: Nvfp4Bank, prefix: str, global_scales=None) -> dict:
    """The per-expert checkpoint tensors of ``bank`` (inverse of ``bank_from_modelopt``).
    ``global_scales`` (optional ``[E, 3]`` fp32: gate, up, down) are the ``weight_scale_2``
    values; by default the first row of each fp16 global."""
    I, H = bank.inter, bank.hidden
    out = {}
    for e in range(bank.num_experts):
        parts = {"gate_proj": (bank.gate_up_packed[e, :I], bank.gate_up_scale[e, :I],
                               bank.gate_up_global[e, 0]),
                 "up_proj": (bank.gate_up_packed[e, I:], bank.gate_up_scale[e, I:],
                             bank.gate_up_global[e, I]),
                 "down_proj": (bank.down_packed[e], bank.down_scale[e], bank.down_global[e, 0])}
        for j, (proj, (w, s, g)) in enumerate(parts.items()):
            base = f"{prefix}.experts.{e}.{proj}"
            out[f"{base}.weight"] = w.contiguous()
            out[f"{base}.weight_scale"] = _scale_bits(s).contiguous()
            gv = g.float() if global_scales is None else global_scales[e, j].float()
            out[f"{base}.weight_scale_2"] = gv.reshape(()).clone()
    return out
