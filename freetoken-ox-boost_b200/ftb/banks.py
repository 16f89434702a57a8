"""The six native NVFP4 expert banks of one MoE layer (position == expert id).

Same tensors, names, shapes and dtypes as ``ResidentNvfp4Experts``
(overlay/freetoken/models/glm5_next/experts_resident.py:36-41); scales may be
``torch.float8_e4m3fn`` (as there) or their ``uint8`` bit view. Bytes per expert follow the
reference's ``_BANK_BYTES_PER_EXPERT["nvfp4"]`` (patches/moe_offload_cache.patch:13):
``2I*(H/2 + H/16 + 2) + H*(I/2 + I/16 + 2)``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ._lib import Nvfp4BankStruct

FP8 = torch.float8_e4m3fn


def bank_bytes_per_expert(hidden: int, inter: int) -> int:
    H, I = hidden, inter
    return 2 * I * (H // 2 + H // 16 + 2) + H * (I // 2 + I // 16 + 2)


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.dtype == FP8 else t


@dataclass
class Nvfp4Bank:
    gate_up_packed: torch.Tensor  # [E, 2I, H/2] uint8
    gate_up_scale: torch.Tensor   # [E, 2I, H/16] e4m3 (or uint8 bits)
    gate_up_global: torch.Tensor  # [E, 2I] fp16
    down_packed: torch.Tensor     # [E, H, I/2] uint8
    down_scale: torch.Tensor      # [E, H, I/16] e4m3 (or uint8 bits)
    down_global: torch.Tensor     # [E, H] fp16

    @property
    def num_experts(self) -> int:
        return self.gate_up_packed.shape[0]

    @property
    def hidden(self) -> int:
        return self.down_packed.shape[1]

    @property
    def inter(self) -> int:
        return self.gate_up_packed.shape[1] // 2

    @property
    def device(self) -> torch.device:
        return self.gate_up_packed.device

    def tensors(self):
        return (self.gate_up_packed, self.gate_up_scale, self.gate_up_global,
                self.down_packed, self.down_scale, self.down_global)

    def validate(self) -> None:
        E, H, I = self.num_experts, self.hidden, self.inter
        want = {
            "gate_up_packed": ((E, 2 * I, H // 2), (torch.uint8,)),
            "gate_up_scale": ((E, 2 * I, H // 16), (torch.uint8, FP8)),
            "gate_up_global": ((E, 2 * I), (torch.float16,)),
            "down_packed": ((E, H, I // 2), (torch.uint8,)),
            "down_scale": ((E, H, I // 16), (torch.uint8, FP8)),
            "down_global": ((E, H), (torch.float16,)),
        }
        for name, (shape, dtypes) in want.items():
            t = getattr(self, name)
            if tuple(t.shape) != shape:
                raise ValueError(f"{name}: shape {tuple(t.shape)} != {shape}")
            if t.dtype not in dtypes:
                raise ValueError(f"{name}: dtype {t.dtype} not in {dtypes}")
            if not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous")
            if t.device != self.device:
                raise ValueError(f"{name} on {t.device}, bank on {self.device}")

    def struct(self) -> Nvfp4BankStruct:
        return Nvfp4BankStruct(
            self.gate_up_packed.data_ptr(), _u8(self.gate_up_scale).data_ptr(),
            self.gate_up_global.data_ptr(), self.down_packed.data_ptr(),
            _u8(self.down_scale).data_ptr(), self.down_global.data_ptr(), self.num_experts)

    def to(self, device) -> "Nvfp4Bank":
        return Nvfp4Bank(*(t.to(device) for t in self.tensors()))

    def select(self, experts) -> "Nvfp4Bank":
        """Experts ``experts`` (a slice or index tensor) as a new contiguous bank."""
        return Nvfp4Bank(*(t[experts].contiguous() for t in self.tensors()))

    def numpy(self) -> dict:
        """uint8 / fp16 numpy views keyed by bank name (the oracle's input format)."""
        names = ("gate_up_packed", "gate_up_scale", "gate_up_global",
                 "down_packed", "down_scale", "down_global")
        return {n: _u8(t).detach().cpu().numpy() for n, t in zip(names, self.tensors())}
