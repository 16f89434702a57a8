"""B200 NVFP4 experts behind FreeToken's MoE backend interface.

``B200Nvfp4Experts.routed_forward(hidden_states, topk_weights, topk_ids, overlap_fn=None)``
has the contract of ``ResidentNvfp4Experts`` / ``OffloadMoELayer.routed_forward``
(overlay/freetoken/models/glm5_next/experts_resident.py:49-83; patches/layers_moe.patch:3-12,
:65-98): bf16 [T, H] in, bf16 [T, H] out, fp32/int32 [T, k] routing, raw expert ids
(position == expert id), ``topk_ids`` not modified. ``select_nvfp4_backend`` mirrors the
reference's backend pick (patches/moe_expert_banks.patch:38-42) and answers ``"b200"`` on
sm_100 devices for the activations this build implements.

``Nvfp4MoELayer`` is the model block around it (router GEMV or given logits -> top-k ->
routed experts -> + shared expert; patches/models_glm_moe_dsa_moe.patch:137-207).
"""
from __future__ import annotations

import torch

from .banks import FP8, Nvfp4Bank
from .fused_nvfp4 import _ACTS, PREFILL_MIN_TOKENS, moe_decode, moe_prefill
from .fused_route import fused_route, fused_topk, router_logits

DECODE_MAX_TOKENS = 64  # routed_forward treats larger batches as prefill when not told


def select_nvfp4_backend(device, moe_intermediate_size=None, nvfp4_backend: str = "auto",
                         activation: str = "silu") -> str:
    if nvfp4_backend not in ("auto", "b200"):
        raise ValueError(f"nvfp4 backend {nvfp4_backend!r} is not available in this build")
    if activation not in _ACTS:
        raise NotImplementedError(f"activation {activation!r} is not built (have {sorted(_ACTS)})")
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("the b200 NVFP4 backend needs a CUDA device")
    major, minor = torch.cuda.get_device_capability(dev)
    if major != 10:
        raise NotImplementedError(f"sm_{major}{minor} is not a B200-class (sm_100) device")
    return "b200"


class B200Nvfp4Experts:
    """GPU-resident NVFP4 routed experts (+ optional shared expert) of one MoE layer."""

    def __init__(self, bank: Nvfp4Bank, activation: str = "silu", swiglu_limit=None,
                 shared: Nvfp4Bank | None = None, layer_id: int = -1,
                 hidden_act_alpha: float = 1.702, apply_router_weight_on_input: bool = False):
        if activation not in _ACTS:
            raise NotImplementedError(f"activation {activation!r} is not built (have {sorted(_ACTS)})")
        bank.validate()
        self.bank = bank
        self.shared = shared
        self.layer_id = layer_id
        self.num_experts = bank.num_experts
        self.activation = activation
        # the resident layer's attributes (experts_resident.py:32-33)
        self.apply_router_weight_on_input = apply_router_weight_on_input
        self.hidden_act_alpha = hidden_act_alpha
        self.swiglu_limit = swiglu_limit

    @classmethod
    def empty(cls, num_experts: int, hidden: int, inter: int, device, activation="silu",
              swiglu_limit=None, layer_id: int = -1):
        """Uninitialised banks with the reference's shapes and dtypes (weights to be loaded)."""
        e, h, i = num_experts, hidden, inter
        kw = dict(device=device)
        bank = Nvfp4Bank(torch.empty(e, 2 * i, h // 2, dtype=torch.uint8, **kw),
                         torch.empty(e, 2 * i, h // 16, dtype=FP8, **kw),
                         torch.empty(e, 2 * i, dtype=torch.float16, **kw),
                         torch.empty(e, h, i // 2, dtype=torch.uint8, **kw),
                         torch.empty(e, h, i // 16, dtype=FP8, **kw),
                         torch.empty(e, h, dtype=torch.float16, **kw))
        return cls(bank, activation, swiglu_limit, None, layer_id)

    def _limit(self) -> float:
        L = self.swiglu_limit
        return float("inf") if L is None else float(L)

    def routed_forward(self, hidden_states: torch.Tensor, topk_weights: torch.Tensor,
                       topk_ids: torch.Tensor, overlap_fn=None, split_overlap_fn=None,
                       *, include_shared: bool = False, is_prefill: bool | None = None):
        """Expert compute for an externally computed routing decision.

        ``overlap_fn`` (no-argument callable) runs on the current stream before the expert
        GEMVs, as the resident reference path has no copy to overlap it with.
        ``include_shared=True`` folds ``+ shared_experts(x)`` into the same launch chain."""
        del split_overlap_fn  # offload-only hook: a resident layer never calls it
        if overlap_fn is not None:
            overlap_fn()
        shared = self.shared if include_shared else None
        # the resident reference routes prefill and decode to different drivers
        # (experts_resident.py:69-83); is_prefill=None picks by the token count
        if is_prefill is None:
            is_prefill = hidden_states.shape[0] >= PREFILL_MIN_TOKENS
        layer = moe_prefill if is_prefill else moe_decode
        return layer(hidden_states, self.bank, topk_weights, topk_ids,
                     activation=self.activation, act_limit=self._limit(),
                     act_alpha=self.hidden_act_alpha,
                     apply_router_weight_on_input=self.apply_router_weight_on_input,
                     shared=shared)


class Nvfp4MoELayer:
    """Router + routed NVFP4 experts + shared expert: one MoE layer of the model block."""

    def __init__(self, experts: B200Nvfp4Experts, top_k: int, renormalize: bool = True,
                 router: str = "softmax", gate_weight: torch.Tensor | None = None,
                 score_bias: torch.Tensor | None = None, routed_scaling: float = 1.0):
        if router not in ("softmax", "sigmoid", "sqrtsoftplus"):
            raise ValueError(f"router {router!r}")
        self.experts = experts
        self.top_k = top_k
        self.renormalize = renormalize
        self.router = router
        self.gate_weight = gate_weight
        self.score_bias = score_bias
        self.routed_scaling = routed_scaling

    def route(self, hidden_states: torch.Tensor, logits: torch.Tensor | None = None):
        if logits is None:
            if self.gate_weight is None:
                raise ValueError("no router logits and no gate weight")
            logits = router_logits(hidden_states, self.gate_weight)
        if self.router == "softmax":
            return fused_topk(hidden_states, logits, self.top_k, self.renormalize)
        bias = self.score_bias if self.score_bias is not None else torch.zeros(
            logits.shape[1], device=logits.device)
        return fused_route(logits, bias, self.top_k, self.renormalize, self.routed_scaling,
                           act=self.router)

    def forward(self, hidden_states: torch.Tensor, logits: torch.Tensor | None = None):
        w, ids = self.route(hidden_states, logits)
        return self.experts.routed_forward(hidden_states, w, ids,
                                           include_shared=self.experts.shared is not None)

    __call__ = forward
