"""Router: fp32 gate GEMV and the two top-k epilogues, on libftb.

Mirrors the reference's routing entry points:
  * ``fused_topk(hidden_states, gating_output, topk, renormalize)`` - the generic softmax
    router of ``OffloadMoELayer.decode_forward`` (patches/layers_moe.patch:100-113);
  * ``fused_route(logits, bias, top_k, renorm, scaling, act)`` - the GLM sigmoid+bias
    epilogue (overlay/freetoken/kernel/triton/fused_route.py:65-82);
  * ``router_logits(x, gate_weight)`` - ``F.linear(x.float(), gate.float())``
    (patches/models_glm_moe_dsa_moe.patch:129).
Results: ``(topk_weights fp32 [T, k], topk_ids int32 [T, k])``.
"""
from __future__ import annotations

import torch

from . import _lib
from ._runtime import ptr, require, require_cuda, stream_handle


def _route(logits: torch.Tensor, top_k: int, mode: int, bias, scaling: float, renorm: bool):
    dev = require_cuda(logits)
    require(logits, "logits", torch.float32)
    if logits.dim() != 2:
        raise ValueError("logits must be [T, E]")
    T, E = logits.shape
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    ids = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    b = None
    if bias is not None:
        b = bias.to(device=dev, dtype=torch.float32).contiguous()
    st = _lib.load().ftb_route_topk(ptr(logits), T, E, top_k, mode, ptr(b), float(scaling),
                                    1 if renorm else 0, ptr(w), ptr(ids), stream_handle(dev))
    _lib.check("ftb_route_topk", st)
    return w, ids


def fused_topk(hidden_states: torch.Tensor, gating_output: torch.Tensor, topk: int,
               renormalize: bool):
    """Softmax top-k: ids by descending logit (lowest index on ties), weights = softmax
    probabilities of the selected experts, renormalised to sum 1 when ``renormalize``."""
    del hidden_states  # shape carrier only, as in the reference call
    return _route(gating_output.float().contiguous(), topk, _lib.FTB_ROUTE_SOFTMAX, None, 1.0,
                  renormalize)


def fused_route(logits: torch.Tensor, bias: torch.Tensor, top_k: int, renorm: bool,
                scaling: float, act: str = "sigmoid"):
    """sigmoid(l) + bias -> first-index top-k -> w = sigmoid[ids] / (sum + 1e-20) * scaling."""
    if act != "sigmoid":
        raise NotImplementedError(f"fused_route act={act!r}: only 'sigmoid' is built")
    return _route(logits.contiguous(), top_k, _lib.FTB_ROUTE_SIGMOID, bias, scaling, renorm)


def router_logits(x: torch.Tensor, gate_weight: torch.Tensor) -> torch.Tensor:
    dev = require_cuda(x, gate_weight)
    require(x, "x", torch.bfloat16)
    G = gate_weight.to(torch.float32).contiguous()
    T, H = x.shape
    E = G.shape[0]
    out = torch.empty(T, E, dtype=torch.float32, device=dev)
    st = _lib.load().ftb_router_gemv(ptr(x), ptr(G), T, H, E, ptr(out), stream_handle(dev))
    _lib.check("ftb_router_gemv", st)
    return out
