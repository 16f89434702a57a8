"""Router: fp32 gate GEMV and the two top-k epilogues, on libftb.

Mirrors the reference's routing entry points:
  * ``fused_topk(hidden_states, gating_output, topk, renormalize)`` - the generic softmax
    router of ``OffloadMoELayer.decode_forward`` (patches/layers_moe.patch:100-113);
  * ``fused_route(logits, bias, top_k, renorm, scaling, act)`` - the GLM sigmoid+bias
    epilogue, or its sqrt(softplus) variant (overlay/freetoken/kernel/triton/fused_route.py:65-82);
  * ``fused_route_ranked(logits, bias, top_k, renorm, scaling, n_rank)`` - the same plus the
    ranked top-``n_rank`` list (overlay/freetoken/kernel/triton/fused_route.py:124-137);
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


_ROUTE_ACTS = {"sigmoid": _lib.FTB_ROUTE_SIGMOID, "sqrtsoftplus": _lib.FTB_ROUTE_SQRTSOFTPLUS}


def fused_route(logits: torch.Tensor, bias: torch.Tensor, top_k: int, renorm: bool,
                scaling: float, act: str = "sigmoid"):
    """score(l) + bias -> first-index top-k -> w = score[ids] / (sum + 1e-20) * scaling, with
    score = sigmoid(l) (``act="sigmoid"``) or sqrt(softplus(l)) (``act="sqrtsoftplus"``), as
    ``fused_route`` (overlay/freetoken/kernel/triton/fused_route.py:65-82)."""
    if act not in _ROUTE_ACTS:
        raise ValueError(f"fused_route act={act!r}: expected one of {sorted(_ROUTE_ACTS)}")
    return _route(logits.contiguous(), top_k, _ROUTE_ACTS[act], bias, scaling, renorm)


def fused_route_ranked(logits: torch.Tensor, bias: torch.Tensor, top_k: int, renorm: bool,
                       scaling: float, n_rank: int = 16):
    """``fused_route`` (sigmoid) plus the ranked list of the score-aware expert cache:
    ``(w, ids, rank_ids int32 [T, n_rank], rank_scores fp32 [T, n_rank])``, the top ``n_rank``
    experts by selection score with their raw sigmoid scores (0 for NaN); the first ``top_k``
    ranks are the selected ids (overlay/freetoken/kernel/triton/fused_route.py:124-137)."""
    dev = require_cuda(logits)
    require(logits, "logits", torch.float32)
    if logits.dim() != 2:
        raise ValueError("logits must be [T, E]")
    logits = logits.contiguous()
    T, E = logits.shape
    if not top_k <= n_rank <= E:
        raise ValueError(f"need top_k <= n_rank <= E (got {top_k}, {n_rank}, {E})")
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    ids = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    rid = torch.empty(T, n_rank, dtype=torch.int32, device=dev)
    rsc = torch.empty(T, n_rank, dtype=torch.float32, device=dev)
    b = None if bias is None else bias.to(device=dev, dtype=torch.float32).contiguous()
    st = _lib.load().ftb_route_ranked(ptr(logits), T, E, top_k, n_rank, ptr(b), float(scaling),
                                      1 if renorm else 0, ptr(w), ptr(ids), ptr(rid), ptr(rsc),
                                      stream_handle(dev))
    _lib.check("ftb_route_ranked", st)
    return w, ids, rid, rsc


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
