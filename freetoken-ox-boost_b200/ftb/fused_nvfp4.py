"""NVFP4 fused-MoE entry points on libftb (B200, sm_100a).

Mirrors ``freetoken.moe.fused_nvfp4`` (patches/moe_fused_nvfp4.patch):
  * ``fused_experts_decode_nvfp4_marlin(x, gu_p, gu_s, gu_g, dn_p, dn_s, dn_g, topk_weights,
    topk_ids, activation, apply_router_weight_on_input, act_alpha, act_limit)``
    (decode driver, :136-152) - expert-major HBM-streaming GEMVs;
  * ``fused_experts_nvfp4(..., num_experts, ...)`` (prefill driver, called at
    overlay/freetoken/models/glm5_next/experts_resident.py:71-75);
  * ``moe_align_block_size(topk_ids, block_size, num_experts)`` (:155-156).
Extension: keyword ``shared=`` adds one always-on NVFP4 shared expert exactly as the model
block does after ``routed_forward`` (``out + shared_experts(x)``, routed first, bf16;
patches/models_glm_moe_dsa_moe.patch:203-206).

Activations (``_run_act``, patches/moe_fused_nvfp4.patch:12-22): ``"silu"`` (plain, act_limit
ignored like the reference's silu path), ``"swiglu_clamp"`` (silu(min(g, L)) * clamp(u, +-L)
with L = act_limit) and ``"swigluoai"`` (g' = min(g, L), u' = clamp(u, +-L),
g' * sigmoid(act_alpha * g') * (u' + 1); gate rows 0..I-1, up rows I..2I-1 of the bank).
``apply_router_weight_on_input=True`` puts the routed weight on the gate_up output instead of
the down output, as the reference's two MUL_ROUTED_WEIGHT flags do (:138, :145). Errors mirror
the reference's setup checks: ``ValueError`` for bad shapes/dtypes and unknown activations.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._runtime import ptr, read_status, require, require_cuda, stream_handle, workspace
from .banks import Nvfp4Bank

_ACTS = {"silu": _lib.FTB_ACT_SILU, "swiglu_clamp": _lib.FTB_ACT_SWIGLU_CLAMP,
         "swigluoai": _lib.FTB_ACT_SWIGLUOAI}
# rounding of h before the down GEMM: None = bf16 (NVFP4 layers), "fp8_block128" = the FP8
# round trip per 128 elements of the reference's ds_fp4 layers (fused_swiglu(..., quant=True))
_HQUANT = {None: _lib.FTB_HQUANT_NONE, "fp8_block128": _lib.FTB_HQUANT_FP8_BLOCK128}


def _act_spec(activation: str, act_alpha: float, act_limit: float):
    """(FTB_ACT_*, alpha, limit) for the library."""
    if activation not in _ACTS:
        raise ValueError(f"activation {activation!r} is not one of {sorted(_ACTS)}")
    L = float("inf") if act_limit is None else float(act_limit)
    if activation == "silu":
        L = float("inf")
    return _ACTS[activation], float(act_alpha), L


def _check_inputs(x, bank: Nvfp4Bank, topk_weights, topk_ids, shared):
    dev = require_cuda(x, bank.gate_up_packed, topk_weights, topk_ids)
    bank.validate()
    require(x, "hidden_states", torch.bfloat16)
    T, H = x.shape
    if H != bank.hidden:
        raise ValueError(f"hidden {H} != bank hidden {bank.hidden}")
    require(topk_weights, "topk_weights", torch.float32)
    require(topk_ids, "topk_ids", torch.int32)
    if topk_ids.shape != topk_weights.shape or topk_ids.shape[0] != T:
        raise ValueError("topk_weights/topk_ids must both be [T, top_k]")
    if shared is not None:
        shared.validate()
        if shared.device != dev or shared.hidden != H or shared.inter != bank.inter:
            raise ValueError("shared expert must match the routed bank's device and shape")
    return dev


# Token counts from which fused_experts_nvfp4 runs the tensor-core grouped GEMMs.
PREFILL_MIN_TOKENS = 256


def decode_workspace_bytes(T: int, bank: Nvfp4Bank, top_k: int, has_shared: bool) -> int:
    return int(_lib.load().ftb_moe_decode_workspace_bytes(
        T, bank.hidden, bank.inter, bank.num_experts, top_k, 1 if has_shared else 0))


def decode_plan(T: int, hidden: int, inter: int, num_experts: int, top_k: int,
                has_shared: bool) -> tuple[int, int]:
    """Work-tile rows (gate_up, down) the decode GEMVs use for a call of this shape on the
    current device (a host-side query; no kernel runs)."""
    plan = (ctypes.c_int32 * 2)()
    st = _lib.load().ftb_moe_decode_plan(T, hidden, inter, num_experts, top_k,
                                         1 if has_shared else 0, plan)
    _lib.check("ftb_moe_decode_plan", st)
    return int(plan[0]), int(plan[1])


def prefill_workspace_bytes(T: int, bank: Nvfp4Bank, top_k: int, has_shared: bool) -> int:
    return int(_lib.load().ftb_moe_prefill_workspace_bytes(
        T, bank.hidden, bank.inter, bank.num_experts, top_k, 1 if has_shared else 0))


def moe_decode(x: torch.Tensor, bank: Nvfp4Bank, topk_weights: torch.Tensor,
               topk_ids: torch.Tensor, *, activation: str = "silu", act_limit: float = 7.0,
               act_alpha: float = 1.702, apply_router_weight_on_input: bool = False,
               shared: Nvfp4Bank | None = None, out: torch.Tensor | None = None,
               debug: bool = False, check_status: bool = False, h_quant: str | None = None):
    """Decode layer on a bank object. ``debug=True`` returns (out, intermediates dict).
    ``h_quant="fp8_block128"``: h takes the ds_fp4 layers' FP8 round trip (per 128 elements)."""
    return _layer(_lib.FTB_PATH_DECODE, x, bank, topk_weights, topk_ids, activation, act_alpha,
                  act_limit, apply_router_weight_on_input, shared, out, debug, check_status,
                  h_quant=h_quant)


def moe_prefill(x: torch.Tensor, bank: Nvfp4Bank, topk_weights: torch.Tensor,
                topk_ids: torch.Tensor, *, activation: str = "silu", act_limit: float = 7.0,
                act_alpha: float = 1.702, apply_router_weight_on_input: bool = False,
                shared: Nvfp4Bank | None = None, out: torch.Tensor | None = None,
                debug: bool = False, check_status: bool = False, h_quant: str | None = None):
    """The same layer on the tensor-core grouped GEMMs (large T). Same contract and result
    as ``moe_decode``; ``debug=True`` returns (out, intermediates dict)."""
    return _layer(_lib.FTB_PATH_PREFILL, x, bank, topk_weights, topk_ids, activation, act_alpha,
                  act_limit, apply_router_weight_on_input, shared, out, debug, check_status,
                  h_quant=h_quant)


def prefill_fp4_workspace_bytes(T: int, bank: Nvfp4Bank, top_k: int, has_shared: bool) -> int:
    return int(_lib.load().ftb_moe_prefill_fp4_workspace_bytes(
        T, bank.hidden, bank.inter, bank.num_experts, top_k, 1 if has_shared else 0))


def moe_prefill_fp4(x: torch.Tensor, bank: Nvfp4Bank, topk_weights: torch.Tensor,
                    topk_ids: torch.Tensor, *, activation: str = "silu", act_limit: float = 7.0,
                    act_alpha: float = 1.702, apply_router_weight_on_input: bool = False,
                    shared: Nvfp4Bank | None = None, out: torch.Tensor | None = None,
                    debug: bool = False, check_status: bool = False):
    """Opt-in prefill on the block-scaled FP4 tensor cores (tcgen05 kind::mxf4nvf4): x and h are
    quantised to NVFP4 (``quant_nvfp4``'s rule) before each GEMM. NOT parity-preserving: the
    reference keeps activations in bf16, and its error against that arithmetic is ~1e-1
    (max|d|/max|ref|), not the 1e-2 bar. Needs hidden and inter multiples of 512, <= 4096."""
    return _layer(_lib.FTB_PATH_PREFILL_FP4, x, bank, topk_weights, topk_ids, activation,
                  act_alpha, act_limit, apply_router_weight_on_input, shared, out, debug,
                  check_status)


def quant_nvfp4(x: torch.Tensor):
    """Rows of bf16 / f16 values -> (codes uint8 [rows, K/2], E4M3 scales uint8 [rows, K/16],
    globals fp32 [rows]): g = amax/2688, s = e4m3((amax_block/g)/6), code = e2m1(v*(1/(s*g)))."""
    dev = require_cuda(x)
    if x.dtype not in (torch.bfloat16, torch.float16) or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous [rows, K] bf16 or f16 tensor")
    rows, K = x.shape
    q = torch.empty(rows, K // 2, dtype=torch.uint8, device=dev)
    sf = torch.empty(rows, K // 16, dtype=torch.uint8, device=dev)
    g = torch.empty(rows, dtype=torch.float32, device=dev)
    st = _lib.load().ftb_quant_nvfp4(ptr(x), 1 if x.dtype == torch.bfloat16 else 0, rows, K,
                                     ptr(q), ptr(sf), ptr(g), stream_handle(dev))
    _lib.check("ftb_quant_nvfp4", st)
    return q, sf, g


def _layer(path: int, x, bank, topk_weights, topk_ids, activation, act_alpha, act_limit,
           weight_on_input, shared, out, debug, check_status, route_mask=None, phase=0,
           ws=None, h_quant=None):
    dev = _check_inputs(x, bank, topk_weights, topk_ids, shared)
    kind, alpha, limit = _act_spec(activation, act_alpha, act_limit)
    if h_quant not in _HQUANT:
        raise ValueError(f"h_quant {h_quant!r} is not one of {list(_HQUANT)}")
    if h_quant is not None and path == _lib.FTB_PATH_PREFILL_FP4:
        raise ValueError("the FP4 prefill quantises h to NVFP4 itself; h_quant does not apply")
    T, H = x.shape
    K = topk_ids.shape[1]
    I = bank.inter
    if out is None and (route_mask is None or phase & _lib.PHASE_COMBINE):
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    if ws is None:
        wsb = {_lib.FTB_PATH_PREFILL: prefill_workspace_bytes,
               _lib.FTB_PATH_PREFILL_FP4: prefill_fp4_workspace_bytes}.get(
            path, decode_workspace_bytes)(T, bank, K, shared is not None)
        ws = workspace(wsb, dev)
    b = bank.struct()
    s = shared.struct() if shared is not None else None
    a = _lib.MoeArgsStruct()
    a.x, a.topk_w, a.topk_ids = x.data_ptr(), topk_weights.data_ptr(), topk_ids.data_ptr()
    a.bank = ctypes.pointer(b)
    a.shared = ctypes.pointer(s) if s is not None else None
    a.T, a.H, a.I, a.top_k = T, H, I, K
    a.activation, a.act_alpha, a.act_limit = kind, alpha, limit
    a.weight_on_input = 1 if weight_on_input else 0
    a.path = path
    a.route_mask = route_mask.data_ptr() if route_mask is not None else None
    a.phase = phase
    a.h_quant = _HQUANT[h_quant]
    a.out = out.data_ptr() if out is not None else None
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    inter = None
    if debug:
        bf = torch.bfloat16
        inter = dict(ic1=torch.zeros(T, K, 2 * I, dtype=bf, device=dev),
                     h=torch.zeros(T, K, I, dtype=bf, device=dev),
                     ic3=torch.zeros(T, K, H, dtype=bf, device=dev))
        if shared is not None:
            inter.update(shared_ic1=torch.zeros(T, 2 * I, dtype=bf, device=dev),
                         shared_h=torch.zeros(T, I, dtype=bf, device=dev),
                         shared_out=torch.zeros(T, H, dtype=bf, device=dev))
        for name, t in inter.items():
            setattr(a, name, t.data_ptr())
    st = lib.ftb_moe_layer(ctypes.byref(a), stream_handle(dev))
    _lib.check("ftb_moe_layer", st)
    if check_status or debug:
        status = read_status(ws)
        if inter is not None:
            inter["status"] = status
        if check_status and status & _lib.STATUS_BAD_ID:
            raise ValueError("topk_ids holds ids outside [0, num_experts)")
        if check_status and status & _lib.STATUS_TIMEOUT:
            raise RuntimeError("a bounded device-side wait of the layer timed out")
    return (out, inter) if debug else out


def fused_experts_decode_nvfp4_marlin(
    hidden_states: torch.Tensor,
    gate_up_packed: torch.Tensor,
    gate_up_scale: torch.Tensor,
    gate_up_global: torch.Tensor,
    down_packed: torch.Tensor,
    down_scale: torch.Tensor,
    down_global: torch.Tensor,
    topk_weights: torch.Tensor,
    topk_ids: torch.Tensor,
    activation: str = "silu",
    apply_router_weight_on_input: bool = False,
    act_alpha: float = 1.702,
    act_limit: float = 7.0,
    *,
    shared: Nvfp4Bank | None = None,
) -> torch.Tensor:
    """Drop-in for the reference decode driver (CUDA-graph safe after one eager call)."""
    bank = Nvfp4Bank(gate_up_packed, gate_up_scale, gate_up_global, down_packed, down_scale,
                     down_global)
    return moe_decode(hidden_states, bank, topk_weights, topk_ids, activation=activation,
                      act_limit=act_limit, act_alpha=act_alpha,
                      apply_router_weight_on_input=apply_router_weight_on_input, shared=shared)


def _phase_masks(miss_mask, R: int, dev):
    """(hit, miss) int8 masks over the R routes: a (hit, miss) pair of int8 masks as the
    reference's ensure kernel hands over, or one miss mask (bool or integer, [T, k] or [R])."""
    if isinstance(miss_mask, tuple):
        if len(miss_mask) != 2:
            raise ValueError("miss_mask tuple must be (hit_mask, miss_mask)")
        masks = [m.reshape(-1) for m in miss_mask]
    else:
        mb = miss_mask.reshape(-1)
        masks = [(mb == 0), (mb != 0)]
    out = []
    for m in masks:
        if m.numel() != R:
            raise ValueError(f"route masks must have T*top_k = {R} entries, got {m.numel()}")
        if m.device != dev:
            raise ValueError("route masks must be on the hidden states' device")
        out.append(m.to(torch.int8).contiguous())
    return out


def fused_experts_decode_nvfp4_split(
    hidden_states: torch.Tensor,
    gate_up_packed: torch.Tensor,
    gate_up_scale: torch.Tensor,
    gate_up_global: torch.Tensor,
    down_packed: torch.Tensor,
    down_scale: torch.Tensor,
    down_global: torch.Tensor,
    topk_weights: torch.Tensor,
    topk_ids: torch.Tensor,
    miss_mask,
    copy_event: torch.cuda.Event | None,
    activation: str = "silu",
    apply_router_weight_on_input: bool = False,
    act_alpha: float = 1.702,
    act_limit: float = 7.0,
    *,
    shared: Nvfp4Bank | None = None,
) -> torch.Tensor:
    """Decode MoE in two phases around an in-flight miss copy, as the reference's
    ``fused_experts_decode_nvfp4_split`` (patches/moe_fused_nvfp4.patch:189-272): phase A
    computes the routes whose expert was resident (``~miss_mask``), the stream then waits
    ``copy_event``, phase B computes the missed routes and one combine closes both. The
    phases write disjoint route rows of the same workspace, so the result is bit-identical
    to ``fused_experts_decode_nvfp4_marlin``. ``topk_ids`` may be cache-slot ids of a bank of
    slots (position == slot). The shared expert (keyword, resident) runs in phase A."""
    bank = Nvfp4Bank(gate_up_packed, gate_up_scale, gate_up_global, down_packed, down_scale,
                     down_global)
    x = hidden_states
    dev = _check_inputs(x, bank, topk_weights, topk_ids, shared)
    _act_spec(activation, act_alpha, act_limit)
    T, H = x.shape
    K = topk_ids.shape[1]
    mask_a, mask_b = _phase_masks(miss_mask, T * K, dev)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    ws = workspace(decode_workspace_bytes(T, bank, K, shared is not None), dev)
    for phase, mask in ((0, mask_a), (1, mask_b)):
        if phase == 1 and copy_event is not None:
            torch.cuda.current_stream(dev).wait_event(copy_event)
        flags = _lib.PHASE_SHARED if phase == 0 else _lib.PHASE_COMBINE
        _layer(_lib.FTB_PATH_DECODE, x, bank, topk_weights, topk_ids, activation, act_alpha,
               act_limit, apply_router_weight_on_input, shared, out if phase == 1 else None,
               False, False, route_mask=mask, phase=flags, ws=ws)
    return out


def fused_experts_nvfp4(
    hidden_states: torch.Tensor,
    gate_up_packed: torch.Tensor,
    gate_up_scale: torch.Tensor,
    gate_up_global: torch.Tensor,
    down_packed: torch.Tensor,
    down_scale: torch.Tensor,
    down_global: torch.Tensor,
    topk_weights: torch.Tensor,
    topk_ids: torch.Tensor,
    num_experts: int,
    activation: str = "silu",
    apply_router_weight_on_input: bool = False,
    act_alpha: float = 1.702,
    act_limit: float = 7.0,
    *,
    shared: Nvfp4Bank | None = None,
) -> torch.Tensor:
    """Prefill driver. Same contract and result as the decode driver; from
    PREFILL_MIN_TOKENS tokens it runs the tensor-core grouped GEMMs, below that the decode
    GEMVs (which are faster for few routes per expert)."""
    bank = Nvfp4Bank(gate_up_packed, gate_up_scale, gate_up_global, down_packed, down_scale,
                     down_global)
    if num_experts != bank.num_experts:
        raise ValueError(f"num_experts {num_experts} != bank experts {bank.num_experts}")
    layer = moe_prefill if hidden_states.shape[0] >= PREFILL_MIN_TOKENS else moe_decode
    return layer(hidden_states, bank, topk_weights, topk_ids, activation=activation,
                 act_limit=act_limit, act_alpha=act_alpha,
                 apply_router_weight_on_input=apply_router_weight_on_input, shared=shared)


def moe_sum_reduce(ic3: torch.Tensor, topk_ids: torch.Tensor, num_experts: int,
                   shared_out: torch.Tensor | None = None, out: torch.Tensor | None = None):
    """``moe_sum_reduce_triton(ic3, out)`` (patches/moe_fused_nvfp4.patch:147-148): out[t] =
    bf16(sum_k ic3[t, k]) in k order (fp32), then ``+ shared_out`` in bf16 when given. Routes
    with ids outside [0, num_experts) contribute nothing."""
    dev = require_cuda(ic3, topk_ids)
    require(ic3, "ic3", torch.bfloat16)
    require(topk_ids, "topk_ids", torch.int32)
    T, K, H = ic3.shape
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    if shared_out is not None:
        require(shared_out, "shared_out", torch.bfloat16, (T, H))
    st = _lib.load().ftb_moe_combine(ptr(ic3), ptr(topk_ids), ptr(shared_out), T, H, K,
                                     num_experts, ptr(out), stream_handle(dev))
    _lib.check("ftb_moe_combine", st)
    return out


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int):
    """Stable, deterministic permutation: (sorted_ids [cap], expert_ids [cap/bm],
    num_tokens_post_padded int32 [1]); cap = T*top_k + E*(block_size-1)."""
    dev = require_cuda(topk_ids)
    require(topk_ids, "topk_ids", torch.int32)
    T, K = topk_ids.shape
    cap = T * K + num_experts * (block_size - 1)
    sorted_ids = torch.empty(cap, dtype=torch.int32, device=dev)
    expert_ids = torch.empty((cap + block_size - 1) // block_size, dtype=torch.int32, device=dev)
    ntpp = torch.empty(1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws = workspace(lib.ftb_moe_align_workspace_bytes(T, K, num_experts), dev)
    st = lib.ftb_moe_align(ptr(topk_ids), T, K, num_experts, block_size, ptr(sorted_ids),
                           ptr(expert_ids), ptr(ntpp), None, ptr(ws), ws.numel(),
                           stream_handle(dev))
    _lib.check("ftb_moe_align", st)
    return sorted_ids, expert_ids, ntpp
