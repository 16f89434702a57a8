"""Expert-parallel NVFP4 MoE layer (BASELINE configs 3 and 4): one process per GPU.

Rank r owns experts [r*E/W, (r+1)*E/W) (contiguous shards) and a replica of the shared
expert. Two transports move tokens to experts and outputs back:

``"p2p"`` (default on CUDA; ``EpGroup``, libftb ``ftb_ep_*``): every rank publishes its
tokens and routes in an exchange region that all ranks map (CUDA IPC over NVLink); the
layer's own kernels pull the routes and rows they need, run the GEMVs over the owned
experts, and each rank pulls its routes' outputs back and combines them. Fixed launch
shapes, no host synchronisation, device-side step flags with bounded waits.

``"nccl"`` (the collective-library baseline, and the CPU/gloo test path), per step:
  1. route (softmax top-k) on the token's home rank;
  2. sort the T*k routes by destination rank (stable, so routes stay in flat order within a
     destination) and exchange the counts (all_to_all of W int64);
  3. dispatch: all_to_all_single of the routes' activation rows and (local expert id,
     routed weight) metadata;
  4. each rank runs the decode kernels on its received routes as top-1 routes, so each
     route's output is bf16(acc * global * w) exactly as on one GPU (the per-route GEMV is
     batch-invariant: its bits do not depend on the other routes);
  5. combine: the reverse all_to_all_single brings each route's output home; the home rank
     sums them in k order (fp32) and adds the shared expert (computed locally) in bf16.
  The counts exchange needs the receive sizes on the host (one device->host read per step).
  The expert, shared-expert and combine computations are pluggable, so this transport also
  runs on CPU gloo ranks in tests (with the CPU oracle as compute).

Both reproduce the single-GPU arithmetic, so the W-rank output equals the 1-GPU output bit
for bit.
"""
from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib
from ._runtime import ptr, require, require_cuda, stream_handle
from .banks import Nvfp4Bank


# ftb_ep_set_trace slots, in step order, and the phases between consecutive slots
EP_TRACE_WORDS = 8
EP_TRACE_PHASES = ("publish", "front_wait", "front_work", "gate_up", "down", "combine_wait",
                   "combine_work")
_U64_MAX = (1 << 64) - 1


def trace_reset(trace: torch.Tensor) -> torch.Tensor:
    """Initialise a [EP_TRACE_WORDS] int64 device tensor for one traced step: the min slots to
    UINT64_MAX (all bits set), the max and end slots to 0."""
    init = torch.tensor([-1, -1, 0, -1, -1, -1, 0, 0], dtype=torch.int64)
    trace.copy_(init.to(trace.device), non_blocking=True)
    return trace


def trace_phases_us(words) -> dict:
    """A traced step's slots (8 unsigned ns timestamps, e.g. ``trace.tolist()``) -> phase
    durations in microseconds, plus ``step`` (publish start to combine end)."""
    t = [int(v) & _U64_MAX for v in words]
    out = {name: (t[i + 1] - t[i]) / 1e3 for i, name in enumerate(EP_TRACE_PHASES)}
    out["step"] = (t[7] - t[0]) / 1e3
    return out


def shard_range(num_experts: int, rank: int, world: int):
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not shard evenly over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


class EpGroup:
    """This rank's member of a peer-memory expert-parallel group (``ftb_ep_*``): an exchange
    region and workspace for steps of exactly ``tokens_per_rank`` tokens, shared by every
    layer of that shape (layers run one after another on the stream).

    Construction is collective: every rank of ``group`` must construct its member together
    (the IPC handles are exchanged with ``all_gather_object``). ``close()`` is collective too
    (it starts with a barrier)."""

    def __init__(self, tokens_per_rank: int, hidden: int, inter: int, num_experts: int,
                 top_k: int, has_shared: bool, rank: int, world: int, group=None,
                 wait_ns: int | None = None):
        lib = _lib.load()
        self.T, self.H, self.I, self.E, self.K = tokens_per_rank, hidden, inter, num_experts, top_k
        self.has_shared, self.rank, self.world, self.group = has_shared, rank, world, group
        self.per = num_experts // world
        h = ctypes.c_void_p()
        _lib.check("ftb_ep_create", lib.ftb_ep_create(rank, world, tokens_per_rank, hidden,
                                                      inter, num_experts, top_k,
                                                      1 if has_shared else 0, ctypes.byref(h)))
        self._h = h
        self.device = torch.device("cuda", torch.cuda.current_device())
        if wait_ns is not None:
            _lib.check("ftb_ep_set_wait_ns", lib.ftb_ep_set_wait_ns(h, int(wait_ns)))
        if world > 1:
            buf = ctypes.create_string_buffer(_lib.EP_HANDLE_BYTES)
            _lib.check("ftb_ep_handle", lib.ftb_ep_handle(h, buf))
            handles = [None] * world
            dist.all_gather_object(handles, bytes(buf.raw), group=group)
            joined = b"".join(handles)
            _lib.check("ftb_ep_open", lib.ftb_ep_open(h, joined))

    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                bank: Nvfp4Bank, shared: Nvfp4Bank | None, act_limit: float = float("inf"),
                out: torch.Tensor | None = None, *, activation: str | None = None,
                act_alpha: float = 1.702, apply_router_weight_on_input: bool = False
                ) -> torch.Tensor:
        """One layer step of this rank's tokens: x holds up to ``tokens_per_rank`` rows (a
        varying serving batch needs no padding; ranks may differ). ``activation=None`` picks
        silu for an infinite ``act_limit`` and swiglu_clamp otherwise (the reference's two GLM
        activations); "swigluoai" takes ``act_alpha``."""
        if self._h is None:
            raise RuntimeError("EpGroup is closed")
        dev = require_cuda(x, topk_weights, topk_ids, bank.gate_up_packed)
        n = x.shape[0] if x.dim() == 2 else -1
        if not 0 <= n <= self.T:
            raise ValueError(f"hidden_states must be [n, {self.H}] with n <= {self.T}")
        require(x, "hidden_states", torch.bfloat16, (n, self.H))
        require(topk_weights, "topk_weights", torch.float32, (n, self.K))
        require(topk_ids, "topk_ids", torch.int32, (n, self.K))
        bank.validate()
        if bank.num_experts != self.per or bank.hidden != self.H or bank.inter != self.I:
            raise ValueError(f"local bank must hold {self.per} experts of H{self.H} I{self.I}")
        if (shared is not None) != self.has_shared:
            raise ValueError("shared expert presence differs from the group's")
        if out is None:
            out = torch.empty(n, self.H, dtype=torch.bfloat16, device=dev)
        from .fused_nvfp4 import _act_spec

        if activation is None:
            activation = "silu" if act_limit == float("inf") else "swiglu_clamp"
        kind, alpha, limit = _act_spec(activation, act_alpha, act_limit)
        b = bank.struct()
        s = shared.struct() if shared is not None else None
        st = _lib.load().ftb_ep_forward_tokens(self._h, n, ptr(x), ptr(topk_weights),
                                               ptr(topk_ids), ctypes.byref(b),
                                               ctypes.byref(s) if s is not None else None, kind,
                                               alpha, limit,
                                               1 if apply_router_weight_on_input else 0,
                                               ptr(out), stream_handle(dev))
        _lib.check("ftb_ep_forward_tokens", st)
        return out

    def set_trace(self, trace: torch.Tensor | None):
        """Record phase timestamps of the following steps into ``trace`` (a contiguous int64
        CUDA tensor of ``EP_TRACE_WORDS``, initialised by ``trace_reset`` before each traced
        step), or stop recording (None). See ``trace_phases_us``."""
        if trace is not None:
            if (trace.dtype != torch.int64 or not trace.is_cuda or trace.numel() != EP_TRACE_WORDS
                    or not trace.is_contiguous()):
                raise ValueError(f"trace must be a contiguous int64 CUDA tensor of "
                                 f"{EP_TRACE_WORDS} words")
        st = _lib.load().ftb_ep_set_trace(self._h, ptr(trace) if trace is not None else None)
        _lib.check("ftb_ep_set_trace", st)
        self._trace = trace

    def status(self, clear: bool = True) -> int:
        """The sticky device status word (synchronises the current stream)."""
        v = _lib.load().ftb_ep_status(self._h, 1 if clear else 0, stream_handle(self.device))
        if v < 0:
            _lib.check("ftb_ep_status", -v)
        return v

    def close(self):
        if self._h is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        h, self._h = self._h, None
        _lib.check("ftb_ep_destroy", _lib.load().ftb_ep_destroy(h))


class ExpertParallelMoE:
    """Expert-parallel routed experts + replicated shared expert of one MoE layer."""

    def __init__(self, local_bank: Nvfp4Bank | None, shared: Nvfp4Bank | None, num_experts: int,
                 top_k: int, rank: int, world: int, group=None, activation: str = "silu",
                 act_limit: float = 7.0, act_alpha: float = 1.702,
                 apply_router_weight_on_input: bool = False, expert_fn: Callable | None = None,
                 shared_fn: Callable | None = None, combine_fn: Callable | None = None,
                 transport: str | None = None, ep_group: EpGroup | None = None):
        if transport is None:  # peer memory for libftb compute on CUDA banks, else NCCL
            on_cuda = local_bank is not None and local_bank.gate_up_packed.is_cuda
            custom = expert_fn or shared_fn or combine_fn
            transport = "p2p" if on_cuda and not custom else "nccl"
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport {transport!r}: expected 'nccl' or 'p2p'")
        if transport == "p2p" and (expert_fn or shared_fn or combine_fn):
            raise ValueError("the p2p transport runs libftb's kernels; custom compute needs 'nccl'")
        self.transport, self.ep_group = transport, ep_group
        self.E, self.K = num_experts, top_k
        self.rank, self.world, self.group = rank, world, group
        self.e0, self.e1 = shard_range(num_experts, rank, world)
        self.per = self.e1 - self.e0
        self.bank, self.shared = local_bank, shared
        self.activation, self.act_limit, self.act_alpha = activation, act_limit, act_alpha
        self.w_on_input = apply_router_weight_on_input
        self.expert_fn = expert_fn or self._gpu_experts
        self.shared_fn = shared_fn or self._gpu_shared
        self.combine_fn = combine_fn or self._gpu_combine
        self.last_local_experts = 0  # distinct local experts hit by the last step's routes

    # --- default (GPU, libftb) computations -------------------------------------------
    def _gpu_experts(self, rows, eids, w):
        from .fused_nvfp4 import moe_decode

        return moe_decode(rows, self.bank, w.view(-1, 1), eids.view(-1, 1),
                          activation=self.activation, act_limit=self.act_limit,
                          act_alpha=self.act_alpha,
                          apply_router_weight_on_input=self.w_on_input)

    def _gpu_shared(self, x):
        if self.shared is None:
            return None
        from .fused_nvfp4 import moe_decode

        T = x.shape[0]
        ones = torch.ones(T, 1, dtype=torch.float32, device=x.device)
        zeros = torch.zeros(T, 1, dtype=torch.int32, device=x.device)
        return moe_decode(x, self.shared, ones, zeros, activation=self.activation,
                          act_limit=self.act_limit, act_alpha=self.act_alpha)

    def _gpu_combine(self, ic3, ids, shared_out):
        from .fused_nvfp4 import moe_sum_reduce

        return moe_sum_reduce(ic3, ids, self.E, shared_out)

    # --- the layer ------------------------------------------------------------------
    def forward(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        from .fused_route import fused_topk

        w, ids = fused_topk(x, logits, self.K, True)
        return self.routed_forward(x, w, ids)

    def routed_forward(self, x: torch.Tensor, topk_weights: torch.Tensor,
                       topk_ids: torch.Tensor) -> torch.Tensor:
        if self.transport == "p2p":
            return self._p2p_forward(x, topk_weights, topk_ids)
        return self._nccl_forward(x, topk_weights, topk_ids)

    def _p2p_forward(self, x, topk_weights, topk_ids):
        if self.ep_group is None:
            self.ep_group = EpGroup(x.shape[0], x.shape[1], self.bank.inter, self.E, self.K,
                                    self.shared is not None, self.rank, self.world, self.group)
        return self.ep_group.forward(x, topk_weights, topk_ids, self.bank, self.shared,
                                     self.act_limit, activation=self.activation,
                                     act_alpha=self.act_alpha,
                                     apply_router_weight_on_input=self.w_on_input)

    def _nccl_forward(self, x: torch.Tensor, topk_weights: torch.Tensor,
                      topk_ids: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        K, W = self.K, self.world
        R = T * K
        flat = topk_ids.reshape(-1).to(torch.int64)
        valid = (flat >= 0) & (flat < self.E)
        dest = torch.where(valid, flat // self.per, torch.zeros_like(flat))
        dest_sorted, order = torch.sort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=W).to(torch.int64)
        send_x = x.index_select(0, order // K)
        eid = torch.where(valid, flat - dest * self.per, torch.full_like(flat, -1))
        meta = torch.stack([eid[order].to(torch.int32),
                            topk_weights.reshape(-1)[order].contiguous().view(torch.int32)], 1)

        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        n_recv = int(sum(rc))
        recv_x = x.new_empty((n_recv, H))
        dist.all_to_all_single(recv_x, send_x, rc, sc, group=self.group)
        recv_meta = meta.new_empty((n_recv, 2))
        dist.all_to_all_single(recv_meta, meta, rc, sc, group=self.group)

        r_eid = recv_meta[:, 0].contiguous()
        r_w = recv_meta[:, 1].contiguous().view(torch.float32)
        if n_recv:
            y = self.expert_fn(recv_x, r_eid, r_w)
            self.last_local_experts = int(torch.unique(r_eid[r_eid >= 0]).numel())
        else:
            y = x.new_empty((0, H))
            self.last_local_experts = 0
        back = x.new_empty((R, H))
        dist.all_to_all_single(back, y.contiguous(), sc, rc, group=self.group)
        ic3 = torch.empty_like(back)
        ic3[order] = back
        shared_out = self.shared_fn(x)
        return self.combine_fn(ic3.view(T, K, H), topk_ids.to(torch.int32).contiguous(),
                               shared_out)
