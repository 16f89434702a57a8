"""Expert-parallel NVFP4 MoE layer (BASELINE configs 3 and 4): one process per GPU.

Rank r owns experts [r*E/W, (r+1)*E/W) (contiguous shards) and a replica of the shared
expert. A step on each rank, for its own T tokens:
  1. route (softmax top-k) on the token's home rank;
  2. sort the T*k routes by destination rank (stable, so routes stay in flat order within a
     destination) and exchange the counts (all_to_all of W int64);
  3. dispatch: NCCL all_to_all_single of the routes' activation rows and (local expert id,
     routed weight) metadata;
  4. each rank runs the decode kernels on its received routes as top-1 routes, so each
     route's output is bf16(acc * global * w) exactly as on one GPU (the per-route GEMV is
     batch-invariant: its bits do not depend on the other routes);
  5. combine: the reverse all_to_all_single brings each route's output home; the home rank
     sums them in k order (fp32) and adds the shared expert (computed locally) in bf16.
Because steps 4 and 5 reproduce the single-GPU arithmetic, the W-rank output equals the
1-GPU output bit for bit.

The counts exchange needs the receive sizes on the host (one device->host read per step).
The expert, shared-expert and combine computations are pluggable, so the dispatch/combine
logic also runs on CPU gloo ranks in tests (with the CPU oracle as compute).
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from .banks import Nvfp4Bank


def shard_range(num_experts: int, rank: int, world: int):
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not shard evenly over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


class ExpertParallelMoE:
    """Expert-parallel routed experts + replicated shared expert of one MoE layer."""

    def __init__(self, local_bank: Nvfp4Bank | None, shared: Nvfp4Bank | None, num_experts: int,
                 top_k: int, rank: int, world: int, group=None, activation: str = "silu",
                 act_limit: float = 7.0, expert_fn: Callable | None = None,
                 shared_fn: Callable | None = None, combine_fn: Callable | None = None):
        self.E, self.K = num_experts, top_k
        self.rank, self.world, self.group = rank, world, group
        self.e0, self.e1 = shard_range(num_experts, rank, world)
        self.per = self.e1 - self.e0
        self.bank, self.shared = local_bank, shared
        self.activation, self.act_limit = activation, act_limit
        self.expert_fn = expert_fn or self._gpu_experts
        self.shared_fn = shared_fn or self._gpu_shared
        self.combine_fn = combine_fn or self._gpu_combine
        self.last_local_experts = 0  # distinct local experts hit by the last step's routes

    # --- default (GPU, libftb) computations -------------------------------------------
    def _gpu_experts(self, rows, eids, w):
        from .fused_nvfp4 import moe_decode

        return moe_decode(rows, self.bank, w.view(-1, 1), eids.view(-1, 1),
                          activation=self.activation, act_limit=self.act_limit)

    def _gpu_shared(self, x):
        if self.shared is None:
            return None
        from .fused_nvfp4 import moe_decode

        T = x.shape[0]
        ones = torch.ones(T, 1, dtype=torch.float32, device=x.device)
        zeros = torch.zeros(T, 1, dtype=torch.int32, device=x.device)
        return moe_decode(x, self.shared, ones, zeros, activation=self.activation,
                          act_limit=self.act_limit)

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
