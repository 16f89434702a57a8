"""Seeded MoE cases shared by the GPU parity tests and ``__graft_entry__.smoke()``:
host-generated banks/inputs, the oracle's answer, and the comparison metrics."""
from __future__ import annotations

import numpy as np
import torch

from ftb import synth
from oracle import moe_oracle as m


def build_case(E, H, I, T, K, *, seed=0, shared=True, router_gemv=False, ids=None):
    bank = synth.make_bank(E, H, I, seed=seed)
    sh = synth.make_shared(H, I, seed=seed) if shared else None
    inp = synth.make_inputs(T, H, E, seed=seed, router_gemv=router_gemv)
    w, oid = m.topk_softmax(inp.logits.numpy(), K, True)
    if ids is not None:
        oid = np.asarray(ids, np.int32)
    return dict(bank=bank, shared=sh, inp=inp, w=w.astype(np.float32), ids=oid, K=K)


def oracle_layer(case, limit=float("inf"), **kw):
    """The oracle's layer on a case; ``kw``: act, alpha, w_on_input (moe_oracle.moe_layer)."""
    x = case["inp"].x.float().numpy()
    sh = case["shared"].numpy() if case["shared"] is not None else None
    return m.moe_layer(x, case["bank"].numpy(), case["w"], case["ids"], sh, limit, **kw)


def to_f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def compare(got: np.ndarray, ref: np.ndarray):
    """(max_abs_rel, fraction of elements not bit-identical)."""
    return m.max_abs_rel(got, ref), float(np.mean(got != ref))
