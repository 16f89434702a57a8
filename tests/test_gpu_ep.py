"""Expert parallelism on the GPU.

* 1 GPU: an ``EpGroup`` of world 1 (the peer-memory path with no peers) returns the
  single-GPU decode bit for bit, over several steps and two layers sharing the group, and over
  steps with fewer tokens than the group's slots (an empty one included); a traced step fills
  the phase timestamps in step order.
* 2 GPUs, both transports (NCCL all_to_all and peer memory): each rank's output equals the
  single-GPU decode of the same tokens with the full bank, bit for bit, over several steps
  (one of them with tokens that route to one rank's experts only, which the other does not
  stage; on the peer-memory transport also steps in which the ranks have different numbers of
  tokens, below the group's slots).
* 2 GPUs, peer memory: a rank that stops stepping makes its peer's bounded flag waits give
  up and report the timeout bit, with the peer's process and GPU still usable.
Multi-GPU cases are skipped with fewer than 2 GPUs.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
W = 2
E, H, I, T, K = 16, 512, 256, 9, 4


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paths():
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "freetoken-ox-boost_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)


def test_ep_world1_p2p_bit_exact():
    import ftb
    from ftb import synth
    from ftb.ep import EpGroup, ExpertParallelMoE

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    banks = [synth.make_bank(E, H, I, seed=s, device=dev) for s in (11, 12)]
    shared = [synth.make_shared(H, I, seed=s, device=dev) for s in (11, 12)]
    group = EpGroup(T, H, I, E, K, True, 0, 1)
    layers = [ExpertParallelMoE(b, s, E, K, 0, 1, transport="p2p", ep_group=group)
              for b, s in zip(banks, shared)]
    try:
        for step in range(4):
            layer = step % 2
            inp = synth.make_inputs(T, H, E, seed=100 + step, device=dev)
            w, ids = ftb.fused_topk(inp.x, inp.logits, K, True)
            if step == 3:
                ids = ids.clone()
                ids[2, 1] = E + 3  # out of range: skipped, status bit 0
            out = layers[layer].routed_forward(inp.x, w, ids)
            ref = ftb.moe_decode(inp.x, banks[layer], w, ids, shared=shared[layer])
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), step
        assert group.status() == 1  # the planted bad id, nothing else
        assert group.status() == 0  # cleared
    finally:
        group.close()


def test_ep_world1_fewer_tokens_than_slots():
    """Steps with fewer tokens than the group's slots (a varying serving batch, no padding):
    each step's output equals the single-GPU decode of its tokens, bit for bit; an empty step
    takes part and returns nothing."""
    import ftb
    from ftb import synth
    from ftb.ep import EpGroup

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    bank = synth.make_bank(E, H, I, seed=17, device=dev)
    shared = synth.make_shared(H, I, seed=17, device=dev)
    group = EpGroup(T, H, I, E, K, True, 0, 1)
    try:
        for step, n in enumerate((T, 4, 1, 0, 7)):
            inp = synth.make_inputs(max(n, 1), H, E, seed=200 + step, device=dev)
            x, logits = inp.x[:n].contiguous(), inp.logits[:n].contiguous()
            w, ids = ftb.fused_topk(x, logits, K, True)
            out = group.forward(x, w, ids, bank, shared)
            torch.cuda.synchronize()
            assert out.shape == (n, H)
            if n:
                ref = ftb.moe_decode(x, bank, w, ids, shared=shared)
                torch.cuda.synchronize()
                assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), (step, n)
        assert group.status() == 0
    finally:
        group.close()


def test_ep_world1_phase_trace():
    """ftb_ep_set_trace: the eight slots of a traced step are filled and in step order."""
    import ftb
    from ftb import synth
    from ftb.ep import EP_TRACE_PHASES, EpGroup, trace_phases_us, trace_reset

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    bank = synth.make_bank(E, H, I, seed=13, device=dev)
    shared = synth.make_shared(H, I, seed=13, device=dev)
    group = EpGroup(T, H, I, E, K, True, 0, 1)
    try:
        inp = synth.make_inputs(T, H, E, seed=7, device=dev)
        w, ids = ftb.fused_topk(inp.x, inp.logits, K, True)
        buf = torch.empty(8, dtype=torch.int64, device=dev)
        group.set_trace(buf)
        trace_reset(buf)
        out = group.forward(inp.x, w, ids, bank, shared)
        torch.cuda.synchronize()
        group.set_trace(None)
        words = [int(v) & ((1 << 64) - 1) for v in buf.tolist()]
        assert all(0 < v < (1 << 63) for v in words), words
        assert words == sorted(words), words
        ph = trace_phases_us(buf.tolist())
        assert set(EP_TRACE_PHASES) <= set(ph) and 0 < ph["step"] < 1e6, ph
        ref = ftb.moe_decode(inp.x, bank, w, ids, shared=shared)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        assert group.status() == 0
    finally:
        group.close()


def _worker(rank, port, out_dir, transport, mode):
    _paths()
    import torch.distributed as dist

    import ftb
    from ftb import synth
    from ftb.ep import EpGroup, ExpertParallelMoE, shard_range

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=W, timeout=datetime.timedelta(seconds=60), device_id=dev)
    result = "error"
    group = None
    try:
        full = synth.make_bank(E, H, I, seed=5, device=dev)
        shared = synth.make_shared(H, I, seed=5, device=dev)
        e0, e1 = shard_range(E, rank, W)
        if transport == "p2p":
            group = EpGroup(T, H, I, E, K, True, rank, W,
                            wait_ns=200_000_000 if mode == "dead_peer" else None)
        ep = ExpertParallelMoE(full.select(slice(e0, e1)), shared, E, K, rank, W,
                               transport=transport, ep_group=group)
        if mode == "dead_peer":
            # rank 1 never steps; rank 0's waits must give up and say so
            if rank == 0:
                inp = synth.make_inputs(T, H, E, seed=5, stream=rank, device=dev)
                ep.forward(inp.x, inp.logits)
                torch.cuda.synchronize()
                st = group.status()
                probe = torch.ones(4, device=dev).sum().item()  # the context still works
                result = f"status={st} probe={probe:.0f}"
            else:
                result = "idle"
        else:
            same = True
            # tokens per step on (rank 0, rank 1): full, then ragged (a serving batch of
            # varying size on the p2p transport)
            counts = [(T, T), (T, T), (T, T)]
            if transport == "p2p":
                counts += [(T, 5), (3, T), (1, 2)]
            for step, nt in enumerate(counts):
                n = nt[rank]
                inp = synth.make_inputs(T, H, E, seed=5 + step, stream=rank, device=dev)
                if step == 2:
                    # tokens 0-3 route to rank 0's experts only: rank 1 must not need them
                    inp.logits[:4, E // 2:] -= 50.0
                inp.x, inp.logits = inp.x[:n].contiguous(), inp.logits[:n].contiguous()
                out = ep.forward(inp.x, inp.logits)
                w, ids = ftb.fused_topk(inp.x, inp.logits, K, True)
                ref = ftb.moe_decode(inp.x, full, w, ids, shared=shared)
                torch.cuda.synchronize()
                same = same and bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
            st = group.status() if group is not None else 0
            result = "same" if same and st == 0 else f"differ (status {st})"
    finally:
        with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
            f.write(result)
        if group is not None:
            group.close()
        dist.destroy_process_group()


def _spawn(tmp_path, transport, mode="parity"):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path), transport, mode))
             for r in range(W)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    return [(tmp_path / f"r{r}.txt").read_text() for r in range(W)]


@pytest.mark.skipif(torch.cuda.device_count() < W, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_ep_two_gpus_bit_exact(tmp_path, transport):
    assert _spawn(tmp_path, transport) == ["same", "same"]


@pytest.mark.skipif(torch.cuda.device_count() < W, reason="needs 2 GPUs")
def test_ep_p2p_dead_peer_times_out(tmp_path):
    r0, r1 = _spawn(tmp_path, "p2p", "dead_peer")
    assert r1 == "idle"
    assert r0 == "status=4 probe=4", r0
