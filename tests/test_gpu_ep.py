"""Expert parallelism on 2 GPUs (NCCL): each rank's output equals the single-GPU decode of
the same tokens with the full bank, bit for bit. Skipped with fewer than 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
W = 2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, out_dir):
    import sys

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "freetoken-ox-boost_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import ftb
    from ftb import synth
    from ftb.ep import ExpertParallelMoE, shard_range

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=W, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        E, H, I, T, K = 16, 512, 256, 9, 4
        full = synth.make_bank(E, H, I, seed=5, device=dev)
        shared = synth.make_shared(H, I, seed=5, device=dev)
        e0, e1 = shard_range(E, rank, W)
        ep = ExpertParallelMoE(full.select(slice(e0, e1)), shared, E, K, rank, W)
        inp = synth.make_inputs(T, H, E, seed=5, stream=rank, device=dev)
        out = ep.forward(inp.x, inp.logits)
        w, ids = ftb.fused_topk(inp.x, inp.logits, K, True)
        ref = ftb.moe_decode(inp.x, full, w, ids, shared=shared)
        torch.cuda.synchronize()
        same = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
        with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
            f.write("same" if same else "differ")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < W, reason="needs 2 GPUs")
def test_ep_two_gpus_bit_exact(tmp_path):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path))) for r in range(W)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    for r in range(W):
        assert (tmp_path / f"r{r}.txt").read_text() == "same"
