"""Expert-parallel dispatch/combine on CPU: 2 gloo ranks, the CPU oracle as expert compute.

The EP layer's own host logic (route sort by destination rank, counts exchange, all_to_all
dispatch of rows and metadata, return all_to_all, un-permutation, fixed-order combine) must
reproduce the single-process layer bit for bit. A rank that dies before a collective must
make its peer fail within the process-group timeout, not hang.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

W = 2
E, H, I, T, K = 8, 256, 128, 5, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _to_bf16_tensor(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)


def _ep_worker(rank, port, result_dir, fail_rank):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "freetoken-ox-boost_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from ftb import synth
    from ftb.ep import ExpertParallelMoE, shard_range
    from oracle import moe_oracle as m

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=W, timeout=datetime.timedelta(seconds=5))
    try:
        full = synth.make_bank(E, H, I, seed=3)
        e0, e1 = shard_range(E, rank, W)
        local = full.select(slice(e0, e1)).numpy()
        shared = synth.make_shared(H, I, seed=3).numpy()
        inp = synth.make_inputs(T, H, E, seed=3, stream=rank)
        w, ids = m.topk_softmax(inp.logits.numpy(), K, True)

        def expert_fn(rows, eids, wts):
            out = np.zeros((rows.shape[0], H), np.float32)
            xr = rows.float().numpy()
            for i in range(rows.shape[0]):
                e = int(eids[i])
                if e < 0:
                    continue
                _, _, y = m.expert_forward(xr[i:i + 1], local, e, float("inf"),
                                           np.asarray([float(wts[i])], np.float32))
                out[i] = y[0]
            return _to_bf16_tensor(out)

        def shared_fn(x):
            _, _, y = m.expert_forward(x.float().numpy(), shared, 0, float("inf"), None)
            return _to_bf16_tensor(y)

        def combine_fn(ic3, ids_t, shared_out):
            a = ic3.float().numpy()
            s = a[:, 0].copy()
            for k in range(1, K):
                s = s + a[:, k]
            routed = m.bf16_round(s)
            return _to_bf16_tensor(m.bf16_round(routed + shared_out.float().numpy()))

        ep = ExpertParallelMoE(None, None, E, K, rank, W, expert_fn=expert_fn,
                               shared_fn=shared_fn, combine_fn=combine_fn)
        if rank == fail_rank:
            raise RuntimeError("rank dies before its collectives")
        out = ep.routed_forward(inp.x, torch.from_numpy(w), torch.from_numpy(ids))
        ref = m.moe_layer(inp.x.float().numpy(), full.numpy(), w, ids, shared)["out"]
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out.float().numpy())
        np.save(os.path.join(result_dir, f"ref{rank}.npy"), ref)
    except Exception as exc:  # noqa: BLE001 - record what each rank saw
        with open(os.path.join(result_dir, f"err{rank}.txt"), "w") as f:
            f.write(type(exc).__name__ + ": " + str(exc))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(tmp_path, fail_rank=-1):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, port, str(tmp_path), fail_rank))
             for r in range(W)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("an EP rank did not finish")


def test_ep_two_ranks_bit_exact(tmp_path):
    _run(tmp_path)
    for r in range(W):
        assert not (tmp_path / f"err{r}.txt").exists(), (tmp_path / f"err{r}.txt").read_text()
        out = np.load(tmp_path / f"out{r}.npy")
        ref = np.load(tmp_path / f"ref{r}.npy")
        assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_ep_dead_rank_fails_peer_within_timeout(tmp_path):
    _run(tmp_path, fail_rank=1)
    assert (tmp_path / "err1.txt").exists()
    err0 = tmp_path / "err0.txt"
    assert err0.exists(), "the surviving rank should fail its collective, not complete"
