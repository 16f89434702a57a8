"""Semantic cross-check of the two routing rows whose reference bodies are absent.

The reference calls ``fused_topk`` (softmax top-k + renormalise; patches/layers_moe.patch:100-113)
and ``moe_align_block_size`` (patches/moe_fused_ds_fp4.patch:72,
patches/moe_fused_nvfp4.patch:155-156) from upstream FreeToken code that the patch set does not
contain, so the CPU oracle defines them. vLLM 0.22 (installed in this image) ships CUDA
implementations of the same two functions; this file runs them on the GPU beside ours:
  * fused_topk: ids bit-exact on tie-free logits, weights within 1e-6;
  * moe_align_block_size: vLLM orders routes inside an expert by atomics, so the two are
    compared as the set of route ids in each expert's padded block run, plus the padded total
    and the block -> expert map.
"""
import numpy as np
import pytest
import torch

import ftb

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _vllm():
    try:
        from vllm.model_executor.layers.fused_moe.moe_align_block_size import \
            moe_align_block_size
        from vllm.model_executor.layers.fused_moe.router.fused_topk_router import fused_topk
    except Exception as e:  # noqa: BLE001 - report why the library is not usable here
        pytest.skip(f"vLLM's MoE ops are not importable: {e}")
    return fused_topk, moe_align_block_size


@pytest.mark.parametrize("T,E,K", [(1, 256, 8), (64, 256, 8), (300, 64, 8), (33, 160, 6)])
def test_fused_topk_matches_vllm(T, E, K):
    vllm_topk, _ = _vllm()
    g = torch.Generator(device=DEV).manual_seed(1000 + T)
    logits = torch.randn(T, E, device=DEV, generator=g)
    x = torch.empty(T, 16, dtype=torch.bfloat16, device=DEV)
    w, ids = ftb.fused_topk(x, logits, K, True)
    vw, vids, _ = vllm_topk(x, logits, K, True)
    torch.cuda.synchronize()
    assert torch.equal(ids, vids.to(torch.int32))
    assert float((w - vw).abs().max()) <= 1e-6
    # without renormalisation both return the softmax probabilities themselves
    w2, _ = ftb.fused_topk(x, logits, K, False)
    vw2, _, _ = vllm_topk(x, logits, K, False)
    assert float((w2 - vw2).abs().max()) <= 1e-6


@pytest.mark.parametrize("T,K,E,bm", [(4, 8, 64, 16), (300, 8, 64, 16), (4096, 8, 256, 128),
                                      (17, 6, 160, 64)])
def test_moe_align_matches_vllm_as_sets(T, K, E, bm):
    _, vllm_align = _vllm()
    g = torch.Generator(device=DEV).manual_seed(7 + T)
    ids = torch.randint(0, E, (T, K), device=DEV, dtype=torch.int32, generator=g)
    s, e, n = ftb.moe_align_block_size(ids, bm, E)
    vs, ve, vn = vllm_align(ids, bm, E)
    torch.cuda.synchronize()
    n, vn = int(n.item()), int(vn.item())
    assert n == vn
    s, e = s[:n].cpu().numpy(), e[:n // bm].cpu().numpy()
    vs, ve = vs[:n].cpu().numpy(), ve[:n // bm].cpu().numpy()
    assert np.array_equal(e, ve)
    R = T * K
    for b in range(n // bm):
        ours = sorted(int(v) for v in s[b * bm:(b + 1) * bm] if v < R)
        theirs = sorted(int(v) for v in vs[b * bm:(b + 1) * bm] if v < R)
        if ours != theirs:
            # vLLM may place an expert's routes in a different block of that expert's run:
            # compare the expert's whole run instead
            ex = e[b]
            blocks = np.nonzero(e == ex)[0]
            run = slice(blocks[0] * bm, (blocks[-1] + 1) * bm)
            assert sorted(int(v) for v in s[run] if v < R) == \
                sorted(int(v) for v in vs[run] if v < R), (b, ex)
    # ours is additionally stable: inside an expert, route ids ascend
    flat = ids.flatten().cpu().numpy()
    for b in range(n // bm):
        blk = [int(v) for v in s[b * bm:(b + 1) * bm] if v < R]
        assert all(flat[v] == e[b] for v in blk)
        assert blk == sorted(blk)
