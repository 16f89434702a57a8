"""numpy restatement of the reference's NVFP4 fused-MoE arithmetic: TEST INFRASTRUCTURE.

Imported only by tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs, as the
checker. Every function names the reference file:line it restates (paths relative to the
reference project root; ``patches/*.patch`` lines are diff-file lines).

Parity status (each row of the hot path):
  * e2m1 decode, down GEMV + SwiGLU op order, sigmoid router: PINNED by golden vectors that
    the reference's own Triton kernels produced under Triton's CPU interpreter
    (``tests/golden/make_golden.py``).
  * gate_up GEMV: the reference kernel body is only partly present as diff hunks; it is the
    same GEMV engine as the pinned down GEMV (``nvfp4_marlin_swiglu.py:14-22`` states the
    body is shared), so it is pinned through ``nvfp4_gemv``.
  * softmax top-k (``fused_topk``), ``moe_align_block_size`` and ``moe_sum_reduce_triton``:
    their bodies are upstream FreeToken code absent from the reference, so they are
    DEFINED here (see each docstring) - parity for these rows is unpinned beyond their
    call-site contracts.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32

# E2M1 magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}, sign in bit 3
# (kernel_triton_nvfp4_fused_moe.patch:53-60, ``_e2m1_to_f32``).
E2M1_LUT = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=F32)


def _e4m3_table() -> np.ndarray:
    """FP8-E4M3 (``fn``: bias 7, no inf, S.1111.111 = NaN) byte -> fp32, all 256 bytes.

    Restates the scale decode the reference applies per int32 word
    (``nvfp4_marlin_swiglu.py:96-102``; ``e4m3_u8_to_f32`` of ``e4m3_compat``)."""
    out = np.empty(256, dtype=F32)
    for b in range(256):
        s, e, m = (b >> 7) & 1, (b >> 3) & 15, b & 7
        if e == 15 and m == 7:
            v = np.nan
        elif e == 0:
            v = m * 2.0 ** -9
        else:
            v = (1.0 + m / 8.0) * 2.0 ** (e - 7)
        out[b] = -v if s else v
    return out


E4M3_TABLE = _e4m3_table()


def e4m3_decode(u8: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(u8, dtype=np.uint8)]


def e2m1_decode(codes: np.ndarray) -> np.ndarray:
    return E2M1_LUT[np.asarray(codes, dtype=np.uint8) & 15]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16, returned as fp32 values (the ``.to(tl.bfloat16)`` stores
    of ``nvfp4_marlin_swiglu.py:116,129``). NaN stays NaN."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    r = np.where(np.isnan(x), np.uint32(0x7FC00000), r)
    return r.view(F32)


def bf16_trunc(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 by truncation (round toward zero): the cast Triton's CPU interpreter
    performs for ``.to(tl.bfloat16)``, used only to replay golden vectors the reference
    kernels produced under that interpreter. GPU Triton and this build round to nearest even."""
    x = np.ascontiguousarray(x, dtype=F32)
    return (x.view(np.uint32) & np.uint32(0xFFFF0000)).view(F32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def unpack_codes(packed: np.ndarray) -> np.ndarray:
    """[..., K/2] bytes -> [..., K] codes; byte b holds k=2b (low nibble) and k=2b+1 (high
    nibble) (``b12x_repack.py:11-13``; int32 word w holds k=8w+j in nibble j,
    ``kernel_triton_nvfp4_fused_moe.patch:35``)."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = p & 15
    out[..., 1::2] = p >> 4
    return out


def dequant_rows(packed: np.ndarray, scale_u8: np.ndarray) -> np.ndarray:
    """Exact e2m1 x e4m3 values [..., K] (no global scale). Exact in fp32 and in bf16: the
    product has at most 6 significant bits (kernel_triton_nvfp4_fused_moe.patch:92-94)."""
    codes = unpack_codes(packed)
    sc = e4m3_decode(scale_u8)
    return e2m1_decode(codes) * np.repeat(sc, 16, axis=-1)


def nvfp4_gemv(a: np.ndarray, packed: np.ndarray, scale_u8: np.ndarray, block_kw: int = 32) -> np.ndarray:
    """One NVFP4 weight matrix times activation rows, in the reference kernel's op order.

    a [R, K] fp32 (bf16-valued), packed [N, K/2] u8, scale_u8 [N, K/16] e4m3 bits
    -> acc [R, N] fp32, BEFORE the global scale.

    Op order of ``_decode_nvfp4_marlin_swiglu_kernel`` (``nvfp4_marlin_swiglu.py:82-120``) and
    ``_decode_nvfp4_marlin_kernel`` (``kernel_triton_nvfp4_fused_moe.patch:211-231``): per
    int32 word w (8 k): ``acc_w = sum_{j=0..7} a[8w+j] * lut[code_j]`` accumulated in j order;
    ``partial[w % KW] += acc_w * scale[w // 2]`` over K-iterations in order; then a sum over
    the KW lanes (``tl.sum``: its order is unspecified; lanes are added 0..KW-1 here, the
    order Triton's CPU interpreter uses, so the golden vectors match bit for bit).
    """
    a = np.ascontiguousarray(a, dtype=F32)
    R, K = a.shape
    N = packed.shape[0]
    assert packed.shape[1] * 2 == K and scale_u8.shape[1] * 16 == K and K % 16 == 0
    W = K // 8
    vals = e2m1_decode(unpack_codes(packed)).reshape(N, W, 8)           # [N, W, 8]
    sc = np.repeat(e4m3_decode(scale_u8), 2, axis=1)                    # [N, W]
    av = a.reshape(R, W, 8)
    acc_w = av[:, None, :, 0] * vals[None, :, :, 0]
    for j in range(1, 8):
        acc_w = acc_w + av[:, None, :, j] * vals[None, :, :, j]          # [R, N, W]
    contrib = acc_w * sc[None]                                          # [R, N, W]
    iters = -(-W // block_kw)
    if iters * block_kw != W:
        pad = np.zeros((R, N, iters * block_kw - W), dtype=F32)
        contrib = np.concatenate([contrib, pad], axis=2)
    contrib = contrib.reshape(R, N, iters, block_kw)
    partial = contrib[:, :, 0, :]
    for it in range(1, iters):
        partial = partial + contrib[:, :, it, :]
    acc = partial[:, :, 0].copy()
    for lane in range(1, block_kw):
        acc = acc + partial[:, :, lane]
    return acc


def f32_sigmoid(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=F32)
    with np.errstate(over="ignore"):
        return (F32(1.0) / (F32(1.0) + np.exp(-x))).astype(F32)


def swiglu(gate: np.ndarray, up: np.ndarray, limit: float = float("inf"), rnd=None,
           act: str | None = None, alpha: float = 1.702) -> np.ndarray:
    """The activation between the GEMVs, in fp32 with one bf16 rounding (``_run_act``,
    ``patches/moe_fused_nvfp4.patch:12-22``):

    * silu / swiglu_clamp (``act`` None): ``bf16((min(g,L) * sigmoid(min(g,L))) *
      clamp(u,-L,L))`` (``kernel_triton_dsv4_fused_moe.patch:22-36`` ``_swiglu_kernel``;
      ``nvfp4_marlin_swiglu.py:109-116``; C++ twin ``kernel_csrc_cpu_moe_cpu_moe_ext.patch:7-13``).
      ``limit > 0`` enables the clamps exactly as ``HAS_LIMIT=limit > 0``; +inf is plain silu.
    * ``act="swigluoai"``: ``swigluoai_and_mul(gate_up, out, alpha, limit)`` (called at
      ``patches/moe_fused_nvfp4.patch:12-14``; its body is upstream and absent, so this
      restates the published GPT-OSS gated unit): g' = min(g, L), u' = clamp(u, -L, L),
      ``bf16((g' * sigmoid(alpha * g')) * (u' + 1))``."""
    g = np.asarray(gate, dtype=F32)
    u = np.asarray(up, dtype=F32)
    if limit > 0:
        L = F32(limit)
        g = np.minimum(g, L)
        u = np.minimum(np.maximum(u, -L), L)
    if act == "swigluoai":
        return (rnd or bf16_round)((g * f32_sigmoid(F32(alpha) * g)) * (u + F32(1)))
    return (rnd or bf16_round)((g * f32_sigmoid(g)) * u)


def f32_log2_ceil(x: np.ndarray) -> np.ndarray:
    """ceil(log2(x)) of positive normal fp32 values, exactly (``_log2_ceil``, imported at
    ``patches/kernel_triton_dsv4_fused_moe.patch:10`` from the DSV4 FP8 linear module; its body
    is upstream and absent, so this DEFINES it as the exact mathematical ceiling)."""
    m, e = np.frexp(np.asarray(x, np.float64))  # x = m 2^e, m in [0.5, 1)
    return np.where(m == 0.5, e - 1, e).astype(np.int64)


def e4m3_rn(v: np.ndarray) -> np.ndarray:
    """fp32 -> the nearest E4M3 (fn) value, ties to even mantissa, for |v| <= 448 (the callers
    clamp first), as fp32: normal binades [2^k, 2^k+1) for k >= -6 step 2^(k-3), below 2^-6
    the subnormal step 2^-9 (``.to(tl.float8e4nv)``)."""
    v = np.asarray(v, np.float64)
    a = np.abs(v)
    _, e = np.frexp(a)
    k = np.maximum(e - 1, -6)
    step = np.ldexp(1.0, k - 3)
    q = np.minimum(np.rint(a / step) * step, 448.0)
    return np.copysign(q, v).astype(F32)


def fp8_block128_roundtrip(act: np.ndarray) -> np.ndarray:
    """The ds_fp4 layers' FP8 round trip of the fp32 activation, per 128 consecutive elements of
    a row (``_swiglu_kernel`` with QUANT, ``patches/kernel_triton_dsv4_fused_moe.patch:25-35``):
    amax = max(max|a|, 1e-4); e = _log2_ceil(amax * (1/448)) (fp32 multiply); sc = 2^e;
    q = fp8e4nv(clamp(a / sc, -448, 448)); result q * sc (fp32; exact in bf16)."""
    a = np.asarray(act, F32)
    shp = a.shape
    b = a.reshape(-1, shp[-1] // 128, 128)
    amax = np.maximum(np.abs(b).max(-1), F32(1e-4)).astype(F32)
    e = f32_log2_ceil((amax * F32(1.0 / 448.0)).astype(F32))
    sc = np.ldexp(1.0, e)[..., None]
    q = e4m3_rn(np.clip(b.astype(np.float64) / sc, -448.0, 448.0))
    return (q.astype(np.float64) * sc).astype(F32).reshape(shp)


# ----------------------------------------------------------------------------------------
# Router
# ----------------------------------------------------------------------------------------

def router_logits(x: np.ndarray, gate_w: np.ndarray) -> np.ndarray:
    """``F.linear(x.float(), gate.float())`` (``patches/models_glm_moe_dsa_moe.patch:129``):
    fp32 GEMV, summation order unspecified (cuBLAS); computed here in float64 then rounded."""
    return (np.asarray(x, np.float64) @ np.asarray(gate_w, np.float64).T).astype(F32)


def topk_ids_desc(score: np.ndarray, top_k: int) -> np.ndarray:
    """Top-k indices by descending score, lowest index first on ties (the tie-break of
    ``fused_route.py:51`` and of a sorted ``torch.topk``). NaN ranks below every number."""
    s = np.asarray(score, dtype=F32)
    key = np.where(np.isnan(s), -np.inf, s).astype(np.float64)
    order = np.lexsort((np.broadcast_to(np.arange(s.shape[-1]), s.shape), -key), axis=-1)
    return order[..., :top_k].astype(np.int32)


def topk_softmax(logits: np.ndarray, top_k: int, renormalize: bool = True):
    """Softmax router with renormalisation: the generic ``fused_topk(hidden, gating_output,
    topk, renormalize)`` of ``OffloadMoELayer.decode_forward`` (``patches/layers_moe.patch:100-113``).

    Its body is upstream and absent, so this DEFINES it: p = softmax(logits) in fp32
    (max-subtracted); ids = top-k of the logits (softmax is monotonic, so selecting on logits
    equals selecting on exact probabilities; ties -> lowest index); w = p[ids], renormalised
    by their plain sum in k order when ``renormalize``."""
    lg = np.asarray(logits, dtype=F32)
    ids = topk_ids_desc(lg, top_k)
    m = lg.max(axis=-1, keepdims=True)
    e = np.exp(lg - m).astype(F32)
    p = (e / e.sum(axis=-1, dtype=F32, keepdims=True)).astype(F32)
    w = np.take_along_axis(p, ids.astype(np.int64), axis=-1)
    if renormalize:
        s = w[..., 0].copy()
        for k in range(1, top_k):
            s = s + w[..., k]
        w = (w / s[..., None]).astype(F32)
    return w.astype(F32), ids


def f32_sqrtsoftplus(x: np.ndarray) -> np.ndarray:
    """sqrt(softplus(x)) in its overflow-stable fp32 form max(x, 0) + log(1 + exp(-|x|))
    (``overlay/freetoken/kernel/triton/fused_route.py:39-43``)."""
    x = np.asarray(x, dtype=F32)
    with np.errstate(over="ignore", invalid="ignore"):
        sp = (np.maximum(x, F32(0)) + np.log(F32(1) + np.exp(-np.abs(x)))).astype(F32)
        return np.sqrt(sp).astype(F32)


def fused_route_sigmoid(logits: np.ndarray, bias: np.ndarray, top_k: int, renorm: bool,
                        scaling: float, act: str = "sigmoid", n_rank: int = 0):
    """GLM router epilogue ``_fused_route_kernel`` (``overlay/freetoken/kernel/triton/fused_route.py:28-62``):
    sc = sigmoid(l) (``act="sigmoid"``) or sqrt(softplus(l)) (``act="sqrtsoftplus"``, :39-45);
    s4c = sc + bias (NaN -> -FLT_MAX); ids by iterative first-index argmax; w = sc[ids]; wsum
    accumulated in selection order; w = w / (wsum + 1e-20) if renorm; w *= scaling. Ids are
    clamped to [0, E-1].

    ``n_rank > 0`` restates ``_fused_route_ext_kernel`` (:85-121): the selection runs n_rank
    rounds, the first top_k of which are the routing result, and also returns the ranked list
    (rank_ids [T, n_rank], rank_scores [T, n_rank] = sc of each, 0 where it is NaN)."""
    lg = np.asarray(logits, dtype=F32)
    T, E = lg.shape
    sc = f32_sqrtsoftplus(lg) if act == "sqrtsoftplus" else f32_sigmoid(lg)
    s4c = (sc + np.asarray(bias, dtype=F32)[None, :]).astype(F32)
    s4c = np.where(np.isnan(s4c), F32(-3.4028234663852886e38), s4c)
    rounds = max(top_k, n_rank)
    ids = np.zeros((T, top_k), np.int32)
    w = np.zeros((T, top_k), F32)
    rid = np.zeros((T, n_rank), np.int32)
    rsc = np.zeros((T, n_rank), F32)
    for t in range(T):
        row = s4c[t].copy()
        wsum = F32(0.0)
        for k in range(rounds):
            idx = int(np.argmax(row))  # first index of the max
            idx = min(max(idx, 0), E - 1)
            val = sc[t, idx]
            if k < n_rank:
                rid[t, k] = idx
                rsc[t, k] = val if val == val else F32(0)
            if k < top_k:
                ids[t, k] = idx
                w[t, k] = val
                wsum = F32(wsum + val)
            row[idx] = -np.inf
        for k in range(top_k):
            v = w[t, k]
            if renorm:
                v = F32(v / F32(wsum + F32(1e-20)))
            w[t, k] = F32(v * F32(scaling))
    if n_rank:
        return w, ids, rid, rsc
    return w, ids


# ----------------------------------------------------------------------------------------
# Token -> expert permutation
# ----------------------------------------------------------------------------------------

def moe_align(topk_ids: np.ndarray, num_experts: int, block_m: int):
    """``moe_align_block_size(topk_ids, BLOCK_M, num_experts)`` -> ``(sorted_ids, expert_ids,
    num_tokens_post_padded)`` (call sites ``patches/moe_fused_ds_fp4.patch:72`` and
    ``patches/moe_fused_nvfp4.patch:155-156``; body upstream and absent).

    DEFINED here as a stable counting sort: flat routes r = t*top_k + k ordered by expert,
    ties by r; each expert's segment padded to a multiple of ``block_m`` with the sentinel
    ``T*top_k``; ``expert_ids[b]`` is the expert of block b. Also returns the per-expert
    unpadded offsets [E+1] and the unpadded sorted route list [T*top_k]."""
    ids = np.asarray(topk_ids, dtype=np.int64).reshape(-1)
    R = ids.size
    counts = np.bincount(ids, minlength=num_experts)[:num_experts]
    order = np.argsort(ids, kind="stable").astype(np.int32)
    offsets = np.zeros(num_experts + 1, np.int64)
    offsets[1:] = np.cumsum(counts)
    padded = ((counts + block_m - 1) // block_m) * block_m
    sorted_ids = np.full(int(padded.sum()), R, dtype=np.int32)
    expert_ids = np.zeros(int(padded.sum()) // block_m, dtype=np.int32)
    pos = 0
    for e in range(num_experts):
        c = int(counts[e])
        sorted_ids[pos:pos + c] = order[offsets[e]:offsets[e + 1]]
        expert_ids[pos // block_m:(pos + int(padded[e])) // block_m] = e
        pos += int(padded[e])
    return sorted_ids, expert_ids, int(padded.sum()), offsets.astype(np.int32), order


# ----------------------------------------------------------------------------------------
# The layer
# ----------------------------------------------------------------------------------------

def _f16_to_f32(g) -> np.ndarray:
    """Per-row global scale: fp16 values (or their uint16 bits) -> fp32."""
    g = np.asarray(g)
    if g.dtype == np.uint16:
        g = g.view(np.float16)
    return g.astype(F32)


def expert_forward(a: np.ndarray, bank: dict, e: int, limit: float, route_w=None, rnd=None,
                   act: str | None = None, alpha: float = 1.702, w_on_input: bool = False,
                   h_quant: str | None = None):
    """One expert for the rows ``a`` [R, H]: gate_up GEMV -> ic1 (bf16, x global) ->
    SwiGLU -> h (bf16) -> down GEMV -> ic3 = bf16(acc * global * w) (``route_w`` None = no
    routed weight, the shared-expert case).

    Follows ``fused_experts_decode_nvfp4_marlin`` (``patches/moe_fused_nvfp4.patch:136-152``):
    ``_decode_gemm_marlin`` with ``mul_routed_weight=False`` for gate_up, activation, then
    the down GEMV with the routed weight applied in fp32 before the bf16 store
    (``nvfp4_marlin_swiglu.py:120-129``). Rows 0..I-1 of gate_up are gate, I..2I-1 up.
    ``w_on_input`` (``apply_router_weight_on_input=True``) moves the routed weight to the
    gate_up GEMV's epilogue, as the driver's ``mul_routed_weight`` arguments do
    (``patches/moe_fused_nvfp4.patch:138,145``). ``h_quant="fp8_block128"``: the activation
    takes ``fp8_block128_roundtrip`` before its bf16 store, as the ds_fp4 decode does
    (``fused_swiglu(gate_up, swiglu_limit, quant=True)``, ``patches/moe_fused_ds_fp4.patch:33``)."""
    gu_p, gu_s, gu_g = bank["gate_up_packed"][e], bank["gate_up_scale"][e], bank["gate_up_global"][e]
    dn_p, dn_s, dn_g = bank["down_packed"][e], bank["down_scale"][e], bank["down_global"][e]
    rnd = rnd or bf16_round
    I = gu_p.shape[0] // 2
    rw = None if route_w is None else np.asarray(route_w, F32)[:, None]
    acc1 = nvfp4_gemv(a, gu_p, gu_s) * _f16_to_f32(gu_g)[None, :]
    if w_on_input and rw is not None:
        acc1 = acc1 * rw
    ic1 = rnd(acc1)
    if h_quant == "fp8_block128":
        h = rnd(fp8_block128_roundtrip(swiglu(ic1[:, :I], ic1[:, I:], limit, lambda v: v, act,
                                              alpha)))
    elif h_quant is None:
        h = swiglu(ic1[:, :I], ic1[:, I:], limit, rnd, act, alpha)
    else:
        raise ValueError(f"h_quant {h_quant!r}")
    acc3 = nvfp4_gemv(h, dn_p, dn_s) * _f16_to_f32(dn_g)[None, :]
    if rw is not None and not w_on_input:
        acc3 = acc3 * rw
    return ic1, h, rnd(acc3)


def moe_layer(x: np.ndarray, bank: dict, topk_w: np.ndarray, topk_ids: np.ndarray,
              shared: dict | None = None, limit: float = float("inf"), act: str | None = None,
              alpha: float = 1.702, w_on_input: bool = False, h_quant: str | None = None) -> dict:
    """Full decode/prefill layer on bf16-valued fp32 inputs.

    routed = ``moe_sum_reduce_triton(ic3)`` = bf16(sum over k of fp32(ic3[t,k]), k in order)
    (``patches/moe_fused_nvfp4.patch:147-148``; body absent -> DEFINED as an fp32 sum in k
    order); then ``out = routed + shared_experts(x)`` in bf16, routed first
    (``patches/models_glm_moe_dsa_moe.patch:203-206``)."""
    x = np.asarray(x, F32)
    T, H = x.shape
    K = topk_ids.shape[1]
    I = bank["gate_up_packed"].shape[1] // 2
    ic1 = np.zeros((T, K, 2 * I), F32)
    h = np.zeros((T, K, I), F32)
    ic3 = np.zeros((T, K, H), F32)
    ids = np.asarray(topk_ids, np.int64)
    for e in np.unique(ids):
        tt, kk = np.nonzero(ids == e)
        a, b, c = expert_forward(x[tt], bank, int(e), limit, np.asarray(topk_w, F32)[tt, kk],
                                 act=act, alpha=alpha, w_on_input=w_on_input,
                                 h_quant=h_quant)
        ic1[tt, kk], h[tt, kk], ic3[tt, kk] = a, b, c
    s = ic3[:, 0, :].copy()
    for k in range(1, K):
        s = s + ic3[:, k, :]
    routed = bf16_round(s)
    out = {"ic1": ic1, "h": h, "ic3": ic3, "routed": routed, "out": routed}
    if shared is not None:
        s1, sh, s3 = expert_forward(x, shared, 0, limit, None, act=act, alpha=alpha,
                                    h_quant=h_quant)
        out.update(shared_ic1=s1, shared_h=sh, shared_out=s3, out=bf16_round(routed + s3))
    return out


def moe_layer_f64(x, bank, topk_w, topk_ids, shared=None, limit=float("inf")):
    """Dequantise-then-float64 reference with NO intermediate rounding (for reporting how far
    both the oracle and the GPU path sit from exact arithmetic)."""
    x = np.asarray(x, np.float64)
    T, H = x.shape
    K = topk_ids.shape[1]

    def dq(p, s, g):
        return dequant_rows(p, s).astype(np.float64) * np.asarray(g, np.float64)[:, None]

    def act(gu):
        I = gu.shape[-1] // 2
        g, u = gu[..., :I], gu[..., I:]
        if limit > 0:
            g = np.minimum(g, limit)
            u = np.clip(u, -limit, limit)
        return g / (1.0 + np.exp(-g)) * u

    out = np.zeros((T, H))
    for e in np.unique(topk_ids):
        tt, kk = np.nonzero(np.asarray(topk_ids) == e)
        wgu = dq(bank["gate_up_packed"][e], bank["gate_up_scale"][e], bank["gate_up_global"][e])
        wd = dq(bank["down_packed"][e], bank["down_scale"][e], bank["down_global"][e])
        y = act(x[tt] @ wgu.T) @ wd.T
        np.add.at(out, tt, y * np.asarray(topk_w, np.float64)[tt, kk][:, None])
    if shared is not None:
        wgu = dq(shared["gate_up_packed"][0], shared["gate_up_scale"][0], shared["gate_up_global"][0])
        wd = dq(shared["down_packed"][0], shared["down_scale"][0], shared["down_global"][0])
        out += act(x @ wgu.T) @ wd.T
    return out


def max_abs_rel(got: np.ndarray, ref: np.ndarray) -> float:
    """max|got - ref| / max|ref|: the north-star tolerance metric (bar 1e-2)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(got - ref).max() / (den if den > 0 else 1.0))
