"""Generate the golden vectors under tests/golden/ by running the REFERENCE's own Triton
kernels on the CPU (Triton's interpreter, TRITON_INTERPRET=1).

Run here, in the container that has the reference checkout (never on the GPU box):
    python tests/golden/make_golden.py /path/to/reference

Kernels executed (unmodified, imported from the reference tree):
  * ``_fused_route_kernel`` via ``fused_route`` (sigmoid and sqrtsoftplus scores) and
    ``_fused_route_ext_kernel`` via ``fused_route_ranked`` - overlay/freetoken/kernel/triton/fused_route.py
  * ``_decode_nvfp4_marlin_swiglu_kernel`` - overlay/freetoken/kernel/triton/nvfp4_marlin_swiglu.py
    (the down GEMV with the activation folded in; same GEMV body as the gate_up kernel)
  * ``_e2m1_to_f32`` / ``_e2m1_to_bf16`` - the added lines of
    patches/kernel_triton_nvfp4_fused_moe.patch (only the function bodies, exec'd as-is)
The reference imports ``freetoken.kernel.triton.e4m3_compat`` (upstream, absent); a shim
module provides its two names: ``e4m3_native_cx() -> False`` and ``e4m3_u8_to_f32``, an
E4M3 bit decode checked here against torch's float8_e4m3fn conversion for all 256 bytes.
Inputs are seeded; outputs are stored as raw bit patterns (.npz, a few hundred KB total).
"""
from __future__ import annotations

import importlib.util
import os
import sys
import tempfile

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
if len(sys.argv) < 2:
    sys.exit("usage: python tests/golden/make_golden.py /path/to/reference-checkout")
REF = sys.argv[1]

SHIM = '''
import triton
import triton.language as tl


def e4m3_native_cx():
    return False


@triton.jit
def e4m3_u8_to_f32(u):
    u = u.to(tl.int32)
    s = (u >> 7) & 1
    e = (u >> 3) & 15
    m = u & 7
    normal = ((e + 120) << 23) | (m << 20)
    v = tl.where(e == 0, m.to(tl.float32) * 0.001953125, normal.to(tl.float32, bitcast=True))
    v = tl.where((e == 15) & (m == 7), float("nan"), v)
    return tl.where(s == 1, -v, v)
'''


def _install_shim() -> str:
    d = tempfile.mkdtemp(prefix="ftb_golden_shim_")
    pkg = os.path.join(d, "freetoken", "kernel", "triton")
    os.makedirs(pkg)
    for sub in ("freetoken", "freetoken/kernel", "freetoken/kernel/triton"):
        open(os.path.join(d, sub, "__init__.py"), "w").close()
    with open(os.path.join(pkg, "e4m3_compat.py"), "w") as f:
        f.write(SHIM)
    sys.path.insert(0, d)
    return d


def _load(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, os.path.join(REF, path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def check_shim() -> None:
    from freetoken.kernel.triton.e4m3_compat import e4m3_u8_to_f32

    globals()["_shim_e4m3"] = e4m3_u8_to_f32  # jit bodies resolve names from module globals

    @triton.jit
    def k(src, dst):
        offs = tl.arange(0, 256)
        tl.store(dst + offs, _shim_e4m3(tl.load(src + offs)))  # noqa: F821

    src = torch.arange(256, dtype=torch.uint8)
    dst = torch.empty(256, dtype=torch.float32)
    k[(1,)](src, dst)
    ref = src.view(torch.float8_e4m3fn).float()
    same = (dst == ref) | (torch.isnan(dst) & torch.isnan(ref))
    assert bool(same.all()), "e4m3 shim disagrees with torch.float8_e4m3fn"


def e2m1_table() -> dict:
    """Exec the reference's _e2m1_to_f32 / _e2m1_to_bf16 bodies from the patch."""
    text = open(os.path.join(REF, "patches/kernel_triton_nvfp4_fused_moe.patch")).read().splitlines()
    added = [ln[1:] for ln in text if ln.startswith("+") and not ln.startswith("+++")]
    src, keep, buf = [], False, ["@triton.jit"]  # the first decorator is a context line
    for ln in added:
        if ln.startswith("@triton.jit"):
            keep = False
            buf = [ln]
            continue
        if ln.startswith("def _e2m1_to_"):
            keep = True
            src.extend(buf)
        if keep:
            src.append(ln)
            if ln.strip().startswith("return"):
                keep = False
                src.append("")
    ns = {"triton": triton, "tl": tl}
    exec(compile("\n".join(src), "kernel_triton_nvfp4_fused_moe.patch", "exec"), ns)
    globals()["_ref_e2m1_f32"] = ns["_e2m1_to_f32"]
    globals()["_ref_e2m1_bf16"] = ns["_e2m1_to_bf16"]

    @triton.jit
    def k(codes, o32, o16):
        offs = tl.arange(0, 16)
        c = tl.load(codes + offs)
        tl.store(o32 + offs, _ref_e2m1_f32(c))  # noqa: F821
        tl.store(o16 + offs, _ref_e2m1_bf16(c))  # noqa: F821

    codes = torch.arange(16, dtype=torch.int32)
    o32 = torch.empty(16, dtype=torch.float32)
    o16 = torch.empty(16, dtype=torch.bfloat16)
    k[(1,)](codes, o32, o16)
    return dict(codes=codes.numpy(), f32=o32.numpy(), bf16_bits=_bits16(o16))


def route_cases(fr) -> dict:
    out = {}
    g = torch.Generator().manual_seed(11)
    cases = [
        ("e256_k8_renorm", 8, 256, 8, True, 2.5, None),
        ("e160_k6_norenorm", 5, 160, 6, False, 1.0, None),
        ("ties", 4, 64, 8, True, 1.0, "ties"),
        ("nan_rows", 3, 64, 4, True, 1.0, "nan"),
    ]
    for name, T, E, K, renorm, scaling, kind in cases:
        lg = torch.randn(T, E, generator=g)
        bias = torch.randn(E, generator=g) * 0.1
        if kind == "ties":
            lg = torch.round(lg * 2) / 2  # many equal logits
            bias = torch.zeros(E)
        if kind == "nan":
            lg[0, 5] = float("nan")
            lg[1, :] = float("nan")
        w, ids = fr.fused_route(lg, bias, K, renorm, scaling)
        out[name] = dict(logits=lg.numpy(), bias=bias.numpy(), top_k=K, renorm=int(renorm),
                         scaling=np.float32(scaling), w=w.numpy(), ids=ids.numpy())
    return out


def route_variant_cases(fr) -> dict:
    """sqrt(softplus) scores through ``fused_route(..., act="sqrtsoftplus")`` and the ranked list
    of ``fused_route_ranked`` (both from fused_route.py)."""
    out = {}
    g = torch.Generator().manual_seed(33)
    for name, T, E, K, renorm, scaling, kind in [
        ("sqrtsoftplus_e256_k8", 6, 256, 8, True, 2.5, None),
        ("sqrtsoftplus_e64_k4_nan", 3, 64, 4, False, 1.0, "nan"),
    ]:
        lg = torch.randn(T, E, generator=g) * 3.0
        bias = torch.randn(E, generator=g) * 0.1
        if kind == "nan":
            lg[0, 7] = float("nan")
            lg[2, :] = float("nan")
        w, ids = fr.fused_route(lg, bias, K, renorm, scaling, act="sqrtsoftplus")
        out[name] = dict(logits=lg.numpy(), bias=bias.numpy(), top_k=K, renorm=int(renorm),
                         scaling=np.float32(scaling), act="sqrtsoftplus", w=w.numpy(),
                         ids=ids.numpy())
    for name, T, E, K, NR, renorm, scaling, kind in [
        ("ranked_e256_k8_r16", 5, 256, 8, 16, True, 2.5, None),
        ("ranked_e64_k4_r12_nan", 3, 64, 4, 12, True, 1.0, "nan"),
    ]:
        lg = torch.randn(T, E, generator=g)
        bias = torch.randn(E, generator=g) * 0.1
        if kind == "nan":
            lg[1, 3] = float("nan")
            lg[2, :] = float("nan")
        w, ids, rid, rsc = fr.fused_route_ranked(lg, bias, K, renorm, scaling, n_rank=NR)
        out[name] = dict(logits=lg.numpy(), bias=bias.numpy(), top_k=K, n_rank=NR,
                         renorm=int(renorm), scaling=np.float32(scaling), w=w.numpy(),
                         ids=ids.numpy(), rank_ids=rid.numpy(), rank_scores=rsc.numpy())
    return out


def down_swiglu_cases(ms) -> dict:
    out = {}
    g = torch.Generator().manual_seed(22)
    lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6])
    cases = [
        ("h256_i256_inf", 3, 256, 256, 3, 2, float("inf")),
        ("h384_i512_lim7", 4, 384, 512, 2, 4, 7.0),
        ("h128_i768_lim10", 2, 128, 768, 2, 3, 10.0),
    ]
    for name, S, H, I, T, K, limit in cases:
        routes = T * K
        gate_up = (torch.randn(routes, 2 * I, generator=g) * 2.0).to(torch.bfloat16)
        packed = torch.randint(0, 256, (S, H, I // 2), generator=g, dtype=torch.uint8)
        w = torch.randn(S, H, I // 16, 16, generator=g) * 0.02
        scale = (w.abs().amax(-1) / 6).to(torch.float8_e4m3fn).view(torch.uint8)
        glob = (1.0 + 0.25 * torch.rand(S, H, generator=g)).to(torch.float16)
        c = torch.empty(T, K, H, dtype=torch.bfloat16)
        tw = torch.rand(T, K, generator=g)
        tid = torch.randint(0, S, (T, K), generator=g, dtype=torch.int32)
        pi = packed.view(torch.int32)
        ms._decode_nvfp4_marlin_swiglu_kernel[(routes, triton.cdiv(H, 16))](
            gate_up, pi, scale, glob, c, tw, tid, lut, tid, I, float(limit), routes, H, I,
            gate_up.stride(0), gate_up.stride(1), pi.stride(0), pi.stride(1), pi.stride(2),
            scale.stride(0), scale.stride(1), scale.stride(2), glob.stride(0), glob.stride(1),
            c.stride(0), c.stride(1), c.stride(2), tw.stride(0), tw.stride(1),
            tid.stride(0), tid.stride(1),
            BLOCK_SIZE_N=16, BLOCK_SIZE_KW=32, TOP_K=K, MUL_ROUTED_WEIGHT=True,
            compute_type=tl.bfloat16, act_type=tl.bfloat16, HAS_MASK=False,
            HAS_LIMIT=limit > 0)
        out[name] = dict(gate_up_bits=_bits16(gate_up), down_packed=packed.numpy(),
                         down_scale=scale.numpy(), down_global_bits=_bits16(glob),
                         topk_w=tw.numpy(), topk_ids=tid.numpy(), limit=np.float32(limit),
                         ic3_bits=_bits16(c))
    return out


def main() -> None:
    _install_shim()
    check_shim()
    fr = _load("overlay/freetoken/kernel/triton/fused_route.py", "ref_fused_route")
    ms = _load("overlay/freetoken/kernel/triton/nvfp4_marlin_swiglu.py", "ref_marlin_swiglu")
    np.savez_compressed(os.path.join(HERE, "e2m1_table.npz"), **e2m1_table())
    for name, d in route_cases(fr).items():
        np.savez_compressed(os.path.join(HERE, f"route_sigmoid_{name}.npz"), **d)
    for name, d in route_variant_cases(fr).items():
        np.savez_compressed(os.path.join(HERE, f"route_{name}.npz"), **d)
    for name, d in down_swiglu_cases(ms).items():
        np.savez_compressed(os.path.join(HERE, f"down_swiglu_{name}.npz"), **d)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
