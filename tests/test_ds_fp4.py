"""ds_fp4 (e8m0 per-32 scale) banks on CPU: the conversion to the native NVFP4 bank is exact,
its range rules hold, and the oracle's FP8 round trip of h follows its definition.

The reference's ds_fp4 layer (patches/moe_fused_ds_fp4.patch) keeps code * 2^(s-127) weights;
the conversion must give the same real numbers as code * e4m3_scale * fp16_global.
"""
import numpy as np
import pytest
import torch

from ftb import synth
from ftb.ds_fp4 import DsFp4Bank, ds_fp4_dequant, nvfp4_from_ds_fp4
from oracle import moe_oracle as m


def _nvfp4_dequant(packed, scale, glob):
    v = m.dequant_rows(packed.numpy(), scale.view(torch.uint8).numpy()).astype(np.float64)
    return v * glob.float().numpy().astype(np.float64)[:, None]


def test_conversion_is_exact():
    ds = synth.make_ds_fp4_bank(3, 256, 256, seed=4)
    nv, rep = nvfp4_from_ds_fp4(ds)
    assert rep.flushed_blocks == 0
    for e in range(3):
        for (p, s), (q, t, g) in (((ds.gate_up_packed[e], ds.gate_up_scale[e]),
                                   (nv.gate_up_packed[e], nv.gate_up_scale[e],
                                    nv.gate_up_global[e])),
                                  ((ds.down_packed[e], ds.down_scale[e]),
                                   (nv.down_packed[e], nv.down_scale[e], nv.down_global[e]))):
            want = ds_fp4_dequant(p, s).double().numpy()
            got = _nvfp4_dequant(q, t, g)
            assert np.array_equal(want, got)


def test_conversion_range_edges():
    """Every block exponent 0..17 binades below its row's largest is exact (E4M3 normals and
    subnormals); further below is refused (strict) or flushed and counted."""
    H, I = 1024, 256
    ds = synth.make_ds_fp4_bank(1, H, I, seed=5)
    s = ds.gate_up_scale[0]
    s[:, :] = 120
    s[0, :18] = torch.arange(120, 102, -1, dtype=torch.uint8)  # 0..17 binades below
    s[1, 0] = 137  # a row with a larger scale: global 2^(137-127-8), the rest 17 below
    s[2, 1] = 120 - 18  # one block 18 binades below: not exact
    with pytest.raises(ValueError):
        nvfp4_from_ds_fp4(ds)
    nv, rep = nvfp4_from_ds_fp4(ds, strict=False)
    assert rep.flushed_blocks == 1
    want = ds_fp4_dequant(ds.gate_up_packed[0], s).double().numpy()
    got = _nvfp4_dequant(nv.gate_up_packed[0], nv.gate_up_scale[0], nv.gate_up_global[0])
    bad = want != got
    assert bad[:2].sum() == 0 and bad[3:].sum() == 0
    assert np.all(got[2, 32:64] == 0)  # the flushed block
    s[2, 1] = 255
    with pytest.raises(ValueError):
        nvfp4_from_ds_fp4(ds, strict=False)  # e8m0 NaN
    s[2, 1] = 120
    s[3, :] = 160  # global 2^25: beyond fp16
    with pytest.raises(ValueError):
        nvfp4_from_ds_fp4(ds)


def test_bank_validation():
    ds = synth.make_ds_fp4_bank(2, 256, 256, seed=6)
    bad = DsFp4Bank(ds.gate_up_packed, ds.gate_up_scale[:, :, :4], ds.down_packed, ds.down_scale)
    with pytest.raises(ValueError):
        bad.validate()


def test_fp8_round_trip_definition():
    """fp8_block128_roundtrip: per 128-block, sc = 2^ceil(log2(max(amax, 1e-4) / 448)); the
    result is q * sc with q an E4M3 value, |q| <= 448, nearest to a / sc (ties to even)."""
    rng = np.random.default_rng(3)
    a = (rng.standard_normal((6, 512)) * np.exp(rng.uniform(-6, 6, (6, 1)))).astype(np.float32)
    a[1, 128:256] = 0.0       # an all-zero block: amax floor 1e-4
    a[2, 5] = 2.0 ** 20       # a large element dominates its block
    r = m.fp8_block128_roundtrip(a)
    table = np.unique(np.abs(m.e4m3_decode(np.arange(256, dtype=np.uint8))))
    table = table[np.isfinite(table)]
    for row in range(6):
        for b in range(4):
            blk = a[row, 128 * b:128 * (b + 1)]
            amax = max(np.float32(np.abs(blk).max()), np.float32(1e-4))
            e = int(np.ceil(np.log2(np.float64(np.float32(amax * np.float32(1 / 448))))))
            q = r[row, 128 * b:128 * (b + 1)] / 2.0 ** e
            assert np.all(np.isin(np.abs(q), table))
            # nearest representable
            x = np.clip(blk / 2.0 ** e, -448, 448)
            d = np.abs(np.abs(x)[:, None] - table[None, :]).min(1)
            assert np.all(np.abs(np.abs(q) - np.abs(x)) <= d + 1e-12)
    assert np.all(r[1, 128:256] == 0)
    # bf16-exact
    assert np.array_equal(m.bf16_round(r), r)
