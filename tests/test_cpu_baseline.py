"""The C++ CPU restatement (timed CPU baseline) agrees with the numpy oracle."""
import numpy as np
import pytest

from oracle import cpu_moe
from oracle import moe_oracle as m
from tests.moe_cases import build_case


@pytest.mark.parametrize("T,shared,limit", [(1, True, float("inf")), (5, True, 7.0),
                                            (3, False, float("inf"))])
def test_cpu_baseline_matches_oracle(T, shared, limit):
    case = build_case(8, 256, 128, T, 2, seed=11 + T, shared=shared)
    ref = m.moe_layer(case["inp"].x.float().numpy(), case["bank"].numpy(), case["w"], case["ids"],
                      case["shared"].numpy() if shared else None, limit)["out"]
    x_bits = case["inp"].x.contiguous().view(__import__("torch").int16).numpy().view(np.uint16)
    got = cpu_moe.moe_layer(x_bits, case["bank"].numpy(), case["w"], case["ids"],
                            case["shared"].numpy() if shared else None, limit, nthreads=2)
    assert m.max_abs_rel(m.bf16_from_bits(got), ref) <= 1e-2
    assert np.mean(m.bf16_from_bits(got) != ref) < 0.05


def test_cpu_baseline_threads_deterministic():
    case = build_case(8, 256, 128, 4, 2, seed=2)
    import torch
    x_bits = case["inp"].x.contiguous().view(torch.int16).numpy().view(np.uint16)
    a = cpu_moe.moe_layer(x_bits, case["bank"].numpy(), case["w"], case["ids"], None, nthreads=1)
    b = cpu_moe.moe_layer(x_bits, case["bank"].numpy(), case["w"], case["ids"], None, nthreads=4)
    assert np.array_equal(a, b)
