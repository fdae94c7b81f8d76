"""The EXL3 linear at the model's layer shapes, against the CPU oracle under the reference's gates.

The shapes the bench times: q / o 5120 -> 5120, gate / up 5120 -> 17408, down
17408 -> 5120, at the prefill row counts M = 128 and 2048 (the M > 16 route) and, for the bit widths
the other tests cover only on small matrices, K = 2, 5, 6 and 8 on a layer shape at M = 1 and 16.
Gates: the reference's tests/test_gpu_parity.py:51-52, 65-70 (normalised max-abs 3e-3, RMS 2e-4,
cosine 0.999999, per-element 4e-3 * RMS + 2e-3 * |ref|).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import exl3_oracle as O
from tests.test_gpu_linear import assert_gates, fixtures, stats, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from exl3rocm import ops as _ops
    return _ops


@pytest.mark.parametrize("m,k,n,K", [(128, 5120, 17408, 4), (128, 17408, 5120, 4), (2048, 5120, 17408, 4),
                                     (2048, 5120, 5120, 3), (300, 5120, 1024, 4)])
def test_prefill_rows_at_layer_shapes(ops, m, k, n, K):
    x, tr, suh, svh = fixtures(k, n, K, 9000 + m + K, m=m)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    y = torch.ops.exl3rocm.linear(xd, td, sd, vd, K, False, True)
    torch.cuda.synchronize()
    assert_gates(stats(y.cpu().numpy(), O.linear(x, tr, K, suh, svh, 2)))


@pytest.mark.parametrize("K", [2, 5, 6, 8])
@pytest.mark.parametrize("m", [1, 16])
def test_bit_widths_at_a_layer_shape(ops, K, m):
    k, n = 5120, 5120
    x, tr, suh, svh = fixtures(k, n, K, 9100 + K + m, m=m)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    y = torch.ops.exl3rocm.linear(xd, td, sd, vd, K, False, True)
    torch.cuda.synchronize()
    assert_gates(stats(y.cpu().numpy(), O.linear(x, tr, K, suh, svh, 2)))


def test_grouped_gate_up_at_layer_shape_m2048(ops):
    """The prefill gate/up module: two 5120 -> 17408 groups through linear_groups at M = 2048."""
    k, n, K, m = 5120, 17408, 3, 2048
    x, tr0, su0, sv0 = fixtures(k, n, K, 9200, m=m)
    _, tr1, su1, sv1 = fixtures(k, n, K, 9201, m=m)
    xd, t0, s0, v0 = to_dev(x, tr0, su0, sv0)
    _, t1, s1, v1 = to_dev(x, tr1, su1, sv1)
    y = torch.ops.exl3rocm.linear_groups(xd, [t0, t1], [s0, s1], [v0, v1], [K, K], False, True)
    torch.cuda.synchronize()
    yc = y.cpu().numpy()
    assert_gates(stats(yc[:, :n], O.linear(x, tr0, K, su0, sv0, 2)))
    assert_gates(stats(yc[:, n:], O.linear(x, tr1, K, su1, sv1, 2)))
