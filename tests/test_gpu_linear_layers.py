"""The EXL3 linear at the model's layer shapes, against the CPU oracle under the reference's gates.

The shapes the bench times: q / o 5120 -> 5120, gate / up 5120 -> 17408, down
17408 -> 5120, at the prefill row counts M = 128 and 2048 (the M > 16 route) and, for the bit widths
the other tests cover only on small matrices, K = 2, 5, 6 and 8 on a layer shape at M = 1 and 16.
Gates: the reference's tests/test_gpu_parity.py:51-52, 65-70 (normalised max-abs 3e-3, RMS 2e-4,
cosine 0.999999, per-element 4e-3 * RMS + 2e-3 * |ref|).  Those analytic bounds assume exact fp32
accumulation; the reference's policy takes, per metric, max(analytic bound, 4 x the deviation of the
same-arithmetic baseline) (configs/acceptance_policy.example.json, "final_gate_rule").  For M > 16 the
baseline measured here is the reference's own route on this GPU: the bit-exact dense W (reconstruct)
times A_had in a library fp16 GEMM with fp32 accumulation; at k = 17408 the tensor cores' accumulation
alone moves both routes past the 2e-4 RMS bound, by the same amount.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import exl3_oracle as O
from tests.test_gpu_linear import GATES, assert_gates, fixtures, stats, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from exl3rocm import ops as _ops
    return _ops


def dense_baseline(ops, xd, td, sd, vd, K):
    """The reference's M > 16 arithmetic on this GPU: had_in, the bit-exact dense W, a library fp16 GEMM
    with fp32 accumulation (c_rot rounded to fp16), had_out.  Test infrastructure for the gate rule."""
    m, k = xd.shape
    n = vd.shape[0]
    w = torch.empty(k, n, dtype=torch.float16, device=xd.device)
    ops.reconstruct(w, td, K, False, True)
    xh = torch.empty_like(xd)
    ops.had_r_128(xd, xh, sd, None, 1.0)
    flag = torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    try:
        y = torch.mm(xh, w)
    finally:
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = flag
    ops.had_r_128(y, y, None, vd, 1.0)
    return y


def assert_policy_gates(st: dict, base: dict):
    """max(analytic bound, 4 x baseline deviation) per metric (cosine: 1 - 4 x (1 - baseline))."""
    assert st["normalized_max_abs_err"] <= max(GATES["normalized_max_abs_err"], 4 * base["normalized_max_abs_err"]), (st, base)
    assert st["normalized_rms_err"] <= max(GATES["normalized_rms_err"], 4 * base["normalized_rms_err"]), (st, base)
    assert st["cosine_similarity"] >= min(GATES["cosine_similarity_min"], 1 - 4 * (1 - base["cosine_similarity"])), (st, base)
    assert st["abs_rel_bound_ratio"] <= max(GATES["abs_rel_bound_ratio"], 4 * base["abs_rel_bound_ratio"]), (st, base)


@pytest.mark.parametrize("m,k,n,K", [(128, 5120, 17408, 4), (128, 17408, 5120, 4), (2048, 5120, 17408, 4),
                                     (2048, 5120, 5120, 3), (300, 5120, 1024, 4), (2048, 17408, 5120, 4)])
def test_prefill_rows_at_layer_shapes(ops, m, k, n, K):
    x, tr, suh, svh = fixtures(k, n, K, 9000 + m + K, m=m)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    y = torch.ops.exl3rocm.linear(xd, td, sd, vd, K, False, True)
    base = dense_baseline(ops, xd, td, sd, vd, K)
    torch.cuda.synchronize()
    ref = O.linear(x, tr, K, suh, svh, 2)
    assert_policy_gates(stats(y.cpu().numpy(), ref), stats(base.cpu().numpy(), ref))


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
    b0, b1 = dense_baseline(ops, xd, t0, s0, v0, K), dense_baseline(ops, xd, t1, s1, v1, K)
    torch.cuda.synchronize()
    yc = y.cpu().numpy()
    r0, r1 = O.linear(x, tr0, K, su0, sv0, 2), O.linear(x, tr1, K, su1, sv1, 2)
    assert_policy_gates(stats(yc[:, :n], r0), stats(b0.cpu().numpy(), r0))
    assert_policy_gates(stats(yc[:, n:], r1), stats(b1.cpu().numpy(), r1))
