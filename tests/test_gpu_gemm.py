"""The tcgen05 prefill GEMM (exl3b_gemm) against the CPU oracle, through the C ABI and the torch op.

The reference's M > 16 route (vllm_plugin/exl3rocm/ops.py:86-97) is checked by its own tests under the
same gates as the GEMV (tests/test_gpu_parity.py:51-52, 65-70).  Cases cover every bit width and
codebook, row counts that do not fill a 256-row tile (1, 17, 300), widths that do not fill a 256-column
tile (128, 384), repeatability, the decline of a bf16 flag without touching y, and graph replay.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import exl3_oracle as O
from tests.test_gpu_linear import assert_gates, fixtures, stats, to_dev

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    import exl3rocm.ops  # noqa: F401
    from exl3rocm import _lib
    return _lib


def gemm(lib, x, td, sd, vd, K, cb, n, y=None):
    m, k = x.shape
    ws = torch.zeros(int(lib.lib().exl3b_gemm_workspace_bytes(m, k)), dtype=torch.uint8, device=DEV)
    y = torch.full((m, n), float("nan"), dtype=torch.float16, device=DEV) if y is None else y
    st = lib.lib().exl3b_gemm(x.data_ptr(), m, k, td.data_ptr(), n, K, cb, sd.data_ptr(), vd.data_ptr(), y.data_ptr(),
                              y.stride(0), ws.data_ptr(), ws.numel(),
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return st, y, ws


@pytest.mark.parametrize("m,k,n,K,cb", [
    (256, 256, 256, 4, 2),     # one tile
    (17, 512, 384, 4, 2),      # partial rows and a partial column tile
    (300, 1024, 512, 3, 0),    # two row tiles, 3INST
    (1, 256, 128, 2, 1),       # a single row, MCG
    (513, 768, 768, 5, 2),
    (256, 384, 256, 6, 0),
    (128, 256, 640, 7, 1),
    (200, 512, 256, 8, 2),
    (64, 128, 256, 1, 2),
])
def test_gemm_matches_oracle(lib, m, k, n, K, cb):
    x, tr, suh, svh = fixtures(k, n, K, 7000 + m + K + cb, m=m)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    st, y, ws = gemm(lib, xd, td, sd, vd, K, cb, n)
    assert st == lib.EXL3B_OK, lib.lib().exl3b_status_string(st)
    assert int(ws[:4].view(torch.int32).item()) == 0  # no wait gave up
    assert_gates(stats(y.cpu().numpy(), O.linear(x, tr, K, suh, svh, cb)))


def test_gemm_repeatable_and_row_stride(lib):
    m, k, n, K = 300, 512, 512, 4
    x, tr, suh, svh = fixtures(k, n, K, 7100, m=m)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    _, y1, _ = gemm(lib, xd, td, sd, vd, K, 2, n)
    _, y2, _ = gemm(lib, xd, td, sd, vd, K, 2, n)
    assert torch.equal(y1, y2)
    big = torch.full((m, n + 256), float("nan"), dtype=torch.float16, device=DEV)
    st, _, _ = gemm(lib, xd, td, sd, vd, K, 2, n, y=big[:, 128:128 + n])
    assert st == lib.EXL3B_OK
    assert torch.equal(big[:, 128:128 + n], y1)
    assert torch.isnan(big[:, :128]).all() and torch.isnan(big[:, 128 + n:]).all()


def test_gemm_declines_without_touching_y(lib):
    m, k, n, K = 64, 256, 256, 4
    x, tr, suh, svh = fixtures(k, n, K, 7200, m=m)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    for bad_cb, bad_k in ((2 | 0x100, k), (2, k)):
        st, y, _ = gemm(lib, xd, td, sd, vd, K if bad_cb != 2 else 9, bad_cb, n)
        assert st == lib.EXL3B_DECLINED
        assert torch.isnan(y).all()


def test_op_routes_large_m_to_the_gemm_and_replays_in_a_graph(lib):
    m, k, n, K = 96, 512, 256, 4
    x, tr, suh, svh = fixtures(k, n, K, 7300, m=m)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    eager = torch.ops.exl3rocm.linear(xd, td, sd, vd, K, False, True)
    st, y, _ = gemm(lib, xd, td, sd, vd, K, 2, n)
    assert torch.equal(eager, y)
    from exl3rocm import ops
    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.reserve_gemm_workspace(DEV, m, k)
        torch.ops.exl3rocm.linear(xd, td, sd, vd, K, False, True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = torch.ops.exl3rocm.linear(xd, td, sd, vd, K, False, True)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    del g
