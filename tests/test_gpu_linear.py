"""GPU parity of the EXL3 linear path against the CPU oracle (pinned to the reference's goldens).

Mirrors the reference's tests/test_gpu_parity.py: bit-exact decode and reconstruct, the float
pipeline under the reference's normalised gates (:51-52, 65-70), determinism, stream
independence, zero input and decline-without-modifying-outputs; plus the multi-row bitwise
contract (reference vllm_plugin/tests/mr_check.py) and the grouped path (mrg_check.py).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import exl3_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"

# reference tests/test_gpu_parity.py:51-52, 65-70 (same-arithmetic gates)
GATES = {"normalized_max_abs_err": 3e-3, "normalized_rms_err": 2e-4, "cosine_similarity_min": 0.999999,
         "abs_rel_bound_ratio": 1.0}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from exl3rocm import ops as _ops
    return _ops


def stats(got: np.ndarray, ref: np.ndarray) -> dict:
    got = got.astype(np.float64).ravel()
    ref = ref.astype(np.float64).ravel()
    d = got - ref
    scale = np.sqrt(np.mean(ref ** 2)) or 1.0
    bound = 4e-3 * scale + 2e-3 * np.abs(ref)
    return {"normalized_max_abs_err": float(np.abs(d).max() / scale),
            "normalized_rms_err": float(np.sqrt(np.mean(d ** 2)) / scale),
            "cosine_similarity": float(got @ ref / ((np.linalg.norm(got) * np.linalg.norm(ref)) or 1.0)),
            "abs_rel_bound_ratio": float((np.abs(d) / bound).max())}


def assert_gates(st: dict):
    assert st["normalized_max_abs_err"] <= GATES["normalized_max_abs_err"], st
    assert st["normalized_rms_err"] <= GATES["normalized_rms_err"], st
    assert st["cosine_similarity"] >= GATES["cosine_similarity_min"], st
    assert st["abs_rel_bound_ratio"] <= GATES["abs_rel_bound_ratio"], st


def fixtures(k, n, K, seed, signs=True, m=1):
    rng = np.random.default_rng(seed)
    tr = O.random_trellis(rng, k // 16, n // 16, K)
    if signs:
        suh = np.sign(rng.standard_normal(k)).astype(np.float16)
        svh = np.sign(rng.standard_normal(n)).astype(np.float16)
    else:
        suh = (np.abs(rng.standard_normal(k)) * 0.5 + 0.5).astype(np.float16)
        svh = (np.abs(rng.standard_normal(n)) * 0.5 + 0.5).astype(np.float16)
    x = (rng.standard_normal((m, k)) * 0.3).astype(np.float16)
    return x, tr, suh, svh


def to_dev(x, tr, suh, svh):
    return (torch.from_numpy(x).to(DEV), torch.from_numpy(tr.view(np.int16)).to(DEV),
            torch.from_numpy(suh).to(DEV), torch.from_numpy(svh).to(DEV))


# ---- exactness ----------------------------------------------------------------------------
@pytest.mark.parametrize("cb,mcg,mul1", [(2, False, True), (1, True, False), (0, False, False)])
def test_decode_exhaustive_bitexact(ops, cb, mcg, mul1):
    codes = torch.arange(65536, dtype=torch.int32).to(torch.int16).to(DEV)
    out = torch.empty(65536, dtype=torch.float32, device=DEV)
    ops.decode(codes, out, mcg, mul1)
    got = out.cpu().numpy().astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(got, O.codebook_table(cb))


@pytest.mark.parametrize("K", range(1, 9))
@pytest.mark.parametrize("cb", [0, 1, 2])
def test_reconstruct_bitexact(ops, K, cb):
    rng = np.random.default_rng(100 + K)
    tr = O.random_trellis(rng, 16, 24, K)
    W = torch.empty(256, 384, dtype=torch.float16, device=DEV)
    ops.reconstruct(W, torch.from_numpy(tr.view(np.int16)).to(DEV), K, cb == 1, cb == 2)
    np.testing.assert_array_equal(W.cpu().numpy().view(np.uint16), O.dequant(tr, K, cb).view(np.uint16))


def test_reconstruct_goldens(ops, golden):
    for K in range(1, 9):
        tr = golden[f"dq_trellis_K{K}"]
        for cb in (0, 1, 2):
            W = torch.empty(tr.shape[0] * 16, tr.shape[1] * 16, dtype=torch.float16, device=DEV)
            ops.reconstruct(W, torch.from_numpy(tr.view(np.int16)).to(DEV), K, cb == 1, cb == 2)
            np.testing.assert_array_equal(W.cpu().numpy().view(np.uint16), golden[f"dq_W_K{K}_cb{cb}"])


def test_reconstruct_slice(ops):
    rng = np.random.default_rng(7)
    tr = O.random_trellis(rng, 8, 32, 3)
    t = torch.from_numpy(tr.view(np.int16)).to(DEV)
    W = torch.empty(128, 160, dtype=torch.float16, device=DEV)
    ops.reconstruct_slice(W, t, 3, False, True, 96)
    np.testing.assert_array_equal(W.cpu().numpy(), O.dequant(tr, 3, 2, n0=96, n1=256))


def test_reconstruct_config1_full_size(ops):
    """5120 -> 17408, 4 bits, 3INST codebook, every weight bit-exact."""
    rng = np.random.default_rng(0)
    tr = O.random_trellis(rng, 320, 1088, 4)
    W = torch.empty(5120, 17408, dtype=torch.float16, device=DEV)
    ops.reconstruct(W, torch.from_numpy(tr.view(np.int16)).to(DEV), 4, False, False)
    np.testing.assert_array_equal(W.cpu().numpy().view(np.uint16), O.dequant(tr, 4, 0).view(np.uint16))


def test_had_r_128_matches_oracle(ops, golden):
    x = golden["had_x"].view(np.float16)
    s = golden["had_s"].view(np.float16)
    xt, st = torch.from_numpy(x.copy()).to(DEV), torch.from_numpy(s.copy()).to(DEV)
    y_in = torch.empty_like(xt)
    ops.had_r_128(xt, y_in, st, None, 1.0)
    y_out = xt.clone()
    ops.had_r_128(y_out, y_out, None, st, 1.0)  # in place, as the reference's output stage
    for got, key in ((y_in, "had_in_y"), (y_out, "had_out_y")):
        g = got.cpu().numpy().astype(np.float64)
        r = golden[key].view(np.float16).astype(np.float64)
        ulp = np.maximum(np.abs(r) * 2.0 ** -10, 2.0 ** -24)
        assert (np.abs(g - r) <= ulp).all()
        assert (g == r).mean() > 0.99


# ---- float pipeline ------------------------------------------------------------------------
@pytest.mark.parametrize("shape", [
    (256, 128, 3), (512, 256, 3), (1024, 512, 3),
    (5120, 5120, 3), (17408, 5120, 3), (5120, 17408, 3),
    (5120, 5120, 2), (5120, 5120, 4),
])
def test_linear_m1_parity_reference_shapes(ops, shape):
    """The reference's parity shapes (tests/test_gpu_parity.py:145-149), mul1."""
    k, n, K = shape
    x, tr, suh, svh = fixtures(k, n, K, 7 + k + n, signs=(k % 2 == 0))
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    y = torch.ops.exl3rocm.linear(xd, td, sd, vd, K, False, True)
    torch.cuda.synchronize()
    assert_gates(stats(y.cpu().numpy(), O.linear(x, tr, K, suh, svh, 2)))
    assert ops.workspace_error() == 0


@pytest.mark.parametrize("K", range(1, 9))
@pytest.mark.parametrize("cb", [0, 1, 2])
def test_linear_all_bits_codebooks(ops, K, cb):
    x, tr, suh, svh = fixtures(1024, 768, K, 31 * K + cb, signs=bool(K % 2))
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    y = torch.ops.exl3rocm.linear(xd, td, sd, vd, K, cb == 1, cb == 2)
    assert_gates(stats(y.cpu().numpy(), O.linear(x, tr, K, suh, svh, cb)))


def test_linear_config1_cb0(ops):
    """BASELINE config 1 end to end: 5120 -> 17408, 4 bits, 3INST, x ~ N(0,1)."""
    rng = np.random.default_rng(0)
    tr = O.random_trellis(rng, 320, 1088, 4)
    suh = np.sign(rng.standard_normal(5120)).astype(np.float16)
    svh = np.sign(rng.standard_normal(17408)).astype(np.float16)
    x = rng.standard_normal((1, 5120)).astype(np.float16)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    y = torch.ops.exl3rocm.linear(xd, td, sd, vd, 4, False, False)
    assert_gates(stats(y.cpu().numpy(), O.linear(x, tr, 4, suh, svh, 0)))


def test_linear_goldens(ops, golden):
    for ci, (k, n, K, cb, _s) in enumerate(golden["gemv_cases"]):
        x = golden[f"gemv{ci}_x"].view(np.float16)[None]
        tr = golden[f"gemv{ci}_trellis"]
        suh = golden[f"gemv{ci}_suh"].view(np.float16)
        svh = golden[f"gemv{ci}_svh"].view(np.float16)
        xd, td, sd, vd = to_dev(x.copy(), tr, suh.copy(), svh.copy())
        y = torch.ops.exl3rocm.linear(xd, td, sd, vd, int(K), int(cb) == 1, int(cb) == 2)
        assert_gates(stats(y.cpu().numpy()[0], golden[f"gemv{ci}_y"].view(np.float16)))


# ---- contracts -----------------------------------------------------------------------------
@pytest.mark.parametrize("m", [2, 3, 4, 8, 9, 12, 16])
def test_multirow_rows_bitwise_equal_m1(ops, m):
    x, tr, suh, svh = fixtures(2048, 1024, 4, 1000 + m, m=m)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    y = torch.ops.exl3rocm.linear(xd, td, sd, vd, 4, False, True)
    for r in range(m):
        y1 = torch.ops.exl3rocm.linear(xd[r:r + 1].clone(), td, sd, vd, 4, False, True)
        assert torch.equal(y[r:r + 1], y1), f"row {r} of m={m} differs from its m=1 result"
    assert_gates(stats(y.cpu().numpy(), O.linear(x, tr, 4, suh, svh, 2)))


@pytest.mark.parametrize("m", [1, 4])
def test_grouped_gate_up(ops, m):
    k, n, K = 1024, 1536, 3
    rng = np.random.default_rng(77)
    trs = [O.random_trellis(rng, k // 16, n // 16, K) for _ in range(2)]
    suhs = [np.sign(rng.standard_normal(k)).astype(np.float16) for _ in range(2)]
    svhs = [np.sign(rng.standard_normal(n)).astype(np.float16) for _ in range(2)]
    x = rng.standard_normal((m, k)).astype(np.float16)
    xd = torch.from_numpy(x).to(DEV)
    td = [torch.from_numpy(t.view(np.int16)).to(DEV) for t in trs]
    sd = [torch.from_numpy(s).to(DEV) for s in suhs]
    vd = [torch.from_numpy(s).to(DEV) for s in svhs]
    y = torch.ops.exl3rocm.linear_groups(xd, td, sd, vd, [K, K], False, True)
    ref = np.concatenate([O.linear(x, t, K, s, v, 2) for t, s, v in zip(trs, suhs, svhs)], axis=1)
    assert y.shape == (m, 2 * n)
    assert_gates(stats(y.cpu().numpy(), ref))
    if m > 1:  # rows equal the grouped m = 1 path bit for bit
        for r in range(m):
            y1 = torch.ops.exl3rocm.linear_groups(xd[r:r + 1].clone(), td, sd, vd, [K, K], False, True)
            assert torch.equal(y[r:r + 1], y1)


def test_grouped_mixed_bits_qkv(ops):
    """q/k/v with different widths and bit widths (mixed-bit fused module, reference plugin.py:8-14)."""
    k = 1024
    rng = np.random.default_rng(5)
    spec = [(1024, 2), (256, 5), (256, 5)]
    trs = [O.random_trellis(rng, k // 16, n // 16, K) for n, K in spec]
    suhs = [np.sign(rng.standard_normal(k)).astype(np.float16) for _ in spec]
    svhs = [np.sign(rng.standard_normal(n)).astype(np.float16) for n, _ in spec]
    x = rng.standard_normal((4, k)).astype(np.float16)
    y = torch.ops.exl3rocm.linear_groups(
        torch.from_numpy(x).to(DEV), [torch.from_numpy(t.view(np.int16)).to(DEV) for t in trs],
        [torch.from_numpy(s).to(DEV) for s in suhs], [torch.from_numpy(s).to(DEV) for s in svhs],
        [K for _, K in spec], False, True)
    ref = np.concatenate([O.linear(x, t, K, s, v, 2) for t, s, v, (_, K) in zip(trs, suhs, svhs, spec)], axis=1)
    assert_gates(stats(y.cpu().numpy(), ref))


def test_determinism_and_streams(ops):
    x, tr, suh, svh = fixtures(5120, 2048, 4, 55)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    outs = [torch.ops.exl3rocm.linear(xd, td, sd, vd, 4, False, True).clone() for _ in range(3)]
    for _ in range(2):
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            outs.append(torch.ops.exl3rocm.linear(xd, td, sd, vd, 4, False, True).clone())
        s.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def test_zero_input(ops):
    _, tr, suh, svh = fixtures(256, 128, 3, 3)
    y = torch.ops.exl3rocm.linear(torch.zeros(1, 256, dtype=torch.float16, device=DEV),
                                  torch.from_numpy(tr.view(np.int16)).to(DEV), torch.from_numpy(suh).to(DEV),
                                  torch.from_numpy(svh).to(DEV), 3, False, True)
    assert torch.isfinite(y).all() and y.abs().max().item() <= 1e-3


def test_declined_call_leaves_output_untouched(ops):
    """reference tests/test_gpu_parity.py:236-258: a declined call must not modify outputs."""
    from exl3rocm import _lib
    x, tr, suh, svh = fixtures(256, 128, 3, 9, m=17)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    y = torch.full((17, 128), float("nan"), dtype=torch.float16, device=DEV)
    ws = ops.reserve_workspace(DEV, 256, 128, 1, 16)
    st = _lib.lib().exl3b_linear(xd.data_ptr(), 17, 256, td.data_ptr(), 128, 3, 2, sd.data_ptr(), vd.data_ptr(),
                                 y.data_ptr(), 128, ws.data_ptr(), ws.numel(),
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert st == _lib.EXL3B_DECLINED
    assert torch.isnan(y).all()


def test_graph_capture_replay(ops):
    x, tr, suh, svh = fixtures(2048, 1024, 4, 88, m=4)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    eager = torch.ops.exl3rocm.linear(xd, td, sd, vd, 4, False, True).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.reserve_workspace(DEV, 2048, 1024, 1, 16)
        torch.ops.exl3rocm.linear(xd, td, sd, vd, 4, False, True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = torch.ops.exl3rocm.linear(xd, td, sd, vd, 4, False, True)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


@pytest.mark.parametrize("m", [17, 64, 300])
def test_linear_large_m_route(ops, m):
    x, tr, suh, svh = fixtures(1024, 512, 4, 500 + m, m=m)
    xd, td, sd, vd = to_dev(x, tr, suh, svh)
    y = torch.ops.exl3rocm.linear(xd, td, sd, vd, 4, False, True)
    st = stats(y.cpu().numpy(), O.linear(x, tr, 4, suh, svh, 2))
    assert st["normalized_rms_err"] < 2e-3 and st["cosine_similarity"] > 0.99999, st


@pytest.mark.parametrize("m", [1, 5, 16])
def test_bf16_input_rounded_in_kernel_matches_cast(ops, m):
    """bf16 x is rounded to fp16 inside the kernel: bitwise the same as the reference's cast at the op
    boundary (vllm_plugin/exl3rocm/ops.py:72-73), for one group and for a grouped call."""
    x, tr, suh, svh = fixtures(1024, 512, 4, 31 + m, m=m)
    xb = torch.randn(m, 1024, device=DEV, dtype=torch.float32).to(torch.bfloat16)
    _, td, sd, vd = to_dev(x, tr, suh, svh)
    y_bf = torch.ops.exl3rocm.linear(xb, td, sd, vd, 4, False, True)
    y_fp = torch.ops.exl3rocm.linear(xb.to(torch.float16), td, sd, vd, 4, False, True)
    assert torch.equal(y_bf, y_fp)
    g_bf = torch.ops.exl3rocm.linear_groups(xb, [td, td], [sd, sd], [vd, vd], [4, 4], False, True)
    g_fp = torch.ops.exl3rocm.linear_groups(xb.to(torch.float16), [td, td], [sd, sd], [vd, vd], [4, 4], False, True)
    assert torch.equal(g_bf, g_fp)
