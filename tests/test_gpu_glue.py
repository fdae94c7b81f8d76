"""The decode-step glue and the fused linear epilogues on the GPU.

* EXL3B_ACT_SILU_MUL (gate/up with SiLU * up in the GEMV epilogue) must equal, bit for bit, the
  unfused route: the grouped linear's [gate | up] output through exl3b_silu_mul (both use the same
  device arithmetic), for every row count, with rows independent of m and calls repeatable (the
  pair counters reset).  exl3b_silu_mul itself is checked against torch's fp16 F.silu(g) * u.
* EXL3B_Y_ADD must equal fp16(residual + linear(x)) bit for bit (one fp16 add, as torch's).
* RMSNorm and the neox rotary embedding against fp32 torch formulas of the same rounding points.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import exl3_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from exl3rocm import glue, ops
    return ops, glue


def _weights(k, n, K, seed):
    rng = np.random.default_rng(seed)
    tr = torch.from_numpy(O.random_trellis(rng, k // 16, n // 16, K).view(np.int16)).to(DEV)
    suh = torch.from_numpy(np.sign(rng.standard_normal(k)).astype(np.float16)).to(DEV)
    svh = torch.from_numpy((np.sign(rng.standard_normal(n)) / np.sqrt(k)).astype(np.float16)).to(DEV)
    return tr, suh, svh


def _ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in units of fp16 spacing at b (finite values)."""
    a32, b32 = a.float(), b.float()
    spacing = torch.where(b32.abs() < 6.1e-5, torch.full_like(b32, 2.0 ** -24),
                          2.0 ** (torch.floor(torch.log2(b32.abs().clamp_min(6.1e-5))) - 10))
    return (a32 - b32).abs() / spacing


@pytest.mark.parametrize("m", [1, 3, 8, 16])
@pytest.mark.parametrize("K", [3, 4])
def test_gate_up_silu_fused_equals_unfused(mods, m, K):
    ops, _ = mods
    k, n = 1024, 2816  # 22 column blocks per group: super-blocks shared by several CTAs
    g, u = _weights(k, n, K, 11 + K), _weights(k, n, K, 23 + K)
    x = torch.randn(m, k, device=DEV).to(torch.float16)
    tr, su, sv = [g[0], u[0]], [g[1], u[1]], [g[2], u[2]]
    fused = torch.ops.exl3rocm.gate_up_silu(x, tr, su, sv, K, False, True)
    gu = torch.ops.exl3rocm.linear_groups(x, tr, su, sv, [K, K], False, True)
    unfused = ops.silu_mul(gu)
    torch.cuda.synchronize()
    assert torch.equal(fused, unfused)
    again = torch.ops.exl3rocm.gate_up_silu(x, tr, su, sv, K, False, True)
    assert torch.equal(again, fused)  # pair counters were left at zero
    if m > 1:  # every row equals the m = 1 call on that row
        row = torch.ops.exl3rocm.gate_up_silu(x[m - 1:], tr, su, sv, K, False, True)
        assert torch.equal(row[0], fused[m - 1])
    assert ops.workspace_error(DEV) == 0


def test_gate_up_silu_large_m_route(mods):
    ops, _ = mods
    k, n, K = 512, 1024, 4
    g, u = _weights(k, n, K, 5), _weights(k, n, K, 6)
    x = torch.randn(40, k, device=DEV).to(torch.float16)
    tr, su, sv = [g[0], u[0]], [g[1], u[1]], [g[2], u[2]]
    y = torch.ops.exl3rocm.gate_up_silu(x, tr, su, sv, K, False, True)
    gu = torch.ops.exl3rocm.linear_groups(x, tr, su, sv, [K, K], False, True)
    assert torch.equal(y, ops.silu_mul(gu))


def test_silu_mul_against_torch(mods):
    ops, _ = mods
    torch.manual_seed(0)
    x = (torch.randn(37, 2 * 1024, device=DEV) * 4).to(torch.float16)
    x[0, :8] = torch.tensor([0.0, -0.0, 65504.0, -65504.0, 11.0, -11.0, 1e-4, -20.0], dtype=torch.float16)
    got = ops.silu_mul(x)
    g, u = x[:, :1024], x[:, 1024:]
    ref = torch.nn.functional.silu(g) * u  # fp16: silu rounded to fp16, then one fp16 multiply
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(got), fin)
    # exp and the division may round the fp32 silu differently from torch's: at most one fp16 step
    # of silu, which the multiply can carry to at most 2 ulps of the product
    assert float(_ulps(got[fin], ref[fin]).max()) <= 2.0
    assert float((got[fin] != ref[fin]).float().mean()) < 0.01


@pytest.mark.parametrize("m", [1, 4, 16])
def test_linear_residual_add(mods, m):
    ops, _ = mods
    k, n, K = 2048, 1536, 4
    tr, suh, svh = _weights(k, n, K, 31)
    x = torch.randn(m, k, device=DEV).to(torch.float16)
    res = torch.randn(m, n, device=DEV).to(torch.float16)
    y = torch.ops.exl3rocm.linear(x, tr, suh, svh, K, False, True)
    ref = res + y  # fp16 add on the GPU: exact sum, one rounding
    torch.ops.exl3rocm.linear_add_(x, tr, suh, svh, K, False, True, res)
    torch.cuda.synchronize()
    assert torch.equal(res, ref)


@pytest.mark.parametrize("with_residual", [False, True])
def test_rmsnorm(mods, with_residual):
    _, glue = mods
    torch.manual_seed(1)
    rows, cols, eps = 5, 5120, 1e-6
    x = (torch.randn(rows, cols, device=DEV) * 3).to(torch.float16)
    w = (1 + 0.1 * torch.randn(cols, device=DEV)).to(torch.float16)
    res = torch.randn(rows, cols, device=DEV).to(torch.float16) if with_residual else None
    v = (x + res) if with_residual else x
    out = glue.rmsnorm(x, w, eps, residual=res)
    if with_residual:
        assert torch.equal(res, v)
    vf = v.float()
    s = torch.rsqrt(vf.pow(2).mean(-1, keepdim=True) + eps)
    ref = (vf * s).to(torch.float16) * w
    # rsqrt and the fp32 summation order may move fp16(v * s) by one step, and the weight multiply
    # can carry that to 2 ulps of the output
    assert float(_ulps(out, ref).max()) <= 2.0
    assert float((out != ref).float().mean()) < 0.01


def test_rope_neox(mods):
    _, glue = mods
    torch.manual_seed(2)
    T, nq, nk, ctx = 6, 40, 8, 4096
    qkv = torch.randn(T, (nq + 2 * nk) * 128, device=DEV).to(torch.float16)
    before = qkv.clone()
    pos = torch.tensor([0, 1, 17, 1000, 4095, 2048], dtype=torch.int64, device=DEV)
    cs = glue.rope_cos_sin(ctx, 1e6, DEV)
    q = torch.empty(T, nq * 128, dtype=torch.float16, device=DEV)
    glue.rope_neox(qkv, q, nq, nk, pos, cs)

    def ref_rot(x):  # x [T, heads, 128] fp16 -> fp16
        c, s = cs[pos, :64][:, None, :], cs[pos, 64:][:, None, :]
        a, b = x[..., :64].float(), x[..., 64:].float()
        return torch.cat([a * c - b * s, b * c + a * s], -1).to(torch.float16)

    q_ref = ref_rot(before[:, :nq * 128].view(T, nq, 128)).view(T, -1)
    k_ref = ref_rot(before[:, nq * 128:(nq + nk) * 128].view(T, nk, 128)).view(T, -1)
    # fma contraction of a*c - b*s may round once less than the separate products
    assert float(_ulps(q, q_ref).max()) <= 1.0
    assert float(_ulps(qkv[:, nq * 128:(nq + nk) * 128], k_ref).max()) <= 1.0
    assert torch.equal(qkv[:, (nq + nk) * 128:], before[:, (nq + nk) * 128:])  # v untouched
    # the table: position 0 is the identity
    assert torch.equal(q[0], before[0, :nq * 128])


# reference tests/test_gpu_parity.py:51-52, 65-70 (the linear's gates)
def _gates(got, ref):
    g, r = got.double().flatten(), ref.double().flatten()
    d = g - r
    scale = float(r.pow(2).mean().sqrt()) or 1.0
    return (float(d.abs().max()) / scale <= 3e-3 and float(d.pow(2).mean().sqrt()) / scale <= 2e-4
            and float(torch.nn.functional.cosine_similarity(g, r, dim=0)) >= 0.999999)


@pytest.mark.parametrize("groups", [1, 3])
def test_linear_with_fused_rmsnorm(mods, groups):
    """The RMSNorm inside the GEMV against exl3b_rmsnorm then the linear: the per-row scale may round
    differently (another fp32 summation order), so the outputs meet the linear's gates rather than
    matching bitwise; rows stay bitwise independent of m."""
    ops, glue = mods
    k, K, eps = 5120, 4, 1e-6
    ns = [1024, 256, 256][:groups]
    ws = [_weights(k, n, K, 40 + i) for i, n in enumerate(ns)]
    tr, su, sv = [w[0] for w in ws], [w[1] for w in ws], [w[2] for w in ws]
    nw = (1 + 0.1 * torch.randn(k, device=DEV)).to(torch.float16)
    x = (torch.randn(5, k, device=DEV) * 2).to(torch.float16)
    fused = torch.empty(5, sum(ns), dtype=torch.float16, device=DEV)
    ops.linear_into(x, tr, su, sv, K, False, True, fused, norm=(nw, eps))
    h = glue.rmsnorm(x, nw, eps)
    ref = torch.empty_like(fused)
    ops.linear_into(h, tr, su, sv, K, False, True, ref)
    torch.cuda.synchronize()
    assert _gates(fused, ref)
    one = torch.empty(1, sum(ns), dtype=torch.float16, device=DEV)
    ops.linear_into(x[3:4], tr, su, sv, K, False, True, one, norm=(nw, eps))
    assert torch.equal(one[0], fused[3])


def test_rope_and_cache_int8_equals_two_kernels(mods):
    ops, glue = mods
    from exl3rocm import kv
    torch.manual_seed(4)
    T, nq, nkv, bs, nblk, ctx = 7, 40, 8, 16, 64, 1024
    qkv = torch.randn(T, (nq + 2 * nkv) * 128, device=DEV).to(torch.float16)
    pos = torch.tensor([0, 5, 100, 1023, 64, 7, 512], dtype=torch.int64, device=DEV)
    slots = torch.tensor([3, 17, 200, -1, 511, 1000, 64], dtype=torch.int64, device=DEV)
    cs = glue.rope_cos_sin(ctx, 1e6, DEV)

    def caches():
        return (torch.zeros(nblk, bs, nkv, 128, dtype=torch.int8, device=DEV),
                torch.zeros(nblk, bs, nkv, 128, dtype=torch.int8, device=DEV),
                torch.zeros(nblk, bs, nkv, device=DEV), torch.zeros(nblk, bs, nkv, device=DEV))
    kc1, vc1, ks1, vs1 = caches()
    q1 = torch.empty(T, nq * 128, dtype=torch.float16, device=DEV)
    kv.rope_and_cache_int8(qkv, q1, nq, nkv, pos, cs, kc1, vc1, slots, ks1, vs1)
    kc2, vc2, ks2, vs2 = caches()
    q2 = torch.empty_like(q1)
    work = qkv.clone()
    glue.rope_neox(work, q2, nq, nkv, pos, cs)
    kv.reshape_and_cache_int8(work[:, nq * 128:(nq + nkv) * 128].view(T, nkv, 128),
                              work[:, (nq + nkv) * 128:].view(T, nkv, 128), kc2, vc2, slots, ks2, vs2)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2)
    for a, b in ((kc1, kc2), (vc1, vc2), (ks1, ks2), (vs1, vs2)):
        assert torch.equal(a, b)
