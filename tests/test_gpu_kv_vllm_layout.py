"""The int8 KV kernels on vLLM's own per-token-head cache layout, through the plugin's routing.

vLLM keeps an int8_per_token_head cache as kv_cache [num_blocks][2][block_size][Hkv][128 + 4] int8, each
row's fp32 scale inline after it and the K and V halves interleaved per block (scale views built by
TritonAttentionImpl._ensure_scale_caches).  The kernels take the views' strides (kv.cache_layout) and,
for rows that are not 16-byte aligned, copy with 4-byte loads.  Checked here:
  * this library's write into vLLM's layout equals its write into the dense layout, byte for byte, and
    reads back as vLLM's own write of the same rows does (codes within one step, scales within 2 ulp:
    vLLM's GPU build divides approximately);
  * attention over a cache vLLM's kernel wrote, through the routed ``unified_attention`` (decode,
    4-token verify, and a 64-token prefill chunk through the gather + fp16 route), against vLLM's own
    unified attention on the same cache, within nRMS 2e-3 / cos 0.9999; and the padded layout's result
    equals the dense layout's bit for bit.
"""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
HKV, HQ, D, BS = 8, 40, 128, 16


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    try:
        from vllm.v1.attention.backends import triton_attn as ta
        from vllm.v1.attention.ops.triton_reshape_and_cache_flash import \
            triton_reshape_and_cache_flash_per_token_head_quant as vllm_write
        from vllm.v1.kv_cache_interface import KVQuantMode
    except ImportError as e:
        pytest.skip(f"vLLM's Triton backend is not importable here: {e}")
    from exl3rocm import kv, plugin
    vllm_attention = ta.unified_attention
    routing = plugin._install_kv_hooks()
    assert routing is not None and ta.unified_attention is not vllm_attention
    return types.SimpleNamespace(ta=ta, vllm_write=vllm_write, vllm_attention=vllm_attention, Mode=KVQuantMode,
                                 kv=kv, routing=routing)


def vllm_cache(env, nblk):
    """A zeroed vLLM int8 per-token-head cache and its K / V halves and scale views."""
    cache = torch.zeros((nblk, 2, BS, HKV, D + 4), dtype=torch.int8, device=DEV)
    holder = types.SimpleNamespace(_k_scale_cache=None, _v_scale_cache=None)
    env.ta.TritonAttentionImpl._ensure_scale_caches(holder, cache)
    kc, vc = cache.unbind(1)
    return cache, kc, vc, holder._k_scale_cache, holder._v_scale_cache


def inputs(n, seed):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    x = torch.randn((n, HKV, D), generator=g, device=DEV)
    x[..., :2] *= 8
    return x.half()


def nrms(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt())


def test_write_into_vllm_layout(env):
    ctx, nblk = 300, 24
    key, val = inputs(ctx, 1), inputs(ctx, 2)
    slots = torch.randperm(nblk * BS, device=DEV)[:ctx].to(torch.int64)
    _, kc, vc, ks, vs = vllm_cache(env, nblk)
    env.kv.reshape_and_cache_int8(key, val, kc[..., :D], vc[..., :D], slots, ks, vs)
    # the dense layout, same kernel
    dk, dv = torch.zeros((nblk, BS, HKV, D), dtype=torch.int8, device=DEV), torch.zeros((nblk, BS, HKV, D), dtype=torch.int8, device=DEV)
    dks, dvs = torch.zeros((nblk, BS, HKV), device=DEV), torch.zeros((nblk, BS, HKV), device=DEV)
    env.kv.reshape_and_cache_int8(key, val, dk, dv, slots, dks, dvs)
    assert torch.equal(kc[..., :D], dk) and torch.equal(vc[..., :D], dv)
    # written slots only: vLLM initialises its scale views to 1
    b, o = slots // BS, slots % BS
    assert torch.equal(ks[b, o], dks[b, o]) and torch.equal(vs[b, o], dvs[b, o])
    # vLLM's own write of the same rows
    _, kc2, vc2, ks2, vs2 = vllm_cache(env, nblk)
    env.vllm_write(key, val, kc2, vc2, ks2, vs2, slots)
    for ours, theirs, so, st in ((kc, kc2, ks, ks2), (vc, vc2, vs, vs2)):
        dq = (ours[b, o][..., :D].int() - theirs[b, o][..., :D].int()).abs()
        assert dq.max().item() <= 1 and (dq > 0).float().mean().item() <= 1e-3
        assert ((so[b, o] - st[b, o]).abs() / st[b, o].abs().clamp_min(1e-30)).max().item() <= 2.5e-7


@pytest.mark.parametrize("batch,ctx,q_len", [(2, 3000, 1), (1, 4096, 4), (2, 700, 64)])
def test_routed_attention_matches_vllm(env, batch, ctx, q_len):
    nb_seq = (ctx + BS - 1) // BS
    nblk = batch * nb_seq + 3
    perm = torch.randperm(nblk, device=DEV).to(torch.int32)
    bt = perm[: batch * nb_seq].view(batch, nb_seq).contiguous()
    pos = torch.arange(ctx, device=DEV)
    slots = torch.cat([bt[s, pos // BS].to(torch.int64) * BS + pos % BS for s in range(batch)])
    key, val = inputs(batch * ctx, 10 + ctx), inputs(batch * ctx, 20 + ctx)
    _, kc, vc, ks, vs = vllm_cache(env, nblk)
    env.vllm_write(key, val, kc, vc, ks, vs, slots)
    g = torch.Generator(device=DEV)
    g.manual_seed(q_len)
    q = torch.randn((batch * q_len, HQ, D), generator=g, device=DEV).half()
    kw = dict(q=q, k=kc, v=vc, cu_seqlens_q=torch.arange(0, batch * q_len + 1, q_len, dtype=torch.int32, device=DEV),
              max_seqlen_q=q_len, seqused_k=torch.full((batch,), ctx, dtype=torch.int32, device=DEV),
              max_seqlen_k=ctx, softmax_scale=D ** -0.5, causal=True, window_size=(-1, -1), block_table=bt,
              softcap=0.0, q_descale=None, k_descale=None, v_descale=None,
              kv_quant_mode=env.Mode.INT8_PER_TOKEN_HEAD, k_scale_cache=ks, v_scale_cache=vs)
    ref = torch.zeros_like(q)
    env.vllm_attention(**dict(kw, out=ref))
    out = torch.full_like(q, float("nan"))
    env.ta.unified_attention(**dict(kw, out=out))  # routed to this library
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    e, c = nrms(out, ref), float(torch.nn.functional.cosine_similarity(out.double().flatten(), ref.double().flatten(), 0))
    assert e <= 2e-3 and c >= 0.9999, (e, c)
    if q_len < env.routing.prefill_min_q:
        # the same rows in the dense layout give the same result bit for bit
        dk, dv = kc[..., :D].contiguous(), vc[..., :D].contiguous()
        out2 = torch.empty_like(q)
        env.kv.attention_int8(**dict(kw, k=dk, v=dv, out=out2, k_scale_cache=ks.contiguous(),
                                     v_scale_cache=vs.contiguous()))
        torch.cuda.synchronize()
        assert torch.equal(out, out2)
