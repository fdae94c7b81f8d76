"""The CUDA KV kernels against the reference's own kernels.

1. On the committed fixtures (tests/golden/kv_golden.npz: vLLM 0.22's int8 per-token-head Triton kernels
   and the reference's kv_int4.py, run on seeded inputs by tests/golden/make_kv_golden.py): the same
   inputs through this library's C ABI; int8 codes and scales bit-exact, int4 codes / tags / exact rows
   bit-exact and scale words as in tests/test_kv_golden.py, attention within nRMS 2e-3 / cos 0.9999.
2. At the BASELINE contexts (32k and 64k tokens, B = 1; 4k, B = 8), int8: vLLM's own Triton write and
   unified attention, compiled for this GPU, side by side with this library on the same inputs (writes
   equal up to the GPU's approximate division in vLLM's build, attention within the gate).  int4: the kernels against the oracle (pinned to the
   reference by the fixtures) — codes re-derived for a sample of rows, attention over the whole context.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import kv_oracle as KV
from tests.test_kv_golden import (ATTN_COS, ATTN_NRMS, QUERIES, check_attention, cos, exact_rows_match,
                                  metadata, nrms, scale_words_match)

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
D, BS = 128, 16
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kv_golden.npz")


@pytest.fixture(scope="module")
def g():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="module")
def xkv():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from exl3rocm import kv
    return kv


def t(a, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return x if dtype is None else x.to(dtype)


def _stream():
    return torch.cuda.current_stream().cuda_stream


def test_int8_write_bit_exact_to_vllm_fixture(g, xkv):
    nb = int(g["num_blocks"])
    kc = torch.zeros((nb, BS, 2, D), dtype=torch.int8, device=DEV)
    vc = torch.zeros_like(kc)
    ks = torch.zeros((nb, BS, 2), dtype=torch.float32, device=DEV)
    vs = torch.zeros_like(ks)
    xkv.reshape_and_cache_int8(t(g["key"]), t(g["value"]), kc, vc, t(g["slots"]), ks, vs)
    assert (kc.cpu().numpy() == g["int8_key_cache"]).all() and (vc.cpu().numpy() == g["int8_value_cache"]).all()
    assert (ks.cpu().numpy().view(np.uint32) == g["int8_k_scale"].view(np.uint32)).all()
    assert (vs.cpu().numpy().view(np.uint32) == g["int8_v_scale"].view(np.uint32)).all()


@pytest.mark.parametrize("name,qkey,qsl", QUERIES)
def test_int8_attention_matches_vllm_fixture(g, xkv, name, qkey, qsl):
    q = t(g[qkey])
    out = torch.empty_like(q)
    xkv.attention_int8(q=q, k=t(g["int8_key_cache"]), v=t(g["int8_value_cache"]), out=out,
                       cu_seqlens_q=t(qsl.astype(np.int32)), max_seqlen_q=int(np.diff(qsl).max()),
                       seqused_k=t(g["seq_lens"]), block_table=t(g["block_table"]), softmax_scale=D ** -0.5,
                       k_scale_cache=t(g["int8_k_scale"]), v_scale_cache=t(g["int8_v_scale"]),
                       max_seqlen_k=int(g["seq_lens"].max()))
    check_attention(out.cpu().numpy(), g[f"int8_out_{name}"].astype(np.float64))


def _int4_write_via_abi(g, layer):
    """The fixture's batch through exl3b_kv_int4_write with the reference's own centering biases."""
    from exl3rocm import _lib
    nb = int(g["num_blocks"])
    sl = g["seq_lens"]
    kc = torch.zeros((nb, BS, 2, D // 2), dtype=torch.uint8, device=DEV)
    vc = torch.zeros_like(kc)
    ks = torch.zeros((nb, BS, 2), dtype=torch.float32, device=DEV)
    vs = torch.zeros_like(ks)
    rows = KV.SINKS + KV.TAIL
    exk = torch.zeros((len(sl), rows, 2, D), dtype=torch.float16, device=DEV)
    exv = torch.zeros_like(exk)
    tag = torch.full((len(sl), rows), -1, dtype=torch.int32, device=DEV)
    key, val, slots = t(g["key"]), t(g["value"]), t(g["slots"])
    p = f"int4_{layer}_"
    bk = t(g[p + "bias_k"]) if p + "bias_k" in g else None
    bv = t(g[p + "bias_v"]) if p + "bias_v" in g else None
    qsl, slt = t(g["qsl_write"]), t(sl)
    seq_slots = torch.arange(len(sl), dtype=torch.int32, device=DEV)
    signs = t(g["signs"])
    _lib.call("exl3b_kv_int4_write", key.data_ptr(), val.data_ptr(), 0, key.shape[0], 2, D, key.stride(0),
              key.stride(1), val.stride(0), val.stride(1), kc.data_ptr(), vc.data_ptr(), ks.data_ptr(), vs.data_ptr(),
              slots.data_ptr(), BS, signs.data_ptr(), bk.data_ptr() if bk is not None else None,
              bv.data_ptr() if bv is not None else None, qsl.data_ptr(), slt.data_ptr(), seq_slots.data_ptr(),
              len(sl), exk.data_ptr(), exv.data_ptr(), tag.data_ptr(), None, _stream())
    torch.cuda.synchronize()
    return kc, vc, ks, vs, exk, exv, tag, seq_slots


@pytest.mark.parametrize("layer", ["plain", "centered"])
def test_int4_write_matches_reference_fixture(g, layer):
    kc, vc, ks, vs, exk, exv, tag, _ = _int4_write_via_abi(g, layer)
    p = f"int4_{layer}_"
    assert (kc.cpu().numpy() == g[p + "key_cache"]).all() and (vc.cpu().numpy() == g[p + "value_cache"]).all()
    scale_words_match(ks.cpu().numpy(), g[p + "k_scale_bits"])
    scale_words_match(vs.cpu().numpy(), g[p + "v_scale_bits"])
    exact_rows_match(g, layer, exk.cpu().numpy(), exv.cpu().numpy(), tag.cpu().numpy())


@pytest.mark.parametrize("layer", ["plain", "centered"])
@pytest.mark.parametrize("name,qkey,qsl", QUERIES)
def test_int4_attention_matches_reference_fixture(g, layer, name, qkey, qsl):
    """Over the reference's own cache bytes and this library's exact rows (bit-equal to the reference's)."""
    from exl3rocm import _lib
    kc, vc, ks, vs, exk, exv, tag, seq_slots = _int4_write_via_abi(g, layer)
    p = f"int4_{layer}_"
    q = t(g[qkey])
    out = torch.empty_like(q)
    T = q.shape[0]
    nbytes = int(_lib.lib().exl3b_kv_attn_workspace_bytes(T, 10, 2, 2, int(g["seq_lens"].max())))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    vmean = t(g["mean_v"]) if layer == "centered" else None
    kref, vref = t(g[p + "key_cache"]), t(g[p + "value_cache"])
    ksr, vsr = t(g[p + "k_scale_bits"].view(np.float32)), t(g[p + "v_scale_bits"].view(np.float32))
    bt, sl, qs = t(g["block_table"]), t(g["seq_lens"]), t(qsl.astype(np.int32))
    _lib.call("exl3b_kv_int4_attn", q.data_ptr(), out.data_ptr(), T, 10, 2, D, kref.data_ptr(), vref.data_ptr(),
              ksr.data_ptr(), vsr.data_ptr(), BS, bt.data_ptr(), bt.stride(0), sl.data_ptr(), qs.data_ptr(), 2,
              int(np.diff(qsl).max()), int(g["seq_lens"].max()), D ** -0.5, t(g["signs"]).data_ptr(), exk.data_ptr(),
              exv.data_ptr(), tag.data_ptr(), seq_slots.data_ptr(), vmean.data_ptr() if vmean is not None else None,
              ws.data_ptr(), ws.numel(), None, _stream())
    torch.cuda.synchronize()
    check_attention(out.cpu().numpy(), g[p + f"out_{name}"].astype(np.float64))


def test_int4_centering_through_the_python_surface(g, xkv):
    """kv.set_kv_means -> reshape_and_cache / attention: the biases the host derives equal the
    reference's bit for bit, so the cache bytes equal the centred fixture's."""
    xkv.set_kv_means({"centered": {"k": g["mean_k"], "v": g["mean_v"]}})
    try:
        b = xkv.layer_bias("centered", 2, DEV)
        assert (b["k"].cpu().numpy() == g["int4_centered_bias_k"]).all()
        assert (b["v"].cpu().numpy() == g["int4_centered_bias_v"]).all()
        nb = int(g["num_blocks"])
        kc = torch.zeros((nb, BS, 2, D // 2), dtype=torch.uint8, device=DEV)
        vc = torch.zeros_like(kc)
        ks = torch.zeros((nb, BS, 2), dtype=torch.float32, device=DEV)
        vs = torch.zeros_like(ks)
        assert (xkv.rht_signs(DEV).cpu().numpy() == g["signs"]).all()  # the fixtures' sign vector
        xkv.reshape_and_cache(t(g["key"]), t(g["value"]), kc, vc, t(g["slots"]), k_scale_cache=ks, v_scale_cache=vs,
                              layer_name="centered")
        assert (kc.cpu().numpy() == g["int4_centered_key_cache"]).all()
        assert (vc.cpu().numpy() == g["int4_centered_value_cache"]).all()
    finally:
        xkv.set_kv_means(None)


# ---------------------------------------------------------------------------------------------
# BASELINE contexts: vLLM's own int8 Triton kernels on this GPU, side by side
# ---------------------------------------------------------------------------------------------
def _kv_inputs(n, heads, seed):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    x = torch.randn((n, heads, D), generator=gen, device=DEV)
    ch = torch.randperm(D, generator=gen, device=DEV)[:2]
    x[..., ch] *= 8
    return x.half()


def _paged_layout(batch, ctx, seed):
    nb = (ctx + BS - 1) // BS
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    bt = torch.randperm(batch * nb, generator=gen, device=DEV).to(torch.int32).view(batch, nb)
    pos = torch.arange(ctx, device=DEV)
    slots = torch.cat([bt[s, pos // BS].to(torch.int64) * BS + pos % BS for s in range(batch)])
    return batch * nb, bt, slots


@pytest.mark.parametrize("ctx,batch", [(32768, 1), (65536, 1), (4096, 8)])
def test_int8_long_context_matches_vllm_triton(xkv, ctx, batch):
    try:
        from vllm.v1.attention.ops.triton_reshape_and_cache_flash import \
            triton_reshape_and_cache_flash_per_token_head_quant
        from vllm.v1.attention.ops.triton_unified_attention import unified_attention
        from vllm.v1.kv_cache_interface import KVQuantMode
    except ImportError as e:
        pytest.skip(f"vLLM's Triton kernels are not importable here: {e}")
    HKV, HQ = 8, 40
    nblk, bt, slots = _paged_layout(batch, ctx, 7 + ctx + batch)
    key, val = _kv_inputs(batch * ctx, HKV, 11 + ctx), _kv_inputs(batch * ctx, HKV, 13 + ctx)
    caches = []
    for writer in ("vllm", "ours"):
        kc = torch.zeros((nblk, BS, HKV, D), dtype=torch.int8, device=DEV)
        vc = torch.zeros_like(kc)
        ks = torch.zeros((nblk, BS, HKV), dtype=torch.float32, device=DEV)
        vs = torch.zeros_like(ks)
        if writer == "vllm":
            triton_reshape_and_cache_flash_per_token_head_quant(key, val, kc, vc, ks, vs, slots)
        else:
            xkv.reshape_and_cache_int8(key, val, kc, vc, slots, ks, vs)
        caches.append((kc, vc, ks, vs))
    # vLLM's Triton build divides with the GPU's approximate fp32 division (the fixtures, run with IEEE
    # division, are bit-exact): scales agree within 2 units in the last place, and a code may sit one
    # step away where x / scale lands next to an integer
    for (cv, sv), (co, so) in (((caches[0][0], caches[0][2]), (caches[1][0], caches[1][2])),
                               ((caches[0][1], caches[0][3]), (caches[1][1], caches[1][3]))):
        rel = ((sv - so).abs() / so.abs().clamp_min(1e-30)).max().item()
        dq = (cv.int() - co.int()).abs()
        frac = (dq > 0).float().mean().item()
        assert rel <= 2.5e-7 and dq.max().item() <= 1 and frac <= 1e-3, (rel, dq.max().item(), frac)
    kc, vc, ks, vs = caches[1]
    del caches
    gen = torch.Generator(device=DEV)
    gen.manual_seed(99 + ctx)
    q = torch.randn((batch, HQ, D), generator=gen, device=DEV).half()
    qsl = torch.arange(batch + 1, dtype=torch.int32, device=DEV)
    sl = torch.full((batch,), ctx, dtype=torch.int32, device=DEV)
    ref = torch.zeros_like(q)
    segs = 16
    unified_attention(q=q, k=kc, v=vc, out=ref, cu_seqlens_q=qsl, max_seqlen_q=1, seqused_k=sl, max_seqlen_k=ctx,
                      softmax_scale=D ** -0.5, causal=True, window_size=(-1, -1), block_table=bt, softcap=0.0,
                      q_descale=None, k_descale=None, v_descale=None, seq_threshold_3D=64,
                      num_par_softmax_segments=segs,
                      softmax_segm_output=torch.empty((batch, HQ, segs, D), dtype=torch.float32, device=DEV),
                      softmax_segm_max=torch.empty((batch, HQ, segs), dtype=torch.float32, device=DEV),
                      softmax_segm_expsum=torch.empty((batch, HQ, segs), dtype=torch.float32, device=DEV),
                      kv_quant_mode=KVQuantMode.INT8_PER_TOKEN_HEAD, k_scale_cache=ks, v_scale_cache=vs)
    out = torch.empty_like(q)
    xkv.attention_int8(q=q, k=kc, v=vc, out=out, cu_seqlens_q=qsl, max_seqlen_q=1, seqused_k=sl, block_table=bt,
                       softmax_scale=D ** -0.5, k_scale_cache=ks, v_scale_cache=vs, max_seqlen_k=ctx)
    torch.cuda.synchronize()
    o, r = out.float().cpu().numpy(), ref.float().cpu().numpy()
    assert nrms(o, r) <= ATTN_NRMS and cos(o, r) >= ATTN_COS, (nrms(o, r), cos(o, r))


@pytest.mark.parametrize("ctx", [32768, 65536])
def test_int4_long_context_against_the_oracle(xkv, ctx):
    """int4 at the BASELINE contexts, B = 1, exact rows on: a sample of 2048 rows re-quantised by the
    oracle (codes bit-exact, scale words per the fixture rule), and decode + 4-token verify attention
    against the float64 oracle over the whole context."""
    HKV, HQ = 8, 40
    nblk, bt, slots = _paged_layout(1, ctx, 17 + ctx)
    key, val = _kv_inputs(ctx, HKV, 19 + ctx), _kv_inputs(ctx, HKV, 23 + ctx)
    xkv.configure_request_slots(1)
    xkv._req["slot"] = None
    xkv._exact.pop("long", None)
    xkv.set_batch_slots(torch.zeros(1, dtype=torch.int32, device=DEV))
    kc = torch.zeros((nblk, BS, HKV, D // 2), dtype=torch.uint8, device=DEV)
    vc = torch.zeros_like(kc)
    ks = torch.zeros((nblk, BS, HKV), dtype=torch.float32, device=DEV)
    vs = torch.zeros_like(ks)
    chunk = 8192
    for t0 in range(0, ctx, chunk):
        xkv.reshape_and_cache(key[t0:t0 + chunk], val[t0:t0 + chunk], kc, vc, slots[t0:t0 + chunk], k_scale_cache=ks,
                              v_scale_cache=vs, layer_name="long",
                              query_start_loc=torch.tensor([0, min(chunk, ctx - t0)], dtype=torch.int32, device=DEV),
                              seq_lens=torch.tensor([min(t0 + chunk, ctx)], dtype=torch.int32, device=DEV))
    torch.cuda.synchronize()
    signs = xkv.rht_signs(DEV).cpu().numpy()
    rng = np.random.default_rng(ctx)
    sample = rng.choice(ctx, size=2048, replace=False)
    s_cpu = slots.cpu().numpy()
    kh = key.cpu().numpy()
    codes, sbits = KV.int4_quantize_rows(KV.fwht128_f32(kh[sample].astype(np.float32) * signs))
    b, o = s_cpu[sample] // BS, s_cpu[sample] % BS
    assert (kc.cpu().numpy()[b, o] == KV.pack_nibbles(codes)).all()
    scale_words_match(ks.cpu().numpy()[b, o], sbits.view(np.float32))
    ex = xkv._exact["long"]
    kcn, vcn, ksn, vsn = kc.cpu().numpy(), vc.cpu().numpy(), ks.cpu().numpy(), vs.cpu().numpy()
    exk, exv, tag = ex["k"].cpu().numpy(), ex["v"].cpu().numpy(), ex["tag"].cpu().numpy()
    btn = bt.cpu().numpy()
    for q_len in (1, 4):
        gen = torch.Generator(device=DEV)
        gen.manual_seed(5 + q_len)
        q = torch.randn((q_len, HQ, D), generator=gen, device=DEV).half()
        out = torch.empty_like(q)
        qsl = torch.tensor([0, q_len], dtype=torch.int32, device=DEV)
        sl = torch.tensor([ctx], dtype=torch.int32, device=DEV)
        xkv.attention(q=q, k=kc, v=vc, out=out, cu_seqlens_q=qsl, max_seqlen_q=q_len, seqused_k=sl, block_table=bt,
                      softmax_scale=D ** -0.5, k_scale_cache=ks, v_scale_cache=vs, max_seqlen_k=ctx, layer_name="long")
        torch.cuda.synchronize()
        ref = KV.int4_attention(q.cpu().numpy(), kcn, vcn, ksn, vsn, exk, exv, tag, [0], btn, [ctx],
                                np.array([0, q_len]), D ** -0.5, signs)
        check_attention(out.cpu().numpy(), ref)
