"""The synthetic decode step (exl3rocm.synthetic) against an unfused reference forward on the GPU.

The reference forward uses the already-verified EXL3 linear op (exl3rocm::linear) and int8 KV write
for each matrix and cache row, and fp32 torch for RMSNorm, RoPE, attention over the dequantised
int8 cache (causal inside the verify window) and SiLU * up; the step under test runs the fused
kernels (grouped qkv, residual adds and the activation in the GEMV epilogues, paged attention).
Logits must agree within a normalised tolerance, CUDA-graph replays must equal the eager step bit
for bit, and repeated steps must be identical (the step rewrites the same cache slots).
"""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
SMALL = dict(layers=2, hidden=512, q_heads=4, kv_heads=2, intermediate=1024, vocab=1024)
# fp16 rounding points differ between the fused and the reference paths (norm, rope, attention's
# fp16 probabilities); over two layers the logits stay within these
LOGIT_NRMS = 1e-2
LOGIT_COS = 0.9999


@pytest.fixture(scope="module")
def syn():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from exl3rocm import synthetic
    return synthetic


def _reference_logits(dec, tokens, k_cache, v_cache, k_scale, v_scale):
    from exl3rocm import kv
    s, M = dec.s, dec.M
    qd, kd, d = s.q_heads * s.head, s.kv_heads * s.head, s.head

    def lin(x, w):
        return torch.ops.exl3rocm.linear(x, w.trellis, w.suh, w.svh, w.K, False, True)

    def rms(x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + s.eps)).to(torch.float16) * w

    cs = dec.cos_sin[dec.positions]

    def rope(x, heads):
        x = x.view(M, heads, d)
        c, sn = cs[:, None, :64], cs[:, None, 64:]
        a, b = x[..., :64].float(), x[..., 64:].float()
        return torch.cat([a * c - b * sn, b * c + a * sn], -1).to(torch.float16)

    res = dec.embed[tokens].clone()
    for i, L in enumerate(dec.layers):
        h = rms(res, L.norm_in)
        q = rope(lin(h, L.q), s.q_heads)
        k = rope(lin(h, L.k), s.kv_heads)
        v = lin(h, L.v).view(M, s.kv_heads, d)
        kv.reshape_and_cache_int8(k, v, k_cache[i], v_cache[i], dec.slot_mapping, k_scale[i], v_scale[i])
        out = torch.empty(M, s.q_heads, d, device=DEV)
        for b in range(dec.batch):
            blocks = dec.block_table[b].long()
            K = (k_cache[i][blocks].float() * k_scale[i][blocks][..., None]).reshape(-1, s.kv_heads, d)
            V = (v_cache[i][blocks].float() * v_scale[i][blocks][..., None]).reshape(-1, s.kv_heads, d)
            for j in range(dec.q_len):
                r = b * dec.q_len + j
                n_vis = dec.ctx - dec.q_len + j + 1
                for hq in range(s.q_heads):
                    hk = hq // (s.q_heads // s.kv_heads)
                    sc = (K[:n_vis, hk] @ q[r, hq].float()) / math.sqrt(d)
                    out[r, hq] = torch.softmax(sc, 0) @ V[:n_vis, hk]
        res = res + lin(out.to(torch.float16).view(M, qd), L.o)
        h = rms(res, L.norm_post)
        a = torch.nn.functional.silu(lin(h, L.gate)) * lin(h, L.up)
        res = res + lin(a, L.down)
    h = rms(res, dec.norm_final)
    return lin(h, dec.head)


@pytest.mark.parametrize("batch,q_len", [(2, 1), (1, 4)])
def test_decode_step_matches_reference(syn, batch, q_len):
    shape = syn.DecoderShape(**SMALL)
    dec = syn.SyntheticDecoder(shape, DEV, batch=batch, q_len=q_len, ctx=256, seed=7)
    caches = [[t.clone() for t in ts] for ts in (dec.k_cache, dec.v_cache, dec.k_scale, dec.v_scale)]
    tokens = torch.randint(0, shape.vocab, (dec.M,), device=DEV)
    ref = _reference_logits(dec, tokens, *caches).float()
    dec.step(tokens)
    got = dec.logits.float()
    torch.cuda.synchronize()
    assert torch.isfinite(got).all() and torch.isfinite(ref).all()
    nrms = float((got - ref).pow(2).mean().sqrt() / ref.pow(2).mean().sqrt())
    cos = float(torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0))
    assert nrms <= LOGIT_NRMS and cos >= LOGIT_COS, (nrms, cos)
    # outside the step's own slots the cache is untouched
    for i in range(shape.layers):
        untouched = torch.ones(dec.k_cache[i].shape[0] * shape.block_size, dtype=torch.bool, device=DEV)
        untouched[dec.slot_mapping] = False
        a = dec.k_cache[i].view(-1, shape.kv_heads, shape.head)[untouched]
        b = caches[0][i].view(-1, shape.kv_heads, shape.head)[untouched]
        assert torch.equal(a, b)


def test_decode_step_graph_replay(syn):
    shape = syn.DecoderShape(**SMALL)
    dec = syn.SyntheticDecoder(shape, DEV, batch=2, q_len=1, ctx=512, seed=3)
    tokens = torch.randint(0, shape.vocab, (dec.M,), device=DEV)
    st = torch.cuda.Stream(DEV)
    st.wait_stream(torch.cuda.current_stream(DEV))
    dec.reserve(st)
    with torch.cuda.stream(st):
        dec.step(tokens)
        eager = dec.logits.clone()
        dec.step(tokens)
        assert torch.equal(dec.logits, eager)  # a step rewrites the same slots: repeatable
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            dec.step(tokens)
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(dec.logits, eager)
    del g


def test_fused_step_matches_unfused(syn):
    """The fused step (RMSNorm inside the GEMVs, RoPE inside the KV write) against the same model run
    with separate RMSNorm, RoPE and KV-write launches: only the norms' per-row scales may round
    differently."""
    shape = syn.DecoderShape(**SMALL)
    a = syn.SyntheticDecoder(shape, DEV, batch=3, q_len=1, ctx=256, seed=11)
    b = syn.SyntheticDecoder(shape, DEV, batch=3, q_len=1, ctx=256, seed=11, fused=False)
    tokens = torch.randint(0, shape.vocab, (a.M,), device=DEV)
    a.step(tokens)
    b.step(tokens)
    got, ref = a.logits.float(), b.logits.float()
    nrms = float((got - ref).pow(2).mean().sqrt() / ref.pow(2).mean().sqrt())
    assert nrms <= 2e-3, nrms
    assert a.launches_per_step() == 7 * shape.layers + 1
