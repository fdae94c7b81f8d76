"""The int8 KV cache against an fp16 cache on a synthetic decoder: the reference's KL gate.

The reference accepts a quantised KV cache when the next-token distributions it gives stay within
KL <= 0.01 of an fp16 cache's (configs/GATE_RATIONALE.md:7; it reports KL 0.00007 for int8 on long
text, vllm_plugin/README.md:113).  Here a seeded synthetic decoder (exl3rocm.synthetic weights: EXL3
linears through this library) runs the same teacher-forced token sequence twice, one token per step:
once with this library's int8 write and paged attention, once with fp16 K/V rows and an fp32 softmax
attention in torch.  Everything else is shared.  The mean KL(p_fp16 || p_int8) over the steps must
stay within the gate; the distributions must be far from uniform, so the gate measures something.
"""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
KL_GATE = 0.01
STEPS = 320
# the synthetic model's logits have about unit spread; a trained model's are several times wider, so
# both runs' logits are sharpened by the same factor before the softmax (this makes the gate stricter)
LOGIT_SCALE = 6.0
SHAPE = dict(layers=4, hidden=1024, q_heads=8, kv_heads=2, intermediate=2048, vocab=8192)


@pytest.fixture(scope="module")
def syn():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from exl3rocm import synthetic
    return synthetic


def _run(dec, tokens, int8: bool):
    """Teacher-forced decode of `tokens`; returns the fp32 log-probabilities of every step."""
    from exl3rocm import kv
    s = dec.s
    d, hq, hkv = s.head, s.q_heads, s.kv_heads
    n = tokens.shape[0]
    bs = s.block_size
    nblk = (n + bs - 1) // bs
    bt = torch.arange(nblk, dtype=torch.int32, device=DEV).view(1, nblk)
    if int8:
        kc = [torch.zeros((nblk, bs, hkv, d), dtype=torch.int8, device=DEV) for _ in range(s.layers)]
        vc = [torch.zeros_like(c) for c in kc]
        ks = [torch.zeros((nblk, bs, hkv), dtype=torch.float32, device=DEV) for _ in range(s.layers)]
        vs = [torch.zeros_like(c) for c in ks]
    else:
        kf = [torch.zeros((n, hkv, d), dtype=torch.float16, device=DEV) for _ in range(s.layers)]
        vf = [torch.zeros_like(c) for c in kf]
    cos_sin = dec.cos_sin

    def lin(x, w):
        return torch.ops.exl3rocm.linear(x, w.trellis, w.suh, w.svh, w.K, False, True)

    def rms(x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + s.eps)).to(torch.float16) * w

    def rope(x, heads, pos):
        x = x.view(1, heads, d)
        cs = cos_sin[pos]
        c, sn = cs[None, :64], cs[None, 64:]
        a, b = x[..., :64].float(), x[..., 64:].float()
        return torch.cat([a * c - b * sn, b * c + a * sn], -1).to(torch.float16)

    out = []
    for p in range(n):
        res = dec.embed[tokens[p:p + 1]].clone()
        slot = torch.tensor([p], dtype=torch.int64, device=DEV)
        for i, L in enumerate(dec.layers):
            h = rms(res, L.norm_in)
            q, k = rope(lin(h, L.q), hq, p), rope(lin(h, L.k), hkv, p)
            v = lin(h, L.v).view(1, hkv, d)
            attn = torch.empty((1, hq, d), dtype=torch.float16, device=DEV)
            if int8:
                kv.reshape_and_cache_int8(k, v, kc[i], vc[i], slot, ks[i], vs[i])
                kv.attention_int8(q=q, k=kc[i], v=vc[i], out=attn,
                                  cu_seqlens_q=torch.tensor([0, 1], dtype=torch.int32, device=DEV), max_seqlen_q=1,
                                  seqused_k=torch.tensor([p + 1], dtype=torch.int32, device=DEV), block_table=bt,
                                  softmax_scale=1.0 / math.sqrt(d), k_scale_cache=ks[i], v_scale_cache=vs[i],
                                  max_seqlen_k=n)
            else:
                kf[i][p] = k[0]
                vf[i][p] = v[0]
                K, V = kf[i][:p + 1].float(), vf[i][:p + 1].float()
                g = hq // hkv
                Kg, Vg = K.repeat_interleave(g, dim=1), V.repeat_interleave(g, dim=1)  # query head h -> h // g
                sc = torch.einsum("hd,thd->ht", q[0].float(), Kg) / math.sqrt(d)
                attn[0] = torch.einsum("ht,thd->hd", torch.softmax(sc, -1), Vg).to(torch.float16)
            res = res + lin(attn.view(1, hq * d), L.o)
            h = rms(res, L.norm_post)
            res = res + lin(torch.nn.functional.silu(lin(h, L.gate)) * lin(h, L.up), L.down)
        logits = lin(rms(res, dec.norm_final), dec.head).float()
        out.append(torch.log_softmax(LOGIT_SCALE * logits[0], -1))
    return torch.stack(out)


def test_int8_kv_within_the_kl_gate_of_an_fp16_cache(syn):
    shape = syn.DecoderShape(**SHAPE)
    dec = syn.SyntheticDecoder(shape, DEV, batch=1, q_len=1, ctx=512, seed=4242)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(17)
    tokens = torch.randint(0, shape.vocab, (STEPS,), generator=gen, device=DEV)
    lp16 = _run(dec, tokens, int8=False)
    lp8 = _run(dec, tokens, int8=True)
    kl = (lp16.exp() * (lp16 - lp8)).sum(-1)
    entropy = -(lp16.exp() * lp16).sum(-1)
    assert torch.isfinite(kl).all()
    # far from uniform (log 8192 = 9.0): the distributions carry information
    assert float(entropy.mean()) < 0.8 * math.log(shape.vocab), float(entropy.mean())
    assert float(kl.mean()) <= KL_GATE, (float(kl.mean()), float(kl.max()))
