"""The synthetic decoder's other modes against its tested fused int8 step (tests/test_gpu_decoder.py).

* GEMM linears (the route of steps above 16 rows and of prefill: exl3b_gemm, separate RMSNorm,
  SiLU * up and residual adds) against the fused GEMV step on the same model, tokens and cache;
* the int4 cache: the GEMV step against the GEMM step on the same int4 cache;
* prefill: the last position's next token from ``prefill`` of a prompt, against decoding the
  prompt's last token after prefilling all but it (two routes through the same cache writes).
Logits within nRMS 1e-2 and cosine 0.9999 (the two routes round norms, activations and residual adds
at different points), as the fused step is held to its unfused reference.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
SMALL = dict(layers=2, hidden=512, q_heads=4, kv_heads=2, intermediate=1024, vocab=1024)


@pytest.fixture(scope="module")
def syn():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from exl3rocm import synthetic
    return synthetic


def close(a, b):
    a, b = a.float(), b.float()
    e = float((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt())
    c = float(torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0))
    assert torch.isfinite(a).all() and e <= 1e-2 and c >= 0.9999, (e, c)


@pytest.mark.parametrize("kv_cache", ["int8", "int4"])
def test_gemm_route_matches_gemv_step(syn, kv_cache):
    shape = syn.DecoderShape(**SMALL)
    a = syn.SyntheticDecoder(shape, DEV, batch=4, q_len=1, ctx=256, seed=21, kv_cache=kv_cache)
    b = syn.SyntheticDecoder(shape, DEV, batch=4, q_len=1, ctx=256, seed=21, kv_cache=kv_cache, gemm_linears=True)
    tokens = torch.randint(0, shape.vocab, (4,), device=DEV)
    a.step(tokens)
    b.step(tokens)
    torch.cuda.synchronize()
    close(b.logits, a.logits)


def test_batched_step_of_32_rows(syn):
    """More than 16 rows: the GEMM route by default, equal to 32 rows of the GEMV route's results."""
    shape = syn.DecoderShape(**SMALL)
    big = syn.SyntheticDecoder(shape, DEV, batch=32, q_len=1, ctx=128, seed=22)
    assert big.batched
    tokens = torch.randint(0, shape.vocab, (32,), device=DEV)
    big.step(tokens)
    # the same rows through the GEMV route, 16 at a time, over the same caches
    parts = []
    for h in (0, 16):
        half = syn.SyntheticDecoder(shape, DEV, batch=16, q_len=1, ctx=128, seed=22, weights_of=big,
                                    gemm_linears=False)
        for i in range(shape.layers):
            for dst, src in ((half.k_cache, big.k_cache), (half.v_cache, big.v_cache), (half.k_scale, big.k_scale),
                             (half.v_scale, big.v_scale)):
                nb = dst[i].shape[0]
                dst[i].copy_(src[i][h * nb // 16: (h + 16) * nb // 16])
        half.step(tokens[h:h + 16])
        parts.append(half.logits.clone())
    torch.cuda.synchronize()
    close(big.logits, torch.cat(parts))


@pytest.mark.parametrize("kv_cache", ["int8", "int4"])
def test_prefill_then_decode(syn, kv_cache):
    shape = syn.DecoderShape(**SMALL)
    P = 208  # a multiple of the block size
    dec = syn.SyntheticDecoder(shape, DEV, batch=1, q_len=1, ctx=P, seed=23, kv_cache=kv_cache)
    prompt = torch.randint(0, shape.vocab, (P,), device=DEV)
    nxt = dec.prefill(prompt)
    # the same prompt: prefill all but the last token, then one decode step at position P - 1
    dec2 = syn.SyntheticDecoder(shape, DEV, batch=1, q_len=1, ctx=P, seed=23, kv_cache=kv_cache, weights_of=dec)
    dec2.prefill(prompt[:-1])
    dec2.step(prompt[-1:])
    torch.cuda.synchronize()
    close(dec2.logits, dec.prefill_logits)
    assert int(nxt[0]) == int(torch.argmax(dec.prefill_logits[0]))
