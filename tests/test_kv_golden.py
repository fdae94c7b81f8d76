"""The KV oracle against the reference's own kernels (CPU; no GPU needed).

tests/golden/kv_golden.npz holds the outputs of vLLM 0.22's int8 per-token-head Triton kernels and of
the reference's vllm_plugin/exl3rocm/kv_int4.py (write and attention, with and without centering),
run on seeded inputs under Triton's CPU interpreter by tests/golden/make_kv_golden.py.  These tests pin
oracle/kv_oracle.py to them; the GPU kernels are then checked against both (tests/test_gpu_kv_golden.py).

Bars: int8 codes and scales bit-exact; int4 codes, tags and exact rows bit-exact; int4 scale words
bit-exact except in rows where the row mean (a sum of 128 values) rounds differently in the
reference's summation order (at most 1 % of rows, one unit in the last place, the same zero point);
attention within a normalised RMS of 2e-3 and a cosine of 0.9999 of the reference's fp16 outputs.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import kv_oracle as KV

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kv_golden.npz")
ATTN_NRMS, ATTN_COS = 2e-3, 0.9999
D, BS = 128, 16


@pytest.fixture(scope="module")
def g():
    return dict(np.load(GOLDEN))


def nrms(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(np.sqrt(np.mean((a - b) ** 2)) / np.sqrt(np.mean(b ** 2)))


def cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def check_attention(got, ref):
    assert nrms(got, ref) <= ATTN_NRMS and cos(got, ref) >= ATTN_COS, (nrms(got, ref), cos(got, ref))


def scale_words_match(ours: np.ndarray, ref: np.ndarray) -> None:
    """Scale words: equal, or (in at most 1 % of rows) one unit apart in the 28 scale bits with the
    same zero point."""
    ours, ref = ours.view(np.uint32).ravel(), ref.view(np.uint32).ravel()
    diff = np.nonzero(ours != ref)[0]
    assert diff.size <= max(1, ours.size // 100), diff.size
    assert ((ours[diff] & 0xF) == (ref[diff] & 0xF)).all()
    assert (np.abs((ours[diff] >> 4).astype(np.int64) - (ref[diff] >> 4).astype(np.int64)) <= 1).all()


def metadata(g):
    sl = g["seq_lens"]
    pos = np.concatenate([np.arange(L) for L in sl])
    rs = np.concatenate([np.full(L, s) for s, L in enumerate(sl)])
    after = np.concatenate([np.full(L, L) for L in sl])
    return sl, pos, rs, after


QUERIES = (("decode", "q_decode", np.array([0, 1, 2])), ("verify", "q_verify", np.array([0, 4, 8])))


def test_int8_write_bit_exact_to_vllm(g):
    nb = int(g["num_blocks"])
    kc, vc = np.zeros((nb, BS, 2, D), np.int8), np.zeros((nb, BS, 2, D), np.int8)
    ks, vs = np.zeros((nb, BS, 2), np.float32), np.zeros((nb, BS, 2), np.float32)
    KV.int8_write(g["key"].astype(np.float32), g["value"].astype(np.float32), g["slots"], kc, vc, ks, vs)
    assert (kc == g["int8_key_cache"]).all() and (vc == g["int8_value_cache"]).all()
    assert (ks.view(np.uint32) == g["int8_k_scale"].view(np.uint32)).all()
    assert (vs.view(np.uint32) == g["int8_v_scale"].view(np.uint32)).all()


@pytest.mark.parametrize("name,qkey,qsl", QUERIES)
def test_int8_attention_matches_vllm(g, name, qkey, qsl):
    ref = KV.int8_attention(g[qkey], g["int8_key_cache"], g["int8_value_cache"], g["int8_k_scale"],
                            g["int8_v_scale"], g["block_table"], g["seq_lens"], qsl, D ** -0.5)
    check_attention(ref, g[f"int8_out_{name}"].astype(np.float64))


def int4_oracle_write(g, layer):
    nb = int(g["num_blocks"])
    sl, pos, rs, after = metadata(g)
    kc, vc = np.zeros((nb, BS, 2, D // 2), np.uint8), np.zeros((nb, BS, 2, D // 2), np.uint8)
    ks, vs = np.zeros((nb, BS, 2), np.float32), np.zeros((nb, BS, 2), np.float32)
    rows = KV.SINKS + KV.TAIL
    exk, exv = np.zeros((len(sl), rows, 2, D), np.float16), np.zeros((len(sl), rows, 2, D), np.float16)
    tag = np.full((len(sl), rows), -1, np.int32)
    p = f"int4_{layer}_"
    KV.int4_write(g["key"], g["value"], g["slots"], pos, rs, kc, vc, ks, vs, exk, exv, tag, after, g["signs"],
                  g.get(p + "bias_k"), g.get(p + "bias_v"))
    return kc, vc, ks, vs, exk, exv, tag


def exact_rows_match(g, layer, exk, exv, tag):
    """Our per-request-slot exact rows against the reference's (sinks per physical block, tail ring
    per request slot): the sequence's first SINKS positions and its newest TAIL ones."""
    p = f"int4_{layer}_"
    assert int(g["int4_sinks"]) == KV.SINKS and int(g["int4_tail"]) == KV.TAIL
    for s, L in enumerate(g["seq_lens"]):
        blk0 = g["block_table"][s, 0]
        n0 = min(KV.SINKS, L)
        assert (exk[s, :n0] == g[p + "sink_k"][blk0, :n0]).all() and (exv[s, :n0] == g[p + "sink_v"][blk0, :n0]).all()
        assert (tag[s, :n0] == np.arange(n0)).all()
        for P in range(max(0, L - KV.TAIL), L):
            r = KV.exact_index(P)
            if P < KV.SINKS:
                continue
            assert tag[s, r] == P == g[p + "ring_tag"][s, P % KV.TAIL]
            assert (exk[s, r] == g[p + "ring_k"][s, P % KV.TAIL]).all()
            assert (exv[s, r] == g[p + "ring_v"][s, P % KV.TAIL]).all()


@pytest.mark.parametrize("layer", ["plain", "centered"])
def test_int4_write_matches_reference(g, layer):
    kc, vc, ks, vs, exk, exv, tag = int4_oracle_write(g, layer)
    p = f"int4_{layer}_"
    assert (kc == g[p + "key_cache"]).all() and (vc == g[p + "value_cache"]).all()
    scale_words_match(ks, g[p + "k_scale_bits"])
    scale_words_match(vs, g[p + "v_scale_bits"])
    exact_rows_match(g, layer, exk, exv, tag)


@pytest.mark.parametrize("layer", ["plain", "centered"])
@pytest.mark.parametrize("name,qkey,qsl", QUERIES)
def test_int4_attention_matches_reference(g, layer, name, qkey, qsl):
    p = f"int4_{layer}_"
    kc, vc, ks, vs, exk, exv, tag = int4_oracle_write(g, layer)
    vm = g["mean_v"] if layer == "centered" else None
    # attention over the reference's own cache bytes (our scale words differ in a last place at most)
    ref_ks, ref_vs = g[p + "k_scale_bits"].view(np.float32), g[p + "v_scale_bits"].view(np.float32)
    got = KV.int4_attention(g[qkey], g[p + "key_cache"], g[p + "value_cache"], ref_ks, ref_vs, exk, exv, tag,
                            [0, 1], g["block_table"], g["seq_lens"], qsl, D ** -0.5, g["signs"], vm)
    check_attention(got, g[p + f"out_{name}"].astype(np.float64))


def test_centering_changes_the_cache(g):
    """The centred layer really is centred: its bytes differ from the plain layer's."""
    assert (g["int4_plain_key_cache"] != g["int4_centered_key_cache"]).mean() > 0.5
