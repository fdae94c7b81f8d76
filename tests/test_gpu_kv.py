"""GPU parity of the int8 / int4 paged KV cache against the CPU oracle (oracle/kv_oracle.py).

Writes: codes and scales bit-exact.  Attention: within NRMS <= 2e-3 and cosine >= 0.9999 of a
float64 softmax over the same quantised cache (the tolerance the build plan fixes for attention).
Synthetic K/V follow BASELINE config 3: N(0,1) with 1% of channels scaled x8; GQA 40 / 8, head 128,
block size 16, random block tables.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kv_oracle as KV

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
HQ, HKV, D, BS = 40, 8, 128, 16
ATOL = {"nrms": 2e-3, "cos": 0.9999}


@pytest.fixture(scope="module")
def kv():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from exl3rocm import kv as _kv
    return _kv


def outlier_rows(rng, n, heads, channels_seed=7):
    x = rng.standard_normal((n, heads, D)).astype(np.float32)
    ch = np.random.default_rng(channels_seed).choice(D, size=max(1, D // 100), replace=False)
    x[..., ch] *= 8.0
    return x.astype(np.float16)


def nrms_cos(got, ref):
    got, ref = got.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    nrms = np.sqrt(np.mean((got - ref) ** 2)) / (np.sqrt(np.mean(ref ** 2)) or 1.0)
    cos = got @ ref / ((np.linalg.norm(got) * np.linalg.norm(ref)) or 1.0)
    return nrms, cos


def make_layout(rng, seq_lens, extra=0):
    """Random block tables covering seq_len + extra tokens per sequence."""
    nblk = [-(-(L + extra) // BS) for L in seq_lens]
    total = sum(nblk) + 3
    perm = rng.permutation(total)
    bt = np.zeros((len(seq_lens), max(nblk)), dtype=np.int32)
    o = 0
    for s, nb in enumerate(nblk):
        bt[s, :nb] = perm[o:o + nb]
        o += nb
    return bt, total


def slots_for(bt, positions_per_seq):
    out = []
    for s, poss in enumerate(positions_per_seq):
        for p in poss:
            out.append(int(bt[s, p // BS]) * BS + p % BS)
    return np.array(out, dtype=np.int64)


# ---------------------------------------------------------------------------------------------
# int8
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_int8_write_bitexact(kv, dtype):
    rng = np.random.default_rng(11)
    seq_lens = [37, 5, 200]
    bt, nblocks = make_layout(rng, seq_lens)
    slot = slots_for(bt, [range(L) for L in seq_lens])
    slot[3] = -1  # a padded token is skipped
    T = len(slot)
    k = outlier_rows(rng, T, HKV)
    v = outlier_rows(rng, T, HKV, channels_seed=8)
    kt = torch.from_numpy(k).to(DEV).to(dtype)
    vt = torch.from_numpy(v).to(DEV).to(dtype)
    kc = torch.zeros((nblocks, BS, HKV, D), dtype=torch.int8, device=DEV)
    vc = torch.zeros_like(kc)
    ks = torch.zeros((nblocks, BS, HKV), dtype=torch.float32, device=DEV)
    vs = torch.zeros_like(ks)
    kv.reshape_and_cache_int8(kt, vt, kc, vc, torch.from_numpy(slot).to(DEV), ks, vs)
    ko, vo = np.zeros((nblocks, BS, HKV, D), np.int8), np.zeros((nblocks, BS, HKV, D), np.int8)
    kso, vso = np.zeros((nblocks, BS, HKV), np.float32), np.zeros((nblocks, BS, HKV), np.float32)
    KV.int8_write(kt.float().cpu().numpy(), vt.float().cpu().numpy(), slot, ko, vo, kso, vso)
    np.testing.assert_array_equal(kc.cpu().numpy(), ko)
    np.testing.assert_array_equal(vc.cpu().numpy(), vo)
    np.testing.assert_array_equal(ks.cpu().numpy(), kso)
    np.testing.assert_array_equal(vs.cpu().numpy(), vso)


def _int8_setup(rng, seq_lens, q_lens):
    bt, nblocks = make_layout(rng, seq_lens)
    slot = slots_for(bt, [range(L) for L in seq_lens])
    k = outlier_rows(rng, len(slot), HKV)
    v = outlier_rows(rng, len(slot), HKV, channels_seed=8)
    kc = np.zeros((nblocks, BS, HKV, D), np.int8)
    vc = np.zeros_like(kc)
    ks = np.zeros((nblocks, BS, HKV), np.float32)
    vs = np.zeros_like(ks)
    KV.int8_write(k, v, slot, kc, vc, ks, vs)
    qsl = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    q = (rng.standard_normal((int(qsl[-1]), HQ, D))).astype(np.float16)
    return bt, kc, vc, ks, vs, qsl, q


@pytest.mark.parametrize("seq_lens,q_lens", [
    ([1], [1]), ([33], [1]), ([1000], [1]), ([5, 300, 64, 4096], [1, 1, 1, 1]),
    ([40, 700], [4, 4]), ([17], [3]), ([2500], [2]),
    # a batch-8 decode at long context: ~27 splits of ~600 keys per (sequence, KV head), so one
    # split's accumulator runs over hundreds of tokens
    ([16384] * 8, [1] * 8),
])
def test_int8_attention(kv, seq_lens, q_lens):
    rng = np.random.default_rng(sum(seq_lens) + 7 * sum(q_lens))
    bt, kc, vc, ks, vs, qsl, q = _int8_setup(rng, seq_lens, q_lens)
    scale = D ** -0.5
    ref = KV.int8_attention(q, kc, vc, ks, vs, bt, seq_lens, qsl, scale)
    out = torch.empty((q.shape[0], HQ, D), dtype=torch.float16, device=DEV)
    kv.attention_int8(q=torch.from_numpy(q).to(DEV), k=torch.from_numpy(kc).to(DEV), v=torch.from_numpy(vc).to(DEV),
                      out=out, cu_seqlens_q=torch.from_numpy(qsl).to(DEV), max_seqlen_q=max(q_lens),
                      seqused_k=torch.tensor(seq_lens, dtype=torch.int32, device=DEV),
                      block_table=torch.from_numpy(bt).to(DEV), softmax_scale=scale,
                      k_scale_cache=torch.from_numpy(ks).to(DEV), v_scale_cache=torch.from_numpy(vs).to(DEV),
                      max_seqlen_k=max(seq_lens))
    nrms, cos = nrms_cos(out.cpu().numpy(), ref)
    assert nrms <= ATOL["nrms"] and cos >= ATOL["cos"], (nrms, cos)


def test_int8_attention_is_deterministic(kv):
    rng = np.random.default_rng(3)
    seq_lens, q_lens = [900, 33], [1, 1]
    bt, kc, vc, ks, vs, qsl, q = _int8_setup(rng, seq_lens, q_lens)
    args = dict(q=torch.from_numpy(q).to(DEV), k=torch.from_numpy(kc).to(DEV), v=torch.from_numpy(vc).to(DEV),
                cu_seqlens_q=torch.from_numpy(qsl).to(DEV), max_seqlen_q=1,
                seqused_k=torch.tensor(seq_lens, dtype=torch.int32, device=DEV),
                block_table=torch.from_numpy(bt).to(DEV), softmax_scale=D ** -0.5,
                k_scale_cache=torch.from_numpy(ks).to(DEV), v_scale_cache=torch.from_numpy(vs).to(DEV),
                max_seqlen_k=900)
    outs = []
    for _ in range(2):
        o = torch.empty((2, HQ, D), dtype=torch.float16, device=DEV)
        kv.attention_int8(out=o, **args)
        outs.append(o.clone())
    assert torch.equal(outs[0], outs[1])


# ---------------------------------------------------------------------------------------------
# int4
# ---------------------------------------------------------------------------------------------
def test_int4_quantizer_bitexact(kv):
    """Rotation + clip search + packing of the write kernel equal the oracle bit for bit."""
    rng = np.random.default_rng(21)
    seq_lens = [70]
    bt, nblocks = make_layout(rng, seq_lens)
    slot = slots_for(bt, [range(70)])
    k = outlier_rows(rng, 70, HKV)
    v = outlier_rows(rng, 70, HKV, channels_seed=8)
    kc = torch.zeros((nblocks, BS, HKV, D // 2), dtype=torch.uint8, device=DEV)
    vc = torch.zeros_like(kc)
    ks = torch.zeros((nblocks, BS, HKV), dtype=torch.float32, device=DEV)
    vs = torch.zeros_like(ks)
    kv.reshape_and_cache(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), kc, vc,
                         torch.from_numpy(slot).to(DEV), k_scale_cache=ks, v_scale_cache=vs)
    signs = KV.rht_signs(D)
    for x, cache, sc in ((k, kc, ks), (v, vc, vs)):
        y = KV.fwht128_f32(x.astype(np.float32) * signs)
        codes, sbits = KV.int4_quantize_rows(y)
        got_c, got_s = cache.cpu().numpy(), sc.cpu().numpy().view(np.uint32)
        for t, sl in enumerate(slot):
            b, o = divmod(int(sl), BS)
            np.testing.assert_array_equal(got_c[b, o], KV.pack_nibbles(codes[t]))
            np.testing.assert_array_equal(got_s[b, o], sbits[t])


def _int4_world(kv, rng, seq_lens, q_lens, slots_of_seq):
    """Prefill every sequence's context through the write kernel (exact rows on), then return the
    device caches and the oracle's mirror of them."""
    kv.configure_request_slots(4)
    kv._req["slot"] = None
    kv._exact.clear()
    bt, nblocks = make_layout(rng, seq_lens)
    T = sum(seq_lens)
    k = outlier_rows(rng, T, HKV)
    v = outlier_rows(rng, T, HKV, channels_seed=8)
    slot = slots_for(bt, [range(L) for L in seq_lens])
    kc = torch.zeros((nblocks, BS, HKV, D // 2), dtype=torch.uint8, device=DEV)
    vc = torch.zeros_like(kc)
    ks = torch.zeros((nblocks, BS, HKV), dtype=torch.float32, device=DEV)
    vs = torch.zeros_like(ks)
    kv.set_batch_slots(torch.tensor(slots_of_seq, dtype=torch.int32, device=DEV))
    qsl_w = np.concatenate([[0], np.cumsum(seq_lens)]).astype(np.int32)
    kv.reshape_and_cache(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), kc, vc,
                         torch.from_numpy(slot).to(DEV), k_scale_cache=ks, v_scale_cache=vs, layer_name="L0",
                         query_start_loc=torch.from_numpy(qsl_w).to(DEV),
                         seq_lens=torch.tensor(seq_lens, dtype=torch.int32, device=DEV))
    # oracle mirror
    rows = 5
    ko = np.zeros((nblocks, BS, HKV, D // 2), np.uint8); vo = np.zeros_like(ko)
    kso = np.zeros((nblocks, BS, HKV), np.float32); vso = np.zeros_like(kso)
    exk = np.zeros((rows, KV.SINKS + KV.TAIL, HKV, D), np.float16); exv = np.zeros_like(exk)
    tag = np.full((rows, KV.SINKS + KV.TAIL), -1, np.int32)
    positions = np.concatenate([np.arange(L) for L in seq_lens])
    req = np.concatenate([[slots_of_seq[s]] * L for s, L in enumerate(seq_lens)])
    after = np.concatenate([[L] * L for L in seq_lens])
    KV.int4_write(k, v, slot, positions, req, ko, vo, kso, vso, exk, exv, tag, after, KV.rht_signs(D))
    _int4_world.raw = (k, v)
    return bt, (kc, vc, ks, vs), (ko, vo, kso, vso, exk, exv, tag)


def test_int4_write_with_exact_rows_bitexact(kv):
    rng = np.random.default_rng(5)
    seq_lens, slots = [300, 9], [2, 0]
    bt, dev, ora = _int4_world(kv, rng, seq_lens, [1, 1], slots)
    kc, vc, ks, vs = dev
    ko, vo, kso, vso, exk, exv, tag = ora
    np.testing.assert_array_equal(kc.cpu().numpy(), ko)
    np.testing.assert_array_equal(vc.cpu().numpy(), vo)
    np.testing.assert_array_equal(ks.cpu().numpy().view(np.uint32), kso.view(np.uint32))
    np.testing.assert_array_equal(vs.cpu().numpy().view(np.uint32), vso.view(np.uint32))
    ex = kv._exact["L0"]
    np.testing.assert_array_equal(ex["tag"].cpu().numpy(), tag)
    for s in slots:
        np.testing.assert_array_equal(ex["k"][s].cpu().numpy(), exk[s])
        np.testing.assert_array_equal(ex["v"][s].cpu().numpy(), exv[s])


@pytest.mark.parametrize("seq_lens,q_lens", [([3], [1]), ([300], [1]), ([40, 1200, 130], [1, 1, 1]),
                                             ([700, 20], [4, 4]), ([3000], [1])])
def test_int4_attention_with_exact_rows(kv, seq_lens, q_lens):
    rng = np.random.default_rng(sum(seq_lens) + 3)
    _check_int4_attention(kv, rng, seq_lens, q_lens, [3, 1, 0][: len(seq_lens)])


def test_int4_attention_long_splits(kv):
    """Eight sequences of 8192 without exact rows: every tile on the packed path, ~27 splits of ~300
    keys per (sequence, KV head)."""
    rng = np.random.default_rng(8192)
    _check_int4_attention(kv, rng, [8192] * 8, [1] * 8, [-1] * 8)


def _check_int4_attention(kv, rng, seq_lens, q_lens, slots):
    bt, dev, ora = _int4_world(kv, rng, seq_lens, q_lens, slots)
    kc, vc, ks, vs = dev
    ko, vo, kso, vso, exk, exv, tag = ora
    qsl = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    q = rng.standard_normal((int(qsl[-1]), HQ, D)).astype(np.float16)
    scale = D ** -0.5
    ref = KV.int4_attention(q, ko, vo, kso, vso, exk, exv, tag, slots, bt, seq_lens, qsl, scale, KV.rht_signs(D))
    out = torch.empty((q.shape[0], HQ, D), dtype=torch.float16, device=DEV)
    kv.attention(q=torch.from_numpy(q).to(DEV), k=kc, v=vc, out=out, cu_seqlens_q=torch.from_numpy(qsl).to(DEV),
                 max_seqlen_q=max(q_lens), seqused_k=torch.tensor(seq_lens, dtype=torch.int32, device=DEV),
                 block_table=torch.from_numpy(bt).to(DEV), softmax_scale=scale, k_scale_cache=ks,
                 v_scale_cache=vs, max_seqlen_k=max(seq_lens), layer_name="L0")
    nrms, cos = nrms_cos(out.cpu().numpy(), ref)
    assert nrms <= ATOL["nrms"] and cos >= ATOL["cos"], (nrms, cos)


def test_int4_close_to_fp16_cache(kv):
    """Sanity bound: the int4 cache (with exact rows) stays near attention over the unquantised fp16
    K/V.  Random Gaussian keys give an almost flat softmax, so the output keeps the ~10 % relative
    error of 4-bit rows; model-level accuracy is what the reference's KL gates measure."""
    rng = np.random.default_rng(77)
    seq_lens = [800]
    bt, dev, ora = _int4_world(kv, rng, seq_lens, [1], [1])
    kc, vc, ks, vs = dev
    q = rng.standard_normal((1, HQ, D)).astype(np.float16)
    out = torch.empty((1, HQ, D), dtype=torch.float16, device=DEV)
    kv.attention(q=torch.from_numpy(q).to(DEV), k=kc, v=vc, out=out,
                 cu_seqlens_q=torch.tensor([0, 1], dtype=torch.int32, device=DEV), max_seqlen_q=1,
                 seqused_k=torch.tensor(seq_lens, dtype=torch.int32, device=DEV),
                 block_table=torch.from_numpy(bt).to(DEV), softmax_scale=D ** -0.5, k_scale_cache=ks,
                 v_scale_cache=vs, max_seqlen_k=800, layer_name="L0")
    k, v = _int4_world.raw
    ref = KV.paged_attention(q, seq_lens, np.array([0, 1], np.int32), bt, D ** -0.5,
                             lambda s_, n: k[:n].astype(np.float64), lambda s_, n: v[:n].astype(np.float64))
    nrms, cos = nrms_cos(out.cpu().numpy(), ref)
    assert cos > 0.98 and nrms < 0.2, (nrms, cos)


# ---------------------------------------------------------------------------------------------
# prefill over the quantised caches: gather + dequantise to fp16, fp16 attention (SDPA here)
# ---------------------------------------------------------------------------------------------
# The fp16 buffer and the fp16 attention kernel (P rounded to fp16 before P.V) add their own
# roundings to the decode path's: the gate is wider than ATOL.
PREFILL_ATOL = {"nrms": 4e-3, "cos": 0.9999}


def _prefill_kw(q, kc, vc, ks, vs, bt, seq_lens, q_lens, qsl):
    return dict(q=torch.from_numpy(q).to(DEV), k=kc, v=vc,
                out=torch.empty((q.shape[0], HQ, D), dtype=torch.float16, device=DEV),
                cu_seqlens_q=torch.from_numpy(qsl).to(DEV), max_seqlen_q=max(q_lens),
                seqused_k=torch.tensor(seq_lens, dtype=torch.int32, device=DEV),
                block_table=torch.from_numpy(bt).to(DEV), softmax_scale=D ** -0.5, k_scale_cache=ks,
                v_scale_cache=vs, max_seqlen_k=max(seq_lens))


def test_int8_gather_matches_oracle_dequant(kv):
    rng = np.random.default_rng(44)
    bt, kc, vc, ks, vs, qsl, q = _int8_setup(rng, [100, 37], [1, 1])
    blocks = torch.from_numpy(bt.reshape(-1).copy()).to(DEV)
    got = kv.gather_dequant_int8(torch.from_numpy(kc).to(DEV), torch.from_numpy(ks).to(DEV), blocks).cpu().numpy()
    ref = (kc[bt.reshape(-1)].astype(np.float32) * ks[bt.reshape(-1)][..., None]).astype(np.float16)
    np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("seq_lens,q_lens", [([600], [64]), ([40, 300], [40, 17]), ([2000, 64], [33, 64])])
def test_int8_prefill(kv, seq_lens, q_lens):
    rng = np.random.default_rng(sum(seq_lens) + 5 * sum(q_lens))
    bt, kc, vc, ks, vs, qsl, q = _int8_setup(rng, seq_lens, q_lens)
    ref = KV.int8_attention(q, kc, vc, ks, vs, bt, seq_lens, qsl, D ** -0.5)
    kw = _prefill_kw(q, torch.from_numpy(kc).to(DEV), torch.from_numpy(vc).to(DEV), torch.from_numpy(ks).to(DEV),
                     torch.from_numpy(vs).to(DEV), bt, seq_lens, q_lens, qsl)
    kv.prefill_int8(None, kw)
    nrms, cos = nrms_cos(kw["out"].cpu().numpy(), ref)
    assert nrms <= PREFILL_ATOL["nrms"] and cos >= PREFILL_ATOL["cos"], (nrms, cos)


@pytest.mark.parametrize("seq_lens,q_lens", [([700, 150], [64, 30]), ([200], [200])])
def test_int4_prefill_with_exact_rows(kv, seq_lens, q_lens):
    rng = np.random.default_rng(sum(seq_lens) + 9)
    slots = [2, 0][: len(seq_lens)]
    bt, dev, ora = _int4_world(kv, rng, seq_lens, q_lens, slots)
    kc, vc, ks, vs = dev
    ko, vo, kso, vso, exk, exv, tag = ora
    qsl = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    q = rng.standard_normal((int(qsl[-1]), HQ, D)).astype(np.float16)
    ref = KV.int4_attention(q, ko, vo, kso, vso, exk, exv, tag, slots, bt, seq_lens, qsl, D ** -0.5,
                            KV.rht_signs(D))
    kw = _prefill_kw(q, kc, vc, ks, vs, bt, seq_lens, q_lens, qsl)
    kv.prefill(None, kw, layer_name="L0")
    nrms, cos = nrms_cos(kw["out"].cpu().numpy(), ref)
    assert nrms <= PREFILL_ATOL["nrms"] and cos >= PREFILL_ATOL["cos"], (nrms, cos)
