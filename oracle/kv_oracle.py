"""CPU oracle for the int8 / int4 paged KV cache: TEST INFRASTRUCTURE, never the product path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU leg may import this module.

int8 per-token-head (vLLM's ``int8_per_token_head`` cache, which the reference runs unmodified):
  write     vllm/v1/attention/ops/triton_reshape_and_cache_flash.py:139-238 (scale = max(absmax/127,
            1e-6); q = clamp(x * (1/scale), -128, 127) stored by truncation toward zero)
  attention vllm/v1/attention/ops/triton_unified_attention.py:473-545 (S = q.K * scale * k_scale[t];
            acc += (P * v_scale[t]) . V; online softmax; split segments reduced by reduce_segments)
int4 per-token-head (reference vllm_plugin/exl3rocm/kv_int4.py):
  write     :176-213, :247-342 (y = x @ diag(s) H unnormalised; 3x3 clip search on [lo, hi] shrunk
            toward the row mean by 0 / 7.5 / 15 %; asymmetric 4 bit, round half away from zero;
            element 2i in the low nibble; scale bits = (fp32 scale & ~0xF) | zp; exact fp16 rows
            for the sequence's first SINKS positions and its newest TAIL positions)
  attention :345-563 (rotated q; S = q.(nibble - zp) * (softmax_scale / d) * k_scale; exact rows
            with scale 1; P * v_scale . (nibble - zp); output un-rotated by (H diag(s)) / d)

Parity status: pinned.  tests/golden/make_kv_golden.py runs the reference's own Triton kernels
(vLLM 0.22's int8 per-token-head write and unified attention; the reference's kv_int4.py write and
attention, with and without centering) under Triton's CPU interpreter and commits their outputs;
tests/test_kv_golden.py checks this module against them: int8 codes and scales bit-exact, int4 codes
and exact rows bit-exact, int4 scales bit-exact except a last-place difference where the row mean
is summed in another order, attention within the tolerance of a float64 softmax.  One input is not
the reference's: the int4 RHT sign vector comes from a vLLM 0.28 helper absent here, so the
fixtures use this repository's seeded vector (the format is parameterised by it).
"""
from __future__ import annotations

import numpy as np

CLIP_STEPS = 3
CLIP_STEP = np.float32(0.075)
SINKS = 4
TAIL = 128
RHT_SEED = 0x5EED1234


# ---------------------------------------------------------------------------------------------
# int8 per-token-head
# ---------------------------------------------------------------------------------------------
def int8_quantize_rows(x: np.ndarray):
    """x [..., D] (fp16 values) -> (codes int8 [..., D], scale fp32 [...]), float32 arithmetic."""
    xf = np.asarray(x, dtype=np.float32)
    amax = np.abs(xf).max(axis=-1)
    scale = np.maximum(amax / np.float32(127.0), np.float32(1e-6)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    q = np.clip(xf * inv[..., None], np.float32(-128.0), np.float32(127.0))
    return np.trunc(q).astype(np.int8), scale


def int8_write(key, value, slot_mapping, key_cache, value_cache, k_scale, v_scale):
    """Scatter quantised rows into [blocks, block_size, H, D] caches (slots < 0 are skipped)."""
    bs = key_cache.shape[1]
    kq, ks = int8_quantize_rows(key)
    vq, vs = int8_quantize_rows(value)
    for t, slot in enumerate(np.asarray(slot_mapping)):
        if slot < 0:
            continue
        b, o = divmod(int(slot), bs)
        key_cache[b, o], value_cache[b, o] = kq[t], vq[t]
        k_scale[b, o], v_scale[b, o] = ks[t], vs[t]


def _gather(cache, block_table_row, n):
    bs = cache.shape[1]
    idx = np.arange(n)
    return cache[np.asarray(block_table_row)[idx // bs], idx % bs]


def paged_attention(q, seq_lens, query_start_loc, block_table, softmax_scale, keys_of, values_of):
    """Causal attention for each sequence's query tokens over its cached rows, float64.

    q [T, Hq, D]; keys_of(seq, n) / values_of(seq, n) -> float64 [n, Hkv, D] dequantised rows.
    Query token i of a sequence with q_len queries sits at position seq_len - q_len + i.
    """
    q = np.asarray(q, dtype=np.float64)
    T, Hq, D = q.shape
    out = np.zeros((T, Hq, D), dtype=np.float64)
    for s in range(len(seq_lens)):
        q0, q1 = int(query_start_loc[s]), int(query_start_loc[s + 1])
        L = int(seq_lens[s])
        if q1 <= q0 or L <= 0:
            continue
        Kd, Vd = keys_of(s, L), values_of(s, L)
        Hkv = Kd.shape[1]
        G = Hq // Hkv
        for i, t in enumerate(range(q0, q1)):
            pos = L - (q1 - q0) + i
            for h in range(Hq):
                kh = h // G
                sc = Kd[: pos + 1, kh] @ q[t, h] * softmax_scale
                p = np.exp(sc - sc.max())
                out[t, h] = (p[:, None] * Vd[: pos + 1, kh]).sum(0) / p.sum()
    return out


def int8_attention(q, key_cache, value_cache, k_scale, v_scale, block_table, seq_lens, query_start_loc,
                   softmax_scale):
    def deq(cache, scale):
        return lambda s, n: (_gather(cache, block_table[s], n).astype(np.float64)
                             * _gather(scale, block_table[s], n).astype(np.float64)[..., None])
    return paged_attention(q, seq_lens, query_start_loc, block_table, softmax_scale,
                           deq(key_cache, k_scale), deq(value_cache, v_scale))


# ---------------------------------------------------------------------------------------------
# int4 per-token-head with RHT, clip search and exact rows
# ---------------------------------------------------------------------------------------------
def sylvester(d: int) -> np.ndarray:
    i = np.arange(d)
    pc = np.vectorize(lambda v: bin(int(v)).count("1"))(i[:, None] & i[None, :])
    return np.where(pc % 2 == 1, -1.0, 1.0).astype(np.float32)


def rht_signs(d: int, seed: int = RHT_SEED) -> np.ndarray:
    """The +-1 sign vector of the randomised Hadamard transform (seeded; shared by write and read)."""
    return np.where(np.random.default_rng(seed).integers(0, 2, size=d) == 1, 1.0, -1.0).astype(np.float32)


def rht_forward(x: np.ndarray, signs: np.ndarray) -> np.ndarray:
    """y = x @ (diag(s) H), unnormalised, float32 (kv_int4.py:161-173, fwd)."""
    d = x.shape[-1]
    return (np.asarray(x, dtype=np.float64) * signs) @ sylvester(d).astype(np.float64)


def rht_inverse_d(y: np.ndarray, signs: np.ndarray) -> np.ndarray:
    """x = y @ (H diag(s)) / d (kv_int4.py:171, inv_d)."""
    d = y.shape[-1]
    return (np.asarray(y, dtype=np.float64) @ sylvester(d).astype(np.float64)) * signs / d


def fwht128_f32(x: np.ndarray) -> np.ndarray:
    """Unnormalised natural-order Hadamard of 128-element rows in float32, in the kernel's order:
    element e = 4 * lane + slot; H4 inside each lane, then xor butterflies over lanes 1, 2, 4, 8, 16
    (upper lane: partner - own, lower lane: own + partner)."""
    f = np.float32
    v = np.asarray(x, dtype=np.float32).reshape(*x.shape[:-1], 32, 4)
    s0, d0 = (v[..., 0] + v[..., 1]).astype(f), (v[..., 0] - v[..., 1]).astype(f)
    s1, d1 = (v[..., 2] + v[..., 3]).astype(f), (v[..., 2] - v[..., 3]).astype(f)
    v = np.stack([(s0 + s1).astype(f), (d0 + d1).astype(f), (s0 - s1).astype(f), (d0 - d1).astype(f)], axis=-1)
    lane = np.arange(32)
    for dist in (1, 2, 4, 8, 16):
        o = v[..., lane ^ dist, :]
        upper = ((lane & dist) != 0)[:, None]
        v = np.where(upper, (o - v).astype(f), (v + o).astype(f)).astype(f)
    return v.reshape(x.shape)


def _lane_sum(y: np.ndarray) -> np.ndarray:
    """Sum of 128 values in the kernel's order: per lane ((y0 + y1) + y2) + y3 over its 4 consecutive
    elements, then a xor butterfly over 32 lanes (distances 16, 8, 4, 2, 1)."""
    f = np.float32
    v = y.astype(np.float32).reshape(*y.shape[:-1], 32, 4)
    s = ((v[..., 0] + v[..., 1]).astype(f) + v[..., 2]).astype(f) + v[..., 3]
    s = s.astype(f)
    for d in (16, 8, 4, 2, 1):
        s = (s + s[..., np.arange(32) ^ d]).astype(f)
    return s[..., 0]


def _fma(a, b, c) -> np.ndarray:
    """float32 fused multiply-add (one rounding), via an exact float64 product."""
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(np.float32)


def _lane_sumsq(e: np.ndarray) -> np.ndarray:
    """Sum of squares in the kernel's order: per lane fma(e3,e3,fma(e2,e2,fma(e1,e1,e0*e0))), then
    the xor butterfly."""
    f = np.float32
    v = e.astype(np.float32).reshape(*e.shape[:-1], 32, 4)
    s = (v[..., 0] * v[..., 0]).astype(f)
    for i in (1, 2, 3):
        s = _fma(v[..., i], v[..., i], s)
    for d in (16, 8, 4, 2, 1):
        s = (s + s[..., np.arange(32) ^ d]).astype(f)
    return s[..., 0]


def _round_half_away(v: np.ndarray) -> np.ndarray:
    """trunc(v + 0.5) for v >= 0 else trunc(v - 0.5) (kv_int4.py:299)."""
    f = np.float32
    return np.trunc(np.where(v >= 0, (v + f(0.5)).astype(f), (v - f(0.5)).astype(f))).astype(np.int32)


def int4_quantize_rows(y: np.ndarray):
    """y [..., 128] float32 rotated rows -> (codes [..., 128] uint8 0..15, scale bits uint32 [...]).

    Clip search of kv_int4.py:290-308 in float32: products feeding an add are single-rounding fused
    multiply-adds (as the reference's compiler contracts them), divisions are IEEE, sums follow the
    kernel's lane order."""
    f = np.float32
    y = np.asarray(y, dtype=np.float32)
    lo0 = y.min(axis=-1)
    hi0 = y.max(axis=-1)
    mu = (_lane_sum(y) * f(1.0 / 128.0)).astype(f)
    best_err = np.full(lo0.shape, np.inf, dtype=np.float32)
    best_sc = np.zeros(lo0.shape, dtype=np.float32)
    best_zp = np.zeros(lo0.shape, dtype=np.int32)
    for c in range(CLIP_STEPS * CLIP_STEPS):
        flo = _fma(-CLIP_STEP, f(c // CLIP_STEPS), f(1.0))
        fhi = _fma(-CLIP_STEP, f(c % CLIP_STEPS), f(1.0))
        lo = _fma((lo0 - mu).astype(f), flo, mu)
        hi = _fma((hi0 - mu).astype(f), fhi, mu)
        sc = np.maximum(((hi - lo).astype(f) / f(15.0)).astype(f), f(1e-6)).astype(f)
        zp = np.clip(_round_half_away((-lo / sc).astype(f)), 0, 15)
        inv = (f(1.0) / sc).astype(f)
        qn = np.clip(_round_half_away(_fma(y, inv[..., None], zp[..., None].astype(f))), 0, 15)
        e = _fma((qn - zp[..., None]).astype(f), sc[..., None], -y)
        err = _lane_sumsq(e)
        better = err < best_err  # strict: the first minimal candidate wins (argmin)
        best_err = np.where(better, err, best_err)
        best_sc = np.where(better, sc, best_sc)
        best_zp = np.where(better, zp, best_zp)
    inv = (f(1.0) / best_sc).astype(f)
    codes = np.clip(_round_half_away(_fma(y, inv[..., None], best_zp[..., None].astype(f))), 0, 15).astype(np.uint8)
    sbits = (best_sc.view(np.uint32) & np.uint32(0xFFFFFFF0)) | best_zp.astype(np.uint32)
    return codes, sbits.astype(np.uint32)


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    out = np.empty((*packed.shape[:-1], packed.shape[-1] * 2), dtype=np.uint8)
    out[..., 0::2] = packed & 0xF
    out[..., 1::2] = packed >> 4
    return out


def int4_dequant_rows(packed: np.ndarray, sbits: np.ndarray) -> np.ndarray:
    """Rotated-domain values (nibble - zp) * scale (float64)."""
    sbits = np.asarray(sbits, dtype=np.uint32)
    zp = (sbits & 0xF).astype(np.float64)
    sc = (sbits & np.uint32(0xFFFFFFF0)).view(np.float32).astype(np.float64)
    return (unpack_nibbles(packed).astype(np.float64) - zp[..., None]) * sc[..., None]


def exact_index(pos: int) -> int:
    """Row of the per-request exact buffer holding position pos (sinks first, then the tail ring)."""
    return pos if pos < SINKS else SINKS + pos % TAIL


def int4_write(key, value, slot_mapping, positions, req_slots, key_cache, value_cache, k_scale, v_scale,
               exact_k, exact_v, exact_tag, seq_lens_after, signs, bias_k=None, bias_v=None):
    """Rotate, quantise and pack K and V rows; keep exact fp16 rows for positions < SINKS and for the
    newest TAIL positions of each request (exact_* [slots, SINKS + TAIL, H, D], tag [slots, SINKS + TAIL]).

    positions[t], req_slots[t]: the token's position in its sequence and its request slot;
    seq_lens_after[t]: that sequence's length once this batch is written.
    bias_k / bias_v [H, D] float32 (optional): rotated-domain biases -(mean @ diag(s) H) added to the
    rotated rows before quantisation, the centering of kv_int4.py:133-148, 265-266."""
    bs = key_cache.shape[1]
    yk = fwht128_f32(np.asarray(key, np.float32) * signs)
    yv = fwht128_f32(np.asarray(value, np.float32) * signs)
    if bias_k is not None:
        yk = (yk + np.asarray(bias_k, np.float32)[None]).astype(np.float32)
    if bias_v is not None:
        yv = (yv + np.asarray(bias_v, np.float32)[None]).astype(np.float32)
    ck, sk = int4_quantize_rows(yk)
    cv, sv = int4_quantize_rows(yv)
    for t, slot in enumerate(np.asarray(slot_mapping)):
        if slot < 0:
            continue
        b, o = divmod(int(slot), bs)
        key_cache[b, o], value_cache[b, o] = pack_nibbles(ck[t]), pack_nibbles(cv[t])
        k_scale[b, o], v_scale[b, o] = sk[t].view(np.float32), sv[t].view(np.float32)
        pos, rs = int(positions[t]), int(req_slots[t])
        if rs >= 0 and (pos < SINKS or pos >= int(seq_lens_after[t]) - TAIL):
            e = exact_index(pos)
            exact_k[rs, e] = yk[t].astype(np.float16)
            exact_v[rs, e] = yv[t].astype(np.float16)
            exact_tag[rs, e] = pos


def int4_attention(q, key_cache, value_cache, k_scale, v_scale, exact_k, exact_v, exact_tag, req_slot_of_seq,
                   block_table, seq_lens, query_start_loc, softmax_scale, signs, v_mean=None):
    """Attention over the int4 cache with exact-row substitution, computed in the rotated domain and
    un-rotated (the RHT is orthogonal up to the factor d, so this equals attention over the
    dequantised, un-rotated rows).  v_mean [H_kv, D] (optional): the value mean of a centred cache,
    added back to the output of every query head of that KV head (kv_int4.py:470-480, 563)."""
    d = q.shape[-1]

    def rows(cache, scale, ex, s, n):
        r = int4_dequant_rows(_gather(cache, block_table[s], n), _gather(scale, block_table[s], n).view(np.uint32))
        rs = int(req_slot_of_seq[s])
        if rs >= 0:
            for pos in range(n):
                e = exact_index(pos) if (pos < SINKS or pos >= n - TAIL) else -1
                if e >= 0 and exact_tag[rs, e] == pos:
                    r[pos] = ex[rs, e].astype(np.float64)
        return r
    qr = rht_forward(q, signs)
    rot = paged_attention(qr, seq_lens, query_start_loc, block_table, softmax_scale / d,
                          lambda s, n: rows(key_cache, k_scale, exact_k, s, n),
                          lambda s, n: rows(value_cache, v_scale, exact_v, s, n))
    out = rht_inverse_d(rot, signs)
    if v_mean is not None:
        vm = np.asarray(v_mean, np.float64)
        out = out + np.repeat(vm, q.shape[1] // vm.shape[0], axis=0)[None]
    return out
