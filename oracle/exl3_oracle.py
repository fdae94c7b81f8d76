"""CPU oracle for the EXL3 linear: TEST INFRASTRUCTURE, never the product path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
module, and only as the checker / the timed CPU restatement.  The CUDA library never calls it.

This is an independent numpy restatement of the reference's CPU oracle
(``reference/exl3_oracle.py`` in Luke458/qwen38-27b-exl3-rdna4), vectorised over tiles so that
full layer shapes finish in seconds.  Each function names the reference lines it restates.  It is
pinned against golden vectors produced by the reference oracle itself
(``tests/golden/make_golden.py`` -> ``tests/golden/exl3_golden.npz``) and against the reference's
known-answer tests (``tests/test_oracle.py`` of the reference, restated in ``tests/test_oracle_port.py``).

Semantics (all integer work bit-exact, floats on the fp16 grid where the kernels store fp16):

* trellis tensor: uint16 ``(k/16, n/16, 16*K)``; one 16x16 tile (rows = input features k,
  cols = output features n) is a 256*K-bit ring read as little-endian uint32 words whose bits are
  numbered from the MSB of word 0.
* position t (0..255) of a tile has the 16-bit state that ends at bit (t+1)*K (mod 256*K).
* t = 8L + i sits at row 2(L%4) + (i&1) + 8((i>>1)&1), col 2(L>>3) + ((L>>2)&1) + 8(i>>2).
* codebooks: cb2 "mul1", cb1 "mcg", cb0 "3inst" (hash, then fp16 arithmetic with one rounding).
* H128 is the natural-order Sylvester Hadamard, scaled by 1/sqrt(128).
"""
from __future__ import annotations

import numpy as np

# fp16 bit patterns and hash constants (reference/exl3_oracle.py:40-47)
K_INV_BITS = 0x1EEE
K_BIAS_BITS = 0xC931
MUL1_MULT = 0x83DCD12D
MCG_MULT = 0xCBAC1FED
CB0_MULT = 89226354
CB0_ADD = 64248484
LOP3_AND = 0x8FFF8FFF
LOP3_XOR = 0x3B603B60
R_SCALE = 0.088388347648  # 1/sqrt(128) as every call site passes it (reference/exl3_oracle.py:47)

CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2


def fp16_bits_to_f64(bits) -> np.ndarray:
    """Exact value of binary16 bit patterns (reference/exl3_oracle.py:50-52, 96-98)."""
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float64)


K_INV = float(fp16_bits_to_f64(np.array([K_INV_BITS]))[0])
K_BIAS = float(fp16_bits_to_f64(np.array([K_BIAS_BITS]))[0])


def cb_of(mcg: bool, mul1: bool) -> int:
    """Codebook id from the op flags (reference ops pass (mcg, mul1); tests/test_gpu_parity.py:101)."""
    if mul1:
        return CB_MUL1
    if mcg:
        return CB_MCG
    return CB_3INST


# ---------------------------------------------------------------------------------------------
# codebooks (reference/exl3_oracle.py:67-123)
# ---------------------------------------------------------------------------------------------
def _bytesum(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.uint64)
    return ((x & 0xFF) + ((x >> 8) & 0xFF) + ((x >> 16) & 0xFF) + ((x >> 24) & 0xFF)).astype(np.int64)


def _decode_all_states(cb: int) -> np.ndarray:
    """fp16 value of every 16-bit state for codebook cb, as a uint16 bit-pattern table."""
    w = np.arange(65536, dtype=np.uint64)
    if cb == CB_MUL1:
        # value = fp16_fma(fp16(0x6400 + s), k_inv, k_bias), s = bytesum(w * M): the exact
        # float64 result rounded once (reference/exl3_oracle.py:81-93)
        s = _bytesum((w * MUL1_MULT) & 0xFFFFFFFF)
        v = (1024.0 + s.astype(np.float64)) * K_INV + K_BIAS
        return v.astype(np.float16).view(np.uint16)
    if cb == CB_MCG:
        x = (w * MCG_MULT) & 0xFFFFFFFF
    elif cb == CB_3INST:
        x = (w * CB0_MULT + CB0_ADD) & 0xFFFFFFFF
    else:
        raise ValueError(f"codebook must be 0, 1 or 2, got {cb}")
    # lop3 imm 0x6a == (x & 0x8fff8fff) ^ 0x3b603b60, then the fp16 add of both halves with one
    # rounding (reference/exl3_oracle.py:73-78, 110-119)
    x = (x & LOP3_AND) ^ LOP3_XOR
    lo = fp16_bits_to_f64((x & 0xFFFF).astype(np.uint16))
    hi = fp16_bits_to_f64((x >> 16).astype(np.uint16))
    return (lo + hi).astype(np.float16).view(np.uint16)


_TABLES: dict[int, np.ndarray] = {}


def codebook_table(cb: int) -> np.ndarray:
    """uint16 fp16 bit patterns, indexed by state (cached)."""
    if cb not in _TABLES:
        _TABLES[cb] = _decode_all_states(cb)
    return _TABLES[cb]


def decode_states(states: np.ndarray, cb: int) -> np.ndarray:
    """States (any shape, uint16) -> fp16 values (reference decode_codebook, :101-119)."""
    return codebook_table(cb)[np.asarray(states, dtype=np.uint16)].view(np.float16)


# ---------------------------------------------------------------------------------------------
# trellis windows and tile layout (reference/exl3_oracle.py:129-230)
# ---------------------------------------------------------------------------------------------
def t_to_rowcol():
    """(row, col) of every t in 0..255 (reference/exl3_oracle.py:129-146)."""
    t = np.arange(256, dtype=np.int64)
    L, i = t >> 3, t & 7
    row = 2 * (L % 4) + (i & 1) + 8 * ((i >> 1) & 1)
    col = 2 * (L >> 3) + ((L >> 2) & 1) + 8 * (i >> 2)
    return row, col


ROW, COL = t_to_rowcol()
# flat index (row*16 + col) of position t, and its inverse
T_FLAT = ROW * 16 + COL
FLAT_T = np.empty(256, dtype=np.int64)
FLAT_T[T_FLAT] = np.arange(256)


def _window_params(K: int):
    t = np.arange(256, dtype=np.int64)
    b1 = (t + 257) * K  # end bit (exclusive), shifted by one full ring so it stays positive
    b0 = b1 - 16
    n_words = 8 * K
    i0 = (b0 // 32) % n_words
    i1 = ((b1 - 1) // 32) % n_words
    s0 = ((b1 - 1) // 32 + 1) * 32 - b1
    return i0, i1, s0.astype(np.uint64)


def tile_states(trellis: np.ndarray, K: int) -> np.ndarray:
    """uint16 trellis [..., 16K] -> uint16 states [..., 256] in t order (reference :156-188)."""
    trellis = np.ascontiguousarray(trellis, dtype=np.uint16)
    assert trellis.shape[-1] == 16 * K, (trellis.shape, K)
    words = trellis.view(np.uint32).astype(np.uint64)
    i0, i1, s0 = _window_params(K)
    merged = (words[..., i0] << np.uint64(32)) | words[..., i1]
    return ((merged >> s0) & np.uint64(0xFFFF)).astype(np.uint16)


def states_to_matrix(states: np.ndarray) -> np.ndarray:
    """[kt, nt, 256] t-ordered values -> [kt*16, nt*16] matrix (reference :206-230)."""
    kt, nt, _ = states.shape
    tiles = states[:, :, FLAT_T].reshape(kt, nt, 16, 16)
    return tiles.transpose(0, 2, 1, 3).reshape(kt * 16, nt * 16)


def trellis_states(trellis: np.ndarray, K: int) -> np.ndarray:
    """State of every weight, laid out as (k, n) (reference trellis_states, :222-230)."""
    return states_to_matrix(tile_states(trellis, K))


def dequant(trellis: np.ndarray, K: int, cb: int, n0: int = 0, n1: int | None = None) -> np.ndarray:
    """Decoded fp16 weights W[k, n0:n1] (reference decode_trellis, :206-219; reconstruct_slice)."""
    kt, nt, _ = trellis.shape
    n1 = nt * 16 if n1 is None else n1
    assert n0 % 16 == 0 and n1 % 16 == 0
    tab = codebook_table(cb)
    out = np.empty((kt * 16, n1 - n0), dtype=np.uint16)
    step = max(1, (1 << 22) // max(1, (n1 - n0)))  # ~4M weights per chunk
    for k0 in range(0, kt, step):
        st = tile_states(trellis[k0:k0 + step, n0 // 16:n1 // 16], K)
        out[k0 * 16:(k0 + st.shape[0]) * 16] = states_to_matrix(tab[st])
    return out.view(np.float16)


# ---------------------------------------------------------------------------------------------
# 128-point Hadamard (reference/exl3_oracle.py:236-301)
# ---------------------------------------------------------------------------------------------
def had128_matrix() -> np.ndarray:
    """Unscaled H128[i, j] = (-1)^popcount(i & j): the kron(H32, H4) of reference :246-258."""
    i = np.arange(128)
    pc = np.vectorize(lambda v: bin(int(v)).count("1"))(i[:, None] & i[None, :])
    return np.where(pc % 2 == 1, -1.0, 1.0)


_H = had128_matrix()


def had128(x: np.ndarray, scale: float = R_SCALE) -> np.ndarray:
    """scale * H128 applied to each 128-block of the last axis, in float64 (reference :264-274)."""
    x = np.asarray(x, dtype=np.float64)
    assert x.shape[-1] % 128 == 0
    return (x.reshape(-1, 128) @ _H.T * scale).reshape(x.shape)


def f16(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float64).astype(np.float16)


def had_in(x: np.ndarray, suh: np.ndarray) -> np.ndarray:
    """fp16(H(fp16(x * suh)) / sqrt(128)) per 128-block (reference had_in faithful, :277-287)."""
    p = f16(f16(x).astype(np.float64) * f16(suh).astype(np.float64))
    return f16(had128(p))


def had_out(c: np.ndarray, svh: np.ndarray) -> np.ndarray:
    """fp16(fp16(H(fp16 c) / sqrt(128)) * svh) (reference had_out faithful, :290-301)."""
    y = f16(had128(f16(c)))
    return f16(y.astype(np.float64) * f16(svh).astype(np.float64))


def had_r_128(x: np.ndarray, pre: np.ndarray | None, post: np.ndarray | None, scale: float = 1.0) -> np.ndarray:
    """The standalone transform op: [pre-scale] -> H/sqrt(128)*scale -> fp16 [-> post-scale]."""
    v = f16(x).astype(np.float64)
    if pre is not None:
        v = f16(v * f16(pre).astype(np.float64)).astype(np.float64)
    y = f16(had128(v, R_SCALE * scale))
    if post is not None:
        y = f16(y.astype(np.float64) * f16(post).astype(np.float64))
    return y


# ---------------------------------------------------------------------------------------------
# the linear (reference gemv_mul1, :307-351, generalised to M rows and all codebooks)
# ---------------------------------------------------------------------------------------------
def linear(x: np.ndarray, trellis: np.ndarray, K: int, suh: np.ndarray, svh: np.ndarray,
           cb: int = CB_MUL1) -> np.ndarray:
    """y[M, n] = had_out(fp16(had_in(x, suh) @ W), svh), with an order-free float64 dot.

    Matches the kernels' staging: fp16 x, fp16 suh pre-scale, fp16 A_had, fp32-or-better
    accumulation, fp16 c_rot, fp16 transform output, fp16 svh post-scale.
    """
    x = np.atleast_2d(np.asarray(x))
    kt, nt, _ = trellis.shape
    k, n = kt * 16, nt * 16
    assert x.shape[1] == k and suh.shape == (k,) and svh.shape == (n,)
    a = had_in(x, suh).astype(np.float64)
    c = np.zeros((x.shape[0], n), dtype=np.float64)
    tab = codebook_table(cb)
    step = max(1, (1 << 22) // n)
    for k0 in range(0, kt, step):
        st = tile_states(trellis[k0:k0 + step], K)
        w = states_to_matrix(tab[st]).view(np.float16).astype(np.float64)
        c += a[:, k0 * 16:k0 * 16 + w.shape[0]] @ w
    return had_out(c, svh)


def random_trellis(rng: np.random.Generator, k_tiles: int, n_tiles: int, K: int) -> np.ndarray:
    """Uniform codes, the reference fixture generator's distribution (reference :415-417)."""
    return rng.integers(0, 65536, size=(k_tiles, n_tiles, 16 * K), dtype=np.uint16)


def state_transition_ok(states: np.ndarray, K: int) -> bool:
    """w_{t+1} == ((w_t << K) & 0xFFFF) | (w_{t+1} & (2^K - 1)) around the ring (reference :420-425)."""
    w = np.asarray(states, dtype=np.uint32)
    nxt = np.roll(w, -1, axis=-1)
    return bool(((((w << K) & 0xFFFF) | (nxt & ((1 << K) - 1))) == nxt).all())
