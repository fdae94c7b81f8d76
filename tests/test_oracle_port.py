"""Pin the CPU oracle port against the reference oracle's golden vectors and known answers.

The known-answer cases restate the reference's own CPU tests (reference tests/test_oracle.py);
the golden vectors come from the reference oracle itself (tests/golden/make_golden.py).
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import exl3_oracle as O

RNG = np.random.default_rng(20260923)


def _sha(a) -> bytes:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest()


# ---- codebooks -------------------------------------------------------------------------------
@pytest.mark.parametrize("cb", [0, 1, 2])
def test_codebook_table_matches_reference_digest(golden, cb):
    table = O.codebook_table(cb)
    assert _sha(table) == golden[f"cb{cb}_table_sha256"].tobytes()
    np.testing.assert_array_equal(table[golden["cb_sample_states"]], golden[f"cb{cb}_sample_values"])


def test_mul1_known_answers():
    # reference tests/test_oracle.py:70-92
    assert O.K_INV == float(np.uint16(0x1EEE).view(np.float16))
    assert O.K_BIAS == float(np.uint16(0xC931).view(np.float16))
    v0 = float(O.decode_states(np.array([0], np.uint16), 2)[0])
    assert v0 == float(np.float16(O.K_INV * 1024.0 + O.K_BIAS))
    vals = O.decode_states(np.arange(65536, dtype=np.uint16), 2).astype(np.float64)
    assert vals.min() >= -3.5 and vals.max() <= 3.5
    w = np.array([0x1234, 0x5678, 0x9ABC, 0xDEF0], dtype=np.uint16)
    s = O._bytesum((w.astype(np.uint64) * O.MUL1_MULT) & 0xFFFFFFFF)
    for si, v in zip(s, O.decode_states(w, 2)):
        assert float(v) == float(np.float16(O.K_INV * (1024.0 + float(si)) + O.K_BIAS))


# ---- windows ---------------------------------------------------------------------------------
@pytest.mark.parametrize("K", range(1, 9))
def test_windows_match_reference(golden, K):
    st = O.tile_states(golden[f"win_tiles_K{K}"], K)
    np.testing.assert_array_equal(st, golden[f"win_states_K{K}"])
    assert O.state_transition_ok(st, K)


@pytest.mark.parametrize("K", range(1, 9))
def test_state_transition_identity_random(K):
    # reference tests/test_oracle.py:21-26
    tiles = RNG.integers(0, 65536, size=(4, 16 * K), dtype=np.uint16)
    assert O.state_transition_ok(O.tile_states(tiles, K), K)


def test_t_rowcol_bijection_and_fragment_layout():
    # reference tests/test_oracle.py:51-66
    assert len(set(zip(O.ROW.tolist(), O.COL.tolist()))) == 256
    for L in (0, 5, 31):
        t = np.array([8 * L + i for i in range(8)])
        r0, cA = 2 * (L % 4), 2 * (L // 8) + ((L >> 2) & 1)
        expect = [(r0, cA), (r0 + 1, cA), (r0 + 8, cA), (r0 + 9, cA),
                  (r0, cA + 8), (r0 + 1, cA + 8), (r0 + 8, cA + 8), (r0 + 9, cA + 8)]
        assert list(zip(O.ROW[t].tolist(), O.COL[t].tolist())) == expect


# ---- dequant ---------------------------------------------------------------------------------
@pytest.mark.parametrize("K", range(1, 9))
def test_dequant_matches_reference(golden, K):
    tr = golden[f"dq_trellis_K{K}"]
    for cb in (0, 1, 2):
        np.testing.assert_array_equal(O.dequant(tr, K, cb).view(np.uint16), golden[f"dq_W_K{K}_cb{cb}"])
    tr128 = golden[f"dq128_trellis_K{K}"]
    for cb in (0, 2):
        assert _sha(O.dequant(tr128, K, cb).view(np.uint16)) == golden[f"dq128_sha256_K{K}_cb{cb}"].tobytes()


def test_dequant_slice_is_column_slice(golden):
    tr = golden["dq128_trellis_K4"]
    full = O.dequant(tr, 4, 2)
    np.testing.assert_array_equal(O.dequant(tr, 4, 2, n0=32, n1=96), full[:, 32:96])


# ---- Hadamard --------------------------------------------------------------------------------
def test_hadamard_matrix_matches_reference(golden):
    assert _sha(O.had128_matrix().astype(np.int8)) == golden["had_matrix_sha256"].tobytes()
    H = O.had128_matrix()
    assert np.allclose(H @ H.T, 128.0 * np.eye(128))
    x = RNG.standard_normal(256)
    assert np.allclose(O.had128(O.had128(x)), x, atol=1e-10)


def test_had_stages_match_reference(golden):
    x = golden["had_x"].view(np.float16)
    s = golden["had_s"].view(np.float16)
    np.testing.assert_array_equal(O.had_in(x, s).view(np.uint16), golden["had_in_y"])
    np.testing.assert_array_equal(O.had_out(x, s).view(np.uint16), golden["had_out_y"])


# ---- the linear ------------------------------------------------------------------------------
def test_linear_matches_reference_gemv(golden):
    for ci, (k, n, K, cb, _signs) in enumerate(golden["gemv_cases"]):
        x = golden[f"gemv{ci}_x"].view(np.float16)
        suh = golden[f"gemv{ci}_suh"].view(np.float16)
        svh = golden[f"gemv{ci}_svh"].view(np.float16)
        tr = golden[f"gemv{ci}_trellis"]
        np.testing.assert_array_equal(O.had_in(x[None], suh)[0].view(np.uint16), golden[f"gemv{ci}_xhad"])
        y = O.linear(x[None], tr, int(K), suh, svh, int(cb))[0]
        ref = golden[f"gemv{ci}_y"].view(np.float16)
        # both sums are exact-ish float64; they can only differ where the fp16 rounding of c_rot
        # meets a tie, which random fixtures essentially never hit
        diff = np.abs(y.astype(np.float64) - ref.astype(np.float64))
        ulp = np.maximum(np.abs(ref.astype(np.float64)) * 2.0 ** -10, 2.0 ** -24)
        assert (diff <= ulp).all(), (ci, diff.max())
        assert (diff == 0).mean() > 0.99, ci


def test_linear_zero_input_and_outliers():
    # reference tests/test_oracle.py:143-148, 170-177
    tr = O.random_trellis(RNG, 8, 8, 3)
    suh = np.ones(128, np.float16)
    svh = np.ones(128, np.float16)
    assert (O.linear(np.zeros((1, 128), np.float16), tr, 3, suh, svh) == 0).all()
    a = np.tile([100.0, -100.0], 64)
    a[0] = 1e4
    assert np.isfinite(O.linear(a[None].astype(np.float16), tr, 3, suh, svh).astype(np.float64)).all()


def test_linear_rows_independent():
    tr = O.random_trellis(RNG, 16, 8, 4)
    suh = np.sign(RNG.standard_normal(256)).astype(np.float16)
    svh = np.sign(RNG.standard_normal(128)).astype(np.float16)
    x = RNG.standard_normal((5, 256)).astype(np.float16)
    y = O.linear(x, tr, 4, suh, svh)
    for r in range(5):
        np.testing.assert_array_equal(O.linear(x[r:r + 1], tr, 4, suh, svh)[0], y[r])
