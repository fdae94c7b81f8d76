"""Generate the EXL3 golden vectors from the reference's own CPU oracle.

Run once, in a container where the reference checkout is present:

    python tests/golden/make_golden.py <path to a Luke458/qwen38-27b-exl3-rdna4 checkout>

It imports ``reference/exl3_oracle.py`` of that checkout by path and writes
``tests/golden/exl3_golden.npz``.  The tests never need the reference at run time: they read the
committed .npz.  Seeds follow the reference tests (20260923, tests/test_oracle.py:17).
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "exl3_golden.npz")


def load_reference(root: str):
    path = os.path.join(root, "reference", "exl3_oracle.py")
    spec = importlib.util.spec_from_file_location("ref_exl3_oracle", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def f16bits(v: np.ndarray) -> np.ndarray:
    """float64 arrays holding exact fp16 values -> uint16 bit patterns (asserting exactness)."""
    h = np.asarray(v, dtype=np.float64).astype(np.float16)
    assert (h.astype(np.float64) == np.asarray(v, dtype=np.float64)).all(), "value not on the fp16 grid"
    return h.view(np.uint16)


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(root: str) -> None:
    R = load_reference(root)
    rng = np.random.default_rng(20260923)
    g: dict[str, np.ndarray] = {}

    # 1. every 16-bit state through every codebook: full-table digests plus a sample
    allw = np.arange(65536, dtype=np.uint16)
    sample = rng.integers(0, 65536, size=2048, dtype=np.uint16)
    g["cb_sample_states"] = sample
    for cb in (0, 1, 2):
        table = f16bits(R.decode_codebook(allw, cb))
        g[f"cb{cb}_table_sha256"] = np.frombuffer(bytes.fromhex(digest(table)), dtype=np.uint8)
        g[f"cb{cb}_sample_values"] = table[sample]

    # 2. state windows for K = 1..8 on random and boundary tiles
    for K in range(1, 9):
        tiles = [rng.integers(0, 65536, size=16 * K, dtype=np.uint16) for _ in range(3)]
        tiles += [np.zeros(16 * K, np.uint16), np.full(16 * K, 0xFFFF, np.uint16),
                  np.arange(16 * K, dtype=np.uint16), (np.arange(16 * K, dtype=np.uint16) * 7919)]
        tiles = np.stack(tiles).astype(np.uint16)
        g[f"win_tiles_K{K}"] = tiles
        g[f"win_states_K{K}"] = np.stack([R.tile_windows(t, K) for t in tiles])

    # 3. full decode (reconstruct) of small trellises, every K and codebook; plus digests of
    #    128x128 decodes (the reference GPU test shape, tests/test_gpu_parity.py:128-139)
    for K in range(1, 9):
        tr = R.random_trellis(rng, 2, 3, K)
        g[f"dq_trellis_K{K}"] = tr
        for cb in (0, 1, 2):
            g[f"dq_W_K{K}_cb{cb}"] = f16bits(R.decode_trellis(tr, K, cb))
        tr128 = R.random_trellis(rng, 8, 8, K)
        g[f"dq128_trellis_K{K}"] = tr128
        for cb in (0, 2):
            W = f16bits(R.decode_trellis(tr128, K, cb))
            g[f"dq128_sha256_K{K}_cb{cb}"] = np.frombuffer(bytes.fromhex(digest(W)), dtype=np.uint8)

    # 4. the faithful GEMV (reference gemv_mul1) on small shapes, several K and codebooks,
    #    with the reference test's two sign families (tests/test_gpu_parity.py:85-95)
    cases = [(256, 128, 3, 2, False), (128, 256, 4, 0, True), (256, 256, 2, 1, True),
             (128, 128, 5, 2, True), (384, 128, 8, 2, False), (128, 384, 6, 0, False),
             (256, 128, 1, 2, True), (128, 128, 7, 1, False)]
    g["gemv_cases"] = np.array([c[:4] + (int(c[4]),) for c in cases], dtype=np.int64)
    for ci, (k, n, K, cb, signs) in enumerate(cases):
        tr = R.random_trellis(rng, k // 16, n // 16, K)
        if signs:
            suh = np.sign(rng.standard_normal(k)).astype(np.float16)
            svh = np.sign(rng.standard_normal(n)).astype(np.float16)
        else:
            suh = (np.abs(rng.standard_normal(k)) * 0.5 + 0.5).astype(np.float16)
            svh = (np.abs(rng.standard_normal(n)) * 0.5 + 0.5).astype(np.float16)
        a = (rng.standard_normal(k) * 0.3).astype(np.float16)
        y = R.gemv_mul1(a.astype(np.float64), tr, K, suh.astype(np.float64), svh.astype(np.float64),
                        cb=cb, faithful=True)
        g[f"gemv{ci}_trellis"] = tr
        g[f"gemv{ci}_suh"] = suh.view(np.uint16)
        g[f"gemv{ci}_svh"] = svh.view(np.uint16)
        g[f"gemv{ci}_x"] = a.view(np.uint16)
        g[f"gemv{ci}_y"] = f16bits(y)
        g[f"gemv{ci}_xhad"] = f16bits(R.had_in(a.astype(np.float64), suh.astype(np.float64), faithful=True))

    # 5. the transform stages alone
    x = rng.standard_normal((4, 256)).astype(np.float16)
    s = np.sign(rng.standard_normal(256)).astype(np.float16)
    g["had_x"] = x.view(np.uint16)
    g["had_s"] = s.view(np.uint16)
    g["had_in_y"] = f16bits(R.had_in(x.astype(np.float64), s.astype(np.float64), faithful=True))
    g["had_out_y"] = f16bits(R.had_out(x.astype(np.float64), s.astype(np.float64), faithful=True))
    g["had_matrix_sha256"] = np.frombuffer(bytes.fromhex(digest(R.had128_matrix().astype(np.int8))),
                                           dtype=np.uint8)

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT}: {len(g)} arrays, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
