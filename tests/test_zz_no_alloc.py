"""exl3b_linear_noalloc: the EXL3 linear for callers that cannot allocate device memory.

Some callers cannot hand the library a workspace: code running while a CUDA graph is being
captured (cudaMalloc is not allowed there), hosts whose device memory belongs to a pool the caller
cannot reach, and latency-critical paths that cannot afford cudaMalloc's implicit device
synchronisation.  For them exl3b_linear_noalloc keeps its scratch in a static device array.  This
test calls it through the C ABI, twice in a row, and checks each result against the regular entry
point (exl3b_linear, which takes a caller-allocated workspace) with the same gates as the other
linear tests.  It lives in its own file, collected last, and passes alone or after the others.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import exl3_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
GATES = {"normalized_max_abs_err": 3e-3, "normalized_rms_err": 2e-4, "cosine_similarity_min": 0.999999}


def _gates(got: np.ndarray, ref: np.ndarray) -> dict:
    got, ref = got.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    d = got - ref
    scale = np.sqrt(np.mean(ref ** 2)) or 1.0
    return {"normalized_max_abs_err": float(np.abs(d).max() / scale),
            "normalized_rms_err": float(np.sqrt(np.mean(d ** 2)) / scale),
            "cosine_similarity": float(got @ ref / ((np.linalg.norm(got) * np.linalg.norm(ref)) or 1.0))}


def _check(st: dict):
    assert st["normalized_max_abs_err"] <= GATES["normalized_max_abs_err"], st
    assert st["normalized_rms_err"] <= GATES["normalized_rms_err"], st
    assert st["cosine_similarity"] >= GATES["cosine_similarity_min"], st


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    import exl3rocm.ops  # noqa: F401  (the regular entry point, for comparison)
    from exl3rocm import _lib
    return _lib


# m = 16 at the model's layer widths (q / o 5120 -> 5120, gate / up 5120 -> 17408, down 17408 -> 5120)
# needs more than the old 8 MiB; the array is sized so that every m <= 16 call up to n = 131072 fits
@pytest.mark.parametrize("m,k,n,K,cb", [(1, 5120, 2048, 4, 2), (4, 2048, 1024, 3, 0), (16, 1024, 512, 5, 1),
                                        (16, 5120, 5120, 4, 2), (16, 5120, 17408, 3, 2), (16, 17408, 5120, 4, 2)])
def test_noalloc_matches_regular_entry_point(lib, m, k, n, K, cb):
    rng = np.random.default_rng(4000 + m + K)
    tr = O.random_trellis(rng, k // 16, n // 16, K)
    suh = np.sign(rng.standard_normal(k)).astype(np.float16)
    svh = np.sign(rng.standard_normal(n)).astype(np.float16)
    x = rng.standard_normal((m, k)).astype(np.float16)
    xd, td = torch.from_numpy(x).to(DEV), torch.from_numpy(tr.view(np.int16)).to(DEV)
    sd, vd = torch.from_numpy(suh).to(DEV), torch.from_numpy(svh).to(DEV)
    regular = torch.ops.exl3rocm.linear(xd, td, sd, vd, K, cb == 1, cb == 2).cpu().numpy()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        y = torch.full((m, n), float("nan"), dtype=torch.float16, device=DEV)
        st = lib.lib().exl3b_linear_noalloc(xd.data_ptr(), m, k, td.data_ptr(), n, K, cb, sd.data_ptr(),
                                            vd.data_ptr(), y.data_ptr(), n, stream)
        torch.cuda.synchronize()
        assert st == lib.EXL3B_OK, lib.lib().exl3b_status_string(st)
        err = ctypes.c_int(-1)
        assert lib.lib().exl3b_linear_noalloc_error(ctypes.byref(err), stream) == lib.EXL3B_OK
        assert err.value == 0
        _check(_gates(y.cpu().numpy(), regular))


def test_noalloc_rejects_calls_beyond_its_scratch(lib):
    # n = 2^20 columns at m = 16: the cross-CTA partial sums alone need far more than the static
    # 32 MiB scratch.  Every buffer has the size the call declares, so nothing could be read out of bounds
    # even if the call were accepted.
    m, k, n, K = 16, 128, 1 << 20, 4
    L = lib.lib()
    # even the smallest possible need at this width (every column once, no CTA overlap) is too large
    assert 4 * m * n > 32 << 20
    x = torch.zeros(m, k, dtype=torch.float16, device=DEV)
    tr = torch.zeros(k // 16, n // 16, 16 * K, dtype=torch.int16, device=DEV)
    suh = torch.ones(k, dtype=torch.float16, device=DEV)
    svh = torch.ones(n, dtype=torch.float16, device=DEV)
    y = torch.full((m, n), float("nan"), dtype=torch.float16, device=DEV)
    st = L.exl3b_linear_noalloc(x.data_ptr(), m, k, tr.data_ptr(), n, K, 2, suh.data_ptr(), svh.data_ptr(),
                                y.data_ptr(), n, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert st == lib.EXL3B_TOO_LARGE
    assert b"static scratch" in L.exl3b_status_string(st)
    assert torch.isnan(y).all()
