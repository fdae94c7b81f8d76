"""The MTP drafter's pruned lm_head (exl3rocm.plugin.prune_draft_head; reference plugin.py:431-528) on
the GPU: splitting the head into [drafted prefix | middle | drafted tail] groups leaves the target's
logits as they were (within the linear's gates: the stream-K partition follows the group widths, so
the summation order may move), and the drafter's logits equal the head's at the drafted columns and
are -inf elsewhere."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def plugin():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return pytest.importorskip("exl3rocm.plugin", reason="vLLM not importable")


def nrms(a, b):
    a, b = a.double(), b.double()
    return float((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt())


def test_pruned_head(plugin, monkeypatch):
    from exl3rocm import sharding as S
    monkeypatch.setenv("EXL3_DRAFT_VOCAB_BLOCKS", "24")
    rng = np.random.default_rng(4)
    k, n, K = 1024, 64 * 128, 4
    shard = S.module_shard([("lm_head", K, k, n)], "column", 1, 0, device=DEV)
    shard.load("trellis", 0, torch.from_numpy(rng.integers(-32768, 32768, (k // 16, n // 16, 16 * K)).astype(np.int16)))
    shard.load("suh", 0, torch.from_numpy(np.sign(rng.standard_normal(k)).astype(np.float16)))
    shard.load("svh", 0, torch.from_numpy(np.sign(rng.standard_normal(n)).astype(np.float16)))
    x = torch.from_numpy((rng.standard_normal((3, k)) * 0.3).astype(np.float16)).to(DEV)
    before = shard.forward(x, False, True)
    layer = torch.nn.Module()
    layer.exl3_shard, layer.exl3_mul1, layer.exl3_mcg = shard, True, False
    assert plugin.prune_draft_head(layer)
    after = shard.forward(x, False, True)
    draft = plugin.draft_logits(layer, x)
    torch.cuda.synchronize()
    assert after.shape == before.shape and nrms(after, before) < 1e-3
    cols = layer.exl3_draft_cols
    assert cols.numel() == (24 + 16) * 128
    assert nrms(draft[:, cols], before[:, cols]) < 1e-3
    mask = torch.ones(n, dtype=torch.bool, device=DEV)
    mask[cols] = False
    assert torch.isinf(draft[:, mask]).all() and (draft[:, mask] < 0).all()
