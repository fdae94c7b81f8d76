"""Host-side sharding of the synthetic decoder (exl3rocm.synthetic), on CPU tensors.

Every rank draws the whole model from the same seed and keeps its shard, so the shards of a
tensor-parallel model must reassemble exactly into the single-GPU model's weights: column-parallel
matrices (q, k, v, gate, up) along n, row-parallel ones (o, down) along k, with the norms
replicated; and the lm_head's column ranges must tile the vocabulary in whole 128-column blocks.
"""
from __future__ import annotations

import pytest
import torch

from exl3rocm.synthetic import DecoderShape, Layer, head_columns

SMALL = DecoderShape(layers=1, hidden=512, q_heads=4, kv_heads=2, intermediate=1024, vocab=1024)


def _layer(tp, rank, seed=9):
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    return Layer(gen, SMALL, "cpu", tp, rank)


@pytest.mark.parametrize("tp", [2])
def test_shards_reassemble_the_single_gpu_layer(tp):
    full = _layer(1, 0)
    shards = [_layer(tp, r) for r in range(tp)]
    for name in ("q", "k", "v", "gate", "up"):  # column-parallel: split n
        w = getattr(full, name)
        assert torch.equal(torch.cat([getattr(s, name).trellis for s in shards], dim=1), w.trellis)
        assert torch.equal(torch.cat([getattr(s, name).svh for s in shards]), w.svh)
        assert all(torch.equal(getattr(s, name).suh, w.suh) for s in shards)
    for name in ("o", "down"):  # row-parallel: split k
        w = getattr(full, name)
        assert torch.equal(torch.cat([getattr(s, name).trellis for s in shards], dim=0), w.trellis)
        assert torch.equal(torch.cat([getattr(s, name).suh for s in shards]), w.suh)
        assert all(torch.equal(getattr(s, name).svh, w.svh) for s in shards)
    for s in shards:
        assert torch.equal(s.norm_in, full.norm_in) and torch.equal(s.norm_post, full.norm_post)
        assert s.o.trellis.shape[0] * 16 == SMALL.q_heads * SMALL.head // tp


@pytest.mark.parametrize("vocab,tp", [(151936, 1), (151936, 2), (151936, 4), (151936, 8), (1024, 2), (384, 8)])
def test_head_columns_tile_the_vocabulary(vocab, tp):
    ranges = [head_columns(vocab, tp, r) for r in range(tp)]
    assert ranges[0][0] == 0 and ranges[-1][1] == vocab
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    for c0, c1 in ranges:
        assert c0 % 128 == 0 and c1 % 128 == 0 and c1 >= c0
