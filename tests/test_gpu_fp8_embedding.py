"""exl3rocm::fp8_embedding (reference vllm_plugin/exl3rocm/ops.py:183-202) on this library's gather
kernel: rows of a float8_e4m3fn table cast to fp16, bit for bit equal to torch's index_select and
.to(float16) of the same rows, for int64 and int32 ids of any shape; ids outside the table give zero
rows (the C ABI's documented rule; vLLM masks ids outside a rank's shard before the lookup)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def table():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    import exl3rocm.ops  # noqa: F401
    g = torch.Generator(device=DEV)
    g.manual_seed(7)
    raw = torch.randint(0, 256, (1000, 5120), generator=g, device=DEV, dtype=torch.int32).to(torch.uint8)
    raw[(raw & 0x7F) == 0x7F] = 0x3C  # no NaN encodings: their payloads need not match
    return raw.view(torch.float8_e4m3fn)


def ref(table, ids):
    return table.view(torch.uint8).index_select(0, ids.reshape(-1).long()).view(torch.float8_e4m3fn) \
        .to(torch.float16).view(*ids.shape, table.shape[1])


@pytest.mark.parametrize("dtype,shape", [(torch.int64, (7,)), (torch.int32, (2, 5)), (torch.int64, (1,)),
                                         (torch.int32, (300,))])
def test_matches_torch_cast(table, dtype, shape):
    g = torch.Generator(device=DEV)
    g.manual_seed(sum(shape))
    ids = torch.randint(0, table.shape[0], shape, generator=g, device=DEV).to(dtype)
    out = torch.ops.exl3rocm.fp8_embedding(table, ids)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16 and out.shape == (*shape, table.shape[1])
    assert torch.equal(out.view(torch.int16), ref(table, ids).view(torch.int16))


def test_out_of_range_ids_give_zero_rows(table):
    ids = torch.tensor([3, -1, 1000, 999], device=DEV)
    out = torch.ops.exl3rocm.fp8_embedding(table, ids)
    torch.cuda.synchronize()
    assert torch.equal(out[0], ref(table, ids[:1])[0]) and torch.equal(out[3], ref(table, ids[3:])[0])
    assert not out[1].any() and not out[2].any()


def test_graph_replay(table):
    ids = torch.randint(0, table.shape[0], (16,), device=DEV)
    torch.ops.exl3rocm.fp8_embedding(table, ids)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = torch.ops.exl3rocm.fp8_embedding(table, ids)
    ids.copy_(torch.randint(0, table.shape[0], (16,), device=DEV))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref(table, ids).view(torch.int16))
