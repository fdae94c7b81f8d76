"""The vLLM plugin surface (exl3rocm.plugin) on the CPU: quant config, checkpoint-header layout,
fused-module groups, and tensor-parallel create_weights + weight loaders slicing full checkpoint
tensors into each rank's shard.  Skipped where vLLM cannot be imported."""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest
import torch

plugin = pytest.importorskip("exl3rocm.plugin", reason="vLLM not importable")
from exl3rocm import sharding as S  # noqa: E402


def _write_safetensors(path, tensors):
    """Header-only-correct safetensors file (the data region is zeros)."""
    header, off = {}, 0
    for name, (dtype, shape, nbytes) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    blob = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        f.write(b"\0" * off)


def test_config_surface():
    cfg = plugin.Exl3Config.from_config({"codebook": "mul1"})
    assert cfg.get_name() == "exl3"
    assert cfg.get_supported_act_dtypes() == [torch.float16]
    assert plugin.Exl3Config.get_min_capability() == 0
    assert plugin.Exl3Config.get_config_filenames() == []


def test_checkpoint_layout_and_groups(tmp_path):
    t = {}
    for name, (K, k, n) in {"q_proj": (2, 512, 512), "k_proj": (5, 512, 128), "v_proj": (5, 512, 128),
                            "gate_proj": (4, 512, 1024), "up_proj": (4, 512, 1024)}.items():
        mod = "self_attn" if name[0] in "qkv" else "mlp"
        t[f"model.language_model.layers.3.{mod}.{name}.trellis"] = ("I16", (k // 16, n // 16, 16 * K), 2)
        t[f"model.language_model.layers.3.{mod}.{name}.suh"] = ("F16", (k,), 2)
    _write_safetensors(tmp_path / "model-00001.safetensors", t)
    cfg = plugin.Exl3Config()
    cfg.maybe_update_config(str(tmp_path))
    assert cfg.modules["layers.3.self_attn.k_proj"] == (5, 512, 128)
    assert cfg.modules["layers.3.mlp.up_proj"] == (4, 512, 1024)
    g = cfg.groups_for("language_model.model.layers.3.self_attn.qkv_proj")
    assert [x[0] for x in g] == ["layers.3.self_attn.q_proj", "layers.3.self_attn.k_proj",
                                 "layers.3.self_attn.v_proj"]
    assert [x[1] for x in g] == [2, 5, 5]
    assert cfg.groups_for("model.layers.3.mlp.down_proj") is None


def _full(rng, K, k, n):
    tr = rng.integers(-32768, 32768, size=(k // 16, n // 16, 16 * K), dtype=np.int64).astype(np.int16)
    return (torch.from_numpy(tr), torch.from_numpy(rng.standard_normal(k).astype(np.float16)),
            torch.from_numpy(rng.standard_normal(n).astype(np.float16)))


@pytest.mark.parametrize("rank", [0, 1])
def test_column_parallel_qkv_loaders(rank):
    rng = np.random.default_rng(1)
    groups = [("q", 4, 512, 512), ("k", 4, 512, 256), ("v", 4, 512, 256)]
    full = [_full(rng, K, k, n) for _, K, k, n in groups]
    cfg = plugin.Exl3Config()
    meth = plugin.Exl3LinearMethod(cfg, groups, tp=(2, rank))
    layer = torch.nn.Module()
    meth.create_weights(layer, 512, [256, 128, 128], 512, 1024, torch.float16)
    for sid, (tr, suh, svh) in zip("qkv", full):
        layer.trellis.weight_loader(layer.trellis, tr, sid)
        layer.suh.weight_loader(layer.suh, suh, sid)
        layer.svh.weight_loader(layer.svh, svh, sid)
    layer.mul1.weight_loader(layer.mul1, torch.tensor(1))
    meth.process_weights_after_loading(layer)
    sh = layer.exl3_shard
    assert sh.parallel == "column" and sh.out_sizes == [256, 128, 128]
    for g, (tr, suh, svh) in enumerate(full):
        n = groups[g][3]
        c0, c1 = rank * n // 2, (rank + 1) * n // 2
        assert torch.equal(sh.shards[g].trellis, tr[:, c0 // 16:c1 // 16])
        assert torch.equal(sh.shards[g].suh, suh)
        assert torch.equal(sh.shards[g].svh, svh[c0:c1])
    assert layer.exl3_mul1 and not layer.exl3_mcg
    assert "trellis" not in layer._parameters


def test_row_parallel_down_loader():
    rng = np.random.default_rng(2)
    groups = [("down", 3, 1024, 256)]
    tr, suh, svh = _full(rng, 3, 1024, 256)
    meth = plugin.Exl3LinearMethod(plugin.Exl3Config(), groups, tp=(4, 2))
    layer = torch.nn.Module()
    meth.create_weights(layer, 256, [256], 1024, 256, torch.float16)
    layer.trellis.weight_loader(layer.trellis, tr)
    layer.suh.weight_loader(layer.suh, suh)
    layer.svh.weight_loader(layer.svh, svh)
    meth.process_weights_after_loading(layer)
    sh = layer.exl3_shard
    assert sh.parallel == "row" and sh.local_k == 256
    assert torch.equal(sh.shards[0].trellis, tr[32:48])
    assert torch.equal(sh.shards[0].suh, suh[512:768]) and torch.equal(sh.shards[0].svh, svh)


def test_missing_tensor_raises_at_process():
    meth = plugin.Exl3LinearMethod(plugin.Exl3Config(), [("o", 4, 256, 128)], tp=(1, 0))
    layer = torch.nn.Module()
    meth.create_weights(layer, 256, [128], 256, 128, torch.float16)
    tr, suh, _ = _full(np.random.default_rng(3), 4, 256, 128)
    layer.trellis.weight_loader(layer.trellis, tr)
    layer.suh.weight_loader(layer.suh, suh)
    with pytest.raises(RuntimeError, match="never loaded"):
        meth.process_weights_after_loading(layer)


def test_partitions_must_tile_groups():
    meth = plugin.Exl3LinearMethod(plugin.Exl3Config(), [("gate", 4, 256, 256), ("up", 4, 256, 256)], tp=(1, 0))
    with pytest.raises(ValueError):
        meth.create_weights(torch.nn.Module(), 256, [256, 128], 256, 384, torch.float16)
