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


def test_fp8_embedding_detected_and_chosen(tmp_path):
    """An F8_E4M3 language-model embed_tokens in the checkpoint makes the input embedding an fp8 table
    looked up by exl3rocm::fp8_embedding (reference plugin.py:117-120, 158-159, 215-233); a vision
    tower's fp8 embedding does not count."""
    from vllm.model_executor.layers.vocab_parallel_embedding import VocabParallelEmbedding
    t = {"model.language_model.layers.0.mlp.down_proj.trellis": ("I16", (32, 8, 64), 2),
         "model.language_model.embed_tokens.weight": ("F8_E4M3", (1024, 512), 1),
         "model.visual.embed_tokens.weight": ("F8_E4M3", (64, 512), 1)}
    _write_safetensors(tmp_path / "model-00001.safetensors", t)
    cfg = plugin.Exl3Config()
    cfg.maybe_update_config(str(tmp_path))
    assert cfg.fp8_embedding and cfg.embed_shape == (1024, 512)
    emb = object.__new__(VocabParallelEmbedding)  # an instance for the type checks, not built
    torch.nn.Module.__init__(emb)
    assert isinstance(cfg.get_quant_method(emb, "model.language_model.embed_tokens"), plugin.Fp8EmbeddingMethod)
    assert cfg.get_quant_method(emb, "model.language_model.other") is None
    assert plugin.wants_fp8_embedding(cfg, 1024, 512) and not plugin.wants_fp8_embedding(cfg, 1024, 256)
    assert not plugin.wants_fp8_embedding(None, 1024, 512)

    meth = plugin.Fp8EmbeddingMethod()
    layer = torch.nn.Module()
    loader = lambda param, w: param.data.copy_(w)  # noqa: E731
    meth.create_weights(layer, 512, [512], 512, 1024, torch.float16, weight_loader=loader)  # a rank's half
    assert layer.weight.dtype == torch.float8_e4m3fn and tuple(layer.weight.shape) == (512, 512)
    assert layer.weight.output_dim == 0 and layer.weight.input_dim == 1 and layer.weight.weight_loader is loader
    with pytest.raises(NotImplementedError):
        meth.apply(layer, torch.zeros(1, 512))


def test_no_fp8_embedding_without_fp8_table(tmp_path):
    t = {"model.embed_tokens.weight": ("BF16", (1024, 512), 2),
         "model.layers.0.mlp.down_proj.trellis": ("I16", (32, 8, 64), 2)}
    _write_safetensors(tmp_path / "model-00001.safetensors", t)
    cfg = plugin.Exl3Config()
    cfg.maybe_update_config(str(tmp_path))
    assert not cfg.fp8_embedding


def _loaded_head(n_blocks, k=256, K=4, seed=9):
    rng = np.random.default_rng(seed)
    n = n_blocks * 128
    shard = S.module_shard([("lm_head", K, k, n)], "column", 1, 0)
    tr, suh, svh = _full(rng, K, k, n)
    shard.load("trellis", 0, tr)
    shard.load("suh", 0, suh)
    shard.load("svh", 0, svh)
    return shard, tr, suh, svh


def test_draft_bounds_rule():
    """First EXL3_DRAFT_VOCAB_BLOCKS blocks plus the last 16 (reference plugin.py:431-441)."""
    assert S.draft_bounds(1187 * 128, 640) == (640 * 128, 1171 * 128)
    assert S.draft_bounds(656 * 128, 640) is None and S.draft_bounds(2000 * 128, 0) is None


def test_split_columns_keeps_the_head():
    shard, tr, suh, svh = _loaded_head(40)
    shard.split_columns([8 * 128, 24 * 128])
    assert [s.stored_n for s in shard.shards] == [1024, 2048, 2048] and shard.out_sizes == [1024, 2048, 2048]
    assert torch.equal(torch.cat([s.trellis for s in shard.shards], 1), tr)
    assert torch.equal(torch.cat([s.svh for s in shard.shards]), svh)
    assert all(s.suh is shard.shards[0].suh for s in shard.shards) and torch.equal(shard.shards[0].suh, suh)
    assert all(s.trellis.is_contiguous() for s in shard.shards) and not shard.missing()
    with pytest.raises(ValueError):
        shard.split_columns([100])


def test_prune_draft_head_and_logits_patch(monkeypatch):
    monkeypatch.setenv("EXL3_DRAFT_VOCAB_BLOCKS", "20")
    shard, *_ = _loaded_head(40)
    layer = torch.nn.Module()
    layer.exl3_shard, layer.exl3_mul1, layer.exl3_mcg = shard, True, False
    assert plugin.prune_draft_head(layer)
    assert layer.exl3_draft_groups == (0, 2) and [s.stored_n for s in shard.shards] == [2560, 512, 2048]
    cols = layer.exl3_draft_cols
    assert torch.equal(cols, torch.cat([torch.arange(0, 2560), torch.arange(3072, 5120)]))

    class FakeMTP:  # compute_logits as vLLM's Qwen3_5MTP declares it
        def __init__(self, lm_head):
            self.lm_head, self.config = lm_head, type("C", (), {"vocab_size": 5000})()

        def compute_logits(self, hidden_states, spec_step_idx=0):
            return "vllm"

    assert plugin._install_draft_logits_patch(FakeMTP) and not plugin._install_draft_logits_patch(FakeMTP)
    monkeypatch.setattr(plugin, "draft_logits", lambda lm, h: torch.zeros(h.shape[0], 5120))
    out = FakeMTP(layer).compute_logits(torch.zeros(3, 256, dtype=torch.float16))
    assert out.shape == (3, 5000) and out.dtype == torch.float16
    assert FakeMTP(torch.nn.Module()).compute_logits(None) == "vllm"  # an unsplit head: vLLM's path
