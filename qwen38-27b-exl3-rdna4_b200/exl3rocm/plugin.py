"""vLLM out-of-tree quantization plugin "exl3" for B200: the reference's plugin surface
(``vllm_plugin/exl3rocm/plugin.py``), with tensor-parallel weights.

Registered through the ``vllm.general_plugins`` entry point ``exl3rocm = exl3rocm.plugin:register``
(reference ``vllm_plugin/pyproject.toml:13-14``).  What it keeps from the reference's behaviour:

* quant method name ``exl3``; fp16 activations; minimum capability 0 (``plugin.py:82-107``);
* the EXL3 module map comes from the checkpoint's safetensors headers, K = trellis last dim / 16
  (``plugin.py:63-79``);
* fused vLLM modules (qkv_proj, gate_up_proj, ...) hold one group per checkpoint tensor, each with
  its own K, trellis, suh and svh, and run as one ``exl3rocm::linear_groups`` op
  (``plugin.py:236-372``).

What differs: ``create_weights`` accepts tensor-parallel partitions (the reference raises,
``plugin.py:255-257``).  Each rank stores only its shard (``exl3rocm.sharding``): column-parallel
modules their output columns, row-parallel modules their 128-blocks of input features, and the
weight loaders slice the full checkpoint tensors they are handed.
"""
from __future__ import annotations

import glob
import json
import os
import re
import struct
from typing import Any, Optional

import torch
from torch.nn import Parameter

from vllm.model_executor.layers.linear import LinearBase, LinearMethodBase, UnquantizedLinearMethod
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig
from vllm.model_executor.layers.vocab_parallel_embedding import ParallelLMHead

from . import sharding

# vLLM fused module -> checkpoint constituents, in output order (reference plugin.py:38-44)
FUSED = {
    "gate_up_proj": ["gate_proj", "up_proj"],
    "qkv_proj": ["q_proj", "k_proj", "v_proj"],
    "in_proj_qkvz": ["in_proj_qkv", "in_proj_z"],
    "in_proj_ba": ["in_proj_b", "in_proj_a"],
    "qkv": ["q_proj", "k_proj", "v_proj"],
}
SHARD_IDS = {"q": 0, "k": 1, "v": 2}


def module_key(name: str) -> str:
    """The module name shared by checkpoint keys and vLLM prefixes: the part from ``layers.N.``
    on (``mtp.`` / ``visual.`` kept as a namespace), else the last component."""
    parts = name.split(".")
    for ns in ("visual", "mtp"):
        if ns in parts:
            return ns + "." + ".".join(parts[parts.index(ns) + 1:])
    m = re.search(r"(layers\.\d+\..*)$", name)
    return m.group(1) if m else parts[-1]


def read_checkpoint_layout(model_dir: str) -> dict[str, tuple[int, int, int]]:
    """{module key: (K, k, n)} for every ``<module>.trellis`` tensor of the checkpoint, read from
    the safetensors headers only (8-byte little-endian header length, then JSON)."""
    layout = {}
    for path in sorted(glob.glob(os.path.join(model_dir, "*.safetensors"))):
        with open(path, "rb") as f:
            (hlen,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(hlen))
        for name, meta in header.items():
            if name == "__metadata__" or not name.endswith(".trellis"):
                continue
            kt, nt, w = meta["shape"]
            layout[module_key(name[: -len(".trellis")])] = (w // 16, kt * 16, nt * 16)
    return layout


def _tp() -> tuple[int, int]:
    try:
        from vllm.distributed import get_tensor_model_parallel_rank, get_tensor_model_parallel_world_size
        return get_tensor_model_parallel_world_size(), get_tensor_model_parallel_rank()
    except Exception:  # no distributed state (single process, tests)
        return 1, 0


def _tp_group():
    try:
        from vllm.distributed import get_tp_group
        return get_tp_group().cpu_group
    except Exception:
        return None


@register_quantization_config("exl3")
class Exl3Config(QuantizationConfig):
    """Quant config "exl3"; the module map is filled from the checkpoint by maybe_update_config."""

    def __init__(self, codebook: str = "mul1"):
        super().__init__()
        self.codebook = codebook
        self.modules: dict[str, tuple[int, int, int]] = {}

    def __repr__(self):
        return f"Exl3Config(codebook={self.codebook}, modules={len(self.modules)})"

    def get_name(self):
        return "exl3"

    def get_supported_act_dtypes(self):
        return [torch.float16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 0

    @staticmethod
    def get_config_filenames() -> list[str]:
        return []

    @classmethod
    def from_config(cls, config: dict[str, Any]) -> "Exl3Config":
        return cls(codebook=config.get("codebook", "mul1"))

    def maybe_update_config(self, model_name: str, hf_config=None, revision=None):
        if not os.path.isdir(model_name):
            raise NotImplementedError("exl3rocm: pass a local checkpoint directory")
        self.modules = read_checkpoint_layout(model_name)

    def groups_for(self, prefix: str) -> Optional[list[tuple[str, int, int, int]]]:
        """The checkpoint members of the (possibly fused) vLLM module at ``prefix`` as
        [(member, K, k, n)], or None when the module is not EXL3."""
        key = module_key(prefix)
        base, _, leaf = key.rpartition(".")
        members = [f"{base}.{p}" if base else p for p in FUSED.get(leaf, [leaf])]
        found = [self.modules.get(m) for m in members]
        if all(f is None for f in found):
            return None
        if any(f is None for f in found):
            raise ValueError(f"exl3rocm: partially quantized fused module {prefix}")
        return [(m, *f) for m, f in zip(members, found)]

    def get_quant_method(self, layer: torch.nn.Module, prefix: str):
        if isinstance(layer, (LinearBase, ParallelLMHead)):
            groups = self.groups_for(prefix)
            if groups is None:
                return UnquantizedLinearMethod() if isinstance(layer, LinearBase) else None
            return Exl3LinearMethod(self, groups)
        return None


def parallel_mode(input_size_per_partition: int, input_size: int, output_partition_sizes: list[int],
                  output_size: int) -> str:
    if input_size_per_partition != input_size:
        return "row"
    if sum(output_partition_sizes) != output_size:
        return "column"
    return "replicated"


class Exl3LinearMethod(LinearMethodBase):
    """Per-group EXL3 storage for one rank.  The registered parameters ``trellis``, ``suh``,
    ``svh`` (and the codebook scalar) are 0-size load targets that vLLM's name mapping resolves to;
    their weight_loader slices each full checkpoint tensor into this rank's shard."""

    def __init__(self, config: Exl3Config, groups, tp: Optional[tuple[int, int]] = None):
        self.config = config
        self.groups = groups  # [(member, K, k, n)]
        self.tp = tp          # (size, rank); None = ask vLLM at create_weights

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **extra_weight_attrs):
        tp_size, tp_rank = self.tp or _tp()
        mode = parallel_mode(input_size_per_partition, input_size, list(output_partition_sizes), output_size)
        shard = sharding.module_shard(self.groups, mode, tp_size, tp_rank,
                                      device=torch.cuda.current_device() if torch.cuda.is_available() else "cpu")
        if mode == "row" and shard.local_k != input_size_per_partition:
            raise ValueError(f"exl3rocm: row shard k={shard.local_k}, vLLM expects {input_size_per_partition}")
        # map vLLM's output partitions onto groups (a group may span partitions, e.g. q, k, v of
        # in_proj_qkv inside in_proj_qkvz)
        widths, part_to_group, gi, acc = shard.out_sizes, [], 0, 0
        for p in output_partition_sizes:
            if gi >= len(widths):
                raise ValueError(f"exl3rocm: partitions {list(output_partition_sizes)} do not tile groups {widths}")
            part_to_group.append(gi)
            acc += p
            if acc > widths[gi]:
                raise ValueError(f"exl3rocm: partitions {list(output_partition_sizes)} do not tile groups {widths}")
            if acc == widths[gi]:
                gi, acc = gi + 1, 0
        if gi != len(widths):
            raise ValueError(f"exl3rocm: partitions {list(output_partition_sizes)} do not tile groups {widths}")
        layer.exl3_shard = shard
        layer.exl3_part_to_group = part_to_group
        layer.exl3_codebook = {}

        def reg(name, loader):
            p = Parameter(torch.empty(0, dtype=torch.int8), requires_grad=False)
            p.weight_loader = loader
            layer.register_parameter(name, p)

        for kind in ("trellis", "suh", "svh"):
            reg(kind, self._loader(layer, kind))
        if self.config.codebook in ("mul1", "mcg"):
            reg(self.config.codebook, self._loader(layer, self.config.codebook))

    @staticmethod
    def _group_of(layer, shard_id) -> int:
        if shard_id is None:
            if len(layer.exl3_shard.groups) != 1:
                raise ValueError("exl3rocm: unsharded load into a fused module")
            return 0
        parts = [SHARD_IDS[shard_id]] if isinstance(shard_id, str) else (
            [shard_id] if isinstance(shard_id, int) else list(shard_id))
        gs = {layer.exl3_part_to_group[p] for p in parts}
        if len(gs) != 1:
            raise ValueError(f"exl3rocm: shard {shard_id} spans groups {gs}")
        return gs.pop()

    def _loader(self, layer, kind):
        def load(param, loaded, shard_id=None, *args, **kwargs):
            if kind in ("mul1", "mcg"):  # one codebook for the whole module: no group needed
                val = int(loaded.item())
                prev = layer.exl3_codebook.get(kind)
                if prev is not None and prev != val:
                    raise ValueError(f"exl3rocm: {kind} differs across groups")
                layer.exl3_codebook[kind] = val
                return
            layer.exl3_shard.load(kind, self._group_of(layer, shard_id), loaded)
        return load

    def process_weights_after_loading(self, layer):
        shard = layer.exl3_shard
        sharding.agree_loaded([shard], _tp_group() if shard.tp_size > 1 else None)
        layer.exl3_mul1 = "mul1" in layer.exl3_codebook
        layer.exl3_mcg = "mcg" in layer.exl3_codebook
        if torch.cuda.is_available():
            from .ops import GEMV_MAX_ROWS, RECON_SLICE_N, reserve_weight_buffer, reserve_workspace
            dev = shard.shards[0].trellis.device
            stored = [s.stored_n for s in shard.shards]
            reserve_workspace(dev, shard.local_k, sum(stored), len(stored), GEMV_MAX_ROWS)
            reserve_weight_buffer(dev, shard.local_k * min(max(stored), RECON_SLICE_N))
        for name in ("trellis", "suh", "svh", "mul1", "mcg"):
            if name in layer._parameters:
                del layer._parameters[name]

    def apply(self, layer, x, bias=None):
        y = layer.exl3_shard.forward(x, layer.exl3_mcg, layer.exl3_mul1)
        if y.dtype != x.dtype:
            y = y.to(x.dtype)
        if bias is not None:
            y = y + bias
        return y

    def embedding(self, layer, input_):
        raise NotImplementedError("exl3rocm: quantized input embeddings are not supported")


def _install_kv_hooks():
    """Route vLLM's int4_per_token_head cache write and decode attention to exl3rocm.kv, where the
    running vLLM has the hook points the reference patches (``plugin.py:639-740``: the triton
    attention backend's ``unified_attention`` and ``do_kv_cache_update``, the V2 runner's request
    states).  Silently absent otherwise (vLLM 0.22 has no int4_per_token_head)."""
    try:
        from vllm.v1.attention.backends import triton_attn as ta
        from vllm.v1.kv_cache_interface import KVQuantMode
    except Exception:
        return False
    if getattr(ta, "_exl3_kv_int4", False):
        return True
    from . import kv
    int4 = KVQuantMode.INT4_PER_TOKEN_HEAD
    inner = ta.unified_attention

    def unified_attention(*args, **kw):
        if args or kw.get("kv_quant_mode") != int4 or not kv.supported(kw):
            return inner(*args, **kw)
        return kv.attention(**kw)

    ta.unified_attention = unified_attention
    cls = ta.TritonAttentionImpl
    orig_update = cls.do_kv_cache_update

    def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
        if getattr(self, "_kv_quant_mode", None) != int4:
            return orig_update(self, layer, key, value, kv_cache, slot_mapping)
        key_cache, value_cache = self._pth_key_value_caches(kv_cache)
        kv.reshape_and_cache(key, value, key_cache, value_cache, slot_mapping,
                             k_scale_cache=self._k_scale_cache, v_scale_cache=self._v_scale_cache,
                             layer_name=getattr(layer, "layer_name", None))

    cls.do_kv_cache_update = do_kv_cache_update
    ta._exl3_kv_int4 = True
    return True


def register():
    """vllm.general_plugins entry point (runs in every vLLM process)."""
    from . import ops  # noqa: F401  registers torch.ops.exl3rocm.*
    if os.environ.get("EXL3_KV_INT4", "1") != "0":
        _install_kv_hooks()
    return None
