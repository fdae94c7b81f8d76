"""vLLM out-of-tree quantization plugin "exl3" for B200: the reference's plugin surface
(``vllm_plugin/exl3rocm/plugin.py``), with tensor-parallel weights and this library's KV kernels.

Registered through the ``vllm.general_plugins`` entry point ``exl3rocm = exl3rocm.plugin:register``
(reference ``vllm_plugin/pyproject.toml:13-14``).  What it keeps from the reference's behaviour:

* quant method name ``exl3``; fp16 activations; minimum capability 0 (``plugin.py:82-107``);
* the EXL3 module map comes from the checkpoint's safetensors headers, K = trellis last dim / 16
  (``plugin.py:63-79``);
* fused vLLM modules (qkv_proj, gate_up_proj, ...) hold one group per checkpoint tensor, each with
  its own K, trellis, suh and svh, and run as one ``exl3rocm::linear_groups`` op
  (``plugin.py:236-372``);
* the per-token-head KV caches are routed to this library's write / attention / prefill kernels
  through the Triton attention backend's hook points (``plugin.py:586-740``; see ``KvRouting``).

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
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig, QuantizeMethodBase
from vllm.model_executor.layers.vocab_parallel_embedding import ParallelLMHead, VocabParallelEmbedding
from vllm.model_executor.utils import set_weight_attrs

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
CODEBOOK_SCALARS = ("mul1", "mcg")  # the scalar tensor a checkpoint stores names its codebook


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


def read_checkpoint_embedding(model_dir: str) -> Optional[tuple[int, int]]:
    """(vocab, hidden) of the language model's input embedding when the checkpoint stores it as
    float8_e4m3fn (safetensors dtype ``F8_E4M3``), else None.  A vision tower's embedding does not
    count, and neither do several candidates (reference plugin.py:117-120)."""
    found = []
    for path in sorted(glob.glob(os.path.join(model_dir, "*.safetensors"))):
        with open(path, "rb") as f:
            (hlen,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(hlen))
        for name, meta in header.items():
            if (name != "__metadata__" and name.endswith("embed_tokens.weight") and meta.get("dtype") == "F8_E4M3"
                    and "visual" not in name.split(".")):
                found.append(tuple(meta["shape"]))
    return found[0] if len(found) == 1 else None


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
    """Quant config "exl3".  ``modules`` maps checkpoint module keys to (K, k, n); vLLM fills it
    through maybe_update_config with the checkpoint directory."""

    def __init__(self, codebook: str = "mul1"):
        super().__init__()
        self.codebook = codebook
        self.modules: dict[str, tuple[int, int, int]] = {}
        self.embed_shape: Optional[tuple[int, int]] = None  # (vocab, hidden) of an fp8 input embedding

    @property
    def fp8_embedding(self) -> bool:
        return self.embed_shape is not None

    def __repr__(self):
        widths = sorted({K for K, _, _ in self.modules.values()})
        return f"exl3[{self.codebook}, {len(self.modules)} EXL3 modules, K in {widths}]"

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
        # the module map is read from the checkpoint's own files: a hub id has none yet
        if not os.path.isdir(model_name):
            raise NotImplementedError(f"exl3: {model_name!r} is not a directory; the EXL3 module map is read "
                                      "from the checkpoint's safetensors headers")
        self.modules = read_checkpoint_layout(model_name)
        self.embed_shape = read_checkpoint_embedding(model_name)

    def groups_for(self, prefix: str) -> Optional[list[tuple[str, int, int, int]]]:
        """[(member, K, k, n)] for the checkpoint tensors behind the (possibly fused) vLLM module at
        ``prefix``; None when none of them is EXL3; ValueError when only some are."""
        key = module_key(prefix)
        parent, _, leaf = key.rpartition(".")
        qualify = (lambda m: f"{parent}.{m}") if parent else (lambda m: m)
        members = [qualify(m) for m in FUSED.get(leaf, [leaf])]
        shapes = {m: self.modules[m] for m in members if m in self.modules}
        if not shapes:
            return None
        if len(shapes) != len(members):
            missing = [m for m in members if m not in shapes]
            raise ValueError(f"exl3: fused module {prefix} is only partly EXL3 (no trellis for {missing})")
        return [(m, *shapes[m]) for m in members]

    def get_quant_method(self, layer: torch.nn.Module, prefix: str):
        is_linear = isinstance(layer, LinearBase)
        if not (is_linear or isinstance(layer, ParallelLMHead)):
            # the input embedding stays in the checkpoint's fp8 (reference plugin.py:158-159)
            if (isinstance(layer, VocabParallelEmbedding) and self.fp8_embedding
                    and prefix.endswith("embed_tokens")):
                return Fp8EmbeddingMethod()
            return None
        groups = self.groups_for(prefix)
        if groups is not None:
            return Exl3LinearMethod(self, groups)
        # a plain (unquantised) linear keeps vLLM's method; an lm_head keeps vLLM's default
        return UnquantizedLinearMethod() if is_linear else None


class Fp8EmbeddingMethod(QuantizeMethodBase):
    """The input embedding kept as the checkpoint's float8_e4m3fn table (no scale) and looked up with
    ``exl3rocm::fp8_embedding``: half the memory of an fp16 table (reference plugin.py:215-233).  Under
    tensor parallelism vLLM hands each rank its vocab rows (``output_partition_sizes``) and masks the
    ids outside them."""

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **extra_weight_attrs):
        weight = Parameter(torch.empty(sum(output_partition_sizes), input_size_per_partition,
                                       dtype=torch.float8_e4m3fn), requires_grad=False)
        set_weight_attrs(weight, {"input_dim": 1, "output_dim": 0})
        set_weight_attrs(weight, extra_weight_attrs)
        layer.register_parameter("weight", weight)

    def apply(self, layer, x, bias=None):
        raise NotImplementedError("exl3: the fp8 input embedding is not an output head")

    def embedding(self, layer, input_):
        from . import ops  # noqa: F401  registers torch.ops.exl3rocm.fp8_embedding
        return torch.ops.exl3rocm.fp8_embedding(layer.weight, input_)


def wants_fp8_embedding(quant_config, num_embeddings: int, embedding_dim: int) -> bool:
    """True for a plain input embedding built without a quant config, of exactly the shape of the
    checkpoint's fp8 table, while an exl3 model with such a table is being built."""
    return (isinstance(quant_config, Exl3Config) and quant_config.fp8_embedding
            and (num_embeddings, embedding_dim) == tuple(quant_config.embed_shape))


def _install_fp8_embedding_hook() -> bool:
    """Models build their input embedding as ``VocabParallelEmbedding(vocab, hidden)`` without the
    quant config, so no quantisation method could keep the fp8 table and vLLM would load it as fp16
    (reference plugin.py:405-425).  While vLLM's current config is an exl3 one with an fp8 embedding,
    a plain VocabParallelEmbedding of the table's shape gets that config (and the ``embed_tokens``
    prefix), so that get_quant_method picks Fp8EmbeddingMethod.  Returns whether the hook went in."""
    import inspect
    try:
        from vllm.config import get_current_vllm_config_or_none
    except ImportError:
        return False
    if getattr(VocabParallelEmbedding, "_exl3_fp8_hook", False):
        return False
    orig = VocabParallelEmbedding.__init__
    sig = inspect.signature(orig)

    def __init__(self, *args, **kwargs):
        if type(self) is VocabParallelEmbedding:
            bound = sig.bind(self, *args, **kwargs)
            a = bound.arguments
            cfg = get_current_vllm_config_or_none()
            qc = getattr(cfg, "quant_config", None) if cfg is not None else None
            if a.get("quant_config") is None and wants_fp8_embedding(qc, a["num_embeddings"], a["embedding_dim"]):
                a["quant_config"] = qc
                a["prefix"] = a.get("prefix") or "embed_tokens"
                return orig(*bound.args, **bound.kwargs)
        return orig(self, *args, **kwargs)

    VocabParallelEmbedding.__init__ = __init__
    VocabParallelEmbedding._exl3_fp8_hook = True
    return True


def _speculative() -> bool:
    try:
        from vllm.config import get_current_vllm_config_or_none
        cfg = get_current_vllm_config_or_none()
    except ImportError:
        return False
    return cfg is not None and getattr(cfg, "speculative_config", None) is not None


def prune_draft_head(layer) -> bool:
    """The MTP drafter's pruned lm_head without a copy (reference plugin.py:431-486): the head's columns
    are re-stored as three groups [drafted prefix | middle | drafted tail] (``sharding.draft_bounds``,
    ``EXL3_DRAFT_VOCAB_BLOCKS`` prefix blocks, default 640, plus the last 16).  The target runs all three
    in order, so its logits are unchanged; the drafter runs groups 0 and 2 only.  Applied to an
    unsharded head (TP 1, as the reference); under tensor parallelism the drafter keeps the full head.
    Returns whether the head was split."""
    shard = layer.exl3_shard
    if len(shard.shards) != 1 or shard.tp_size != 1 or shard.shards[0].trimmed:
        return False
    n = shard.shards[0].stored_n
    bounds = sharding.draft_bounds(n, int(os.environ.get("EXL3_DRAFT_VOCAB_BLOCKS", "640")))
    if bounds is None:
        return False
    a, b = bounds
    shard.split_columns([a, b])
    dev = shard.shards[0].trellis.device
    layer.exl3_draft_groups = (0, 2)
    layer.exl3_draft_cols = torch.cat([torch.arange(0, a, device=dev), torch.arange(b, n, device=dev)])
    return True


def draft_logits(lm_head, hidden_states: torch.Tensor) -> torch.Tensor:
    """The drafter's logits over the pruned head: the drafted columns computed, -inf elsewhere."""
    sub = lm_head.exl3_shard.forward_groups(hidden_states, lm_head.exl3_draft_groups, lm_head.exl3_mcg,
                                            lm_head.exl3_mul1)
    logits = sub.new_full((sub.shape[0], lm_head.exl3_shard.shards[-1].c1), float("-inf"))
    logits.index_copy_(1, lm_head.exl3_draft_cols, sub)
    return logits


def _install_draft_logits_patch(cls=None) -> bool:
    """Qwen3.5's MTP drafter computes its logits through the pruned head when the shared lm_head was
    split (reference plugin.py:489-528); otherwise vLLM's own compute_logits runs."""
    if cls is None:
        try:
            from vllm.model_executor.models import qwen3_5_mtp
        except Exception:
            return False
        cls = getattr(qwen3_5_mtp, "Qwen3_5MTP", None)
    if cls is None or getattr(cls, "_exl3_draft_patch", False):
        return False
    orig = cls.compute_logits

    def compute_logits(self, hidden_states, spec_step_idx: int = 0):
        lm = self.lm_head
        if getattr(lm, "exl3_draft_groups", None) is None:
            return orig(self, hidden_states, spec_step_idx)
        logits = draft_logits(lm, hidden_states)
        return logits[:, : self.config.vocab_size].to(hidden_states.dtype)

    cls.compute_logits = compute_logits
    cls._exl3_draft_patch = True
    return True


def parallel_mode(input_size_per_partition: int, input_size: int, output_partition_sizes: list[int],
                  output_size: int) -> str:
    if input_size_per_partition != input_size:
        return "row"
    if sum(output_partition_sizes) != output_size:
        return "column"
    return "replicated"


class _ShardLoader:
    """weight_loader of one registered load target: hands each full checkpoint tensor to this
    rank's shard of the group the vLLM shard id names (or records the codebook scalar)."""

    def __init__(self, layer, kind: str):
        self.layer, self.kind = layer, kind

    def group(self, shard_id) -> int:
        owner = self.layer.exl3_part_to_group
        if shard_id is None:
            if len(self.layer.exl3_shard.groups) > 1:
                raise ValueError("exl3: a fused module got a tensor without a shard id")
            return 0
        if isinstance(shard_id, str):
            parts = (SHARD_IDS[shard_id],)
        elif isinstance(shard_id, int):
            parts = (shard_id,)
        else:
            parts = tuple(shard_id)
        owners = sorted({owner[p] for p in parts})
        if len(owners) > 1:
            raise ValueError(f"exl3: shard id {shard_id} covers groups {owners} of one module")
        return owners[0]

    def __call__(self, param, loaded: torch.Tensor, shard_id=None, *args, **kwargs):
        if self.kind in CODEBOOK_SCALARS:
            seen = self.layer.exl3_codebook.setdefault(self.kind, int(loaded.item()))
            if seen != int(loaded.item()):
                raise ValueError(f"exl3: the groups of one module disagree on {self.kind}")
            return
        self.layer.exl3_shard.load(self.kind, self.group(shard_id), loaded)


class Exl3LinearMethod(LinearMethodBase):
    """Per-group EXL3 storage for one rank.  The registered parameters ``trellis``, ``suh``,
    ``svh`` (and the codebook scalar) are 0-size load targets that vLLM's name mapping resolves to;
    their weight_loader slices each full checkpoint tensor into this rank's shard."""

    def __init__(self, config: Exl3Config, groups, tp: Optional[tuple[int, int]] = None,
                 drafting: Optional[bool] = None):
        self.config = config
        self.groups = groups  # [(member, K, k, n)]
        self.tp = tp          # (size, rank); None = ask vLLM at create_weights
        self.drafting = drafting  # a speculative (MTP) drafter shares this lm_head; None = ask vLLM

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **extra_weight_attrs):
        tp_size, tp_rank = self.tp or _tp()
        partitions = [int(p) for p in output_partition_sizes]
        mode = parallel_mode(input_size_per_partition, input_size, partitions, output_size)
        shard = sharding.module_shard(self.groups, mode, tp_size, tp_rank,
                                      device=torch.cuda.current_device() if torch.cuda.is_available() else "cpu")
        if mode == "row" and shard.local_k != input_size_per_partition:
            raise ValueError(f"exl3: this rank's input slice has {shard.local_k} features, "
                             f"vLLM expects {input_size_per_partition}")
        layer.exl3_shard = shard
        layer.exl3_part_to_group = sharding.partition_owners(partitions, shard.out_sizes)
        layer.exl3_codebook = {}
        targets = ["trellis", "suh", "svh"]
        if self.config.codebook in CODEBOOK_SCALARS:  # only what the checkpoint stores is registered
            targets.append(self.config.codebook)
        layer.exl3_load_targets = tuple(targets)
        if self.drafting is None:
            self.drafting = isinstance(layer, ParallelLMHead) and _speculative()
        for kind in targets:
            target = Parameter(torch.empty(0, dtype=torch.int8), requires_grad=False)
            target.weight_loader = _ShardLoader(layer, kind)
            layer.register_parameter(kind, target)

    def process_weights_after_loading(self, layer):
        shard = layer.exl3_shard
        sharding.agree_loaded([shard], _tp_group() if shard.tp_size > 1 else None)
        layer.exl3_mul1 = "mul1" in layer.exl3_codebook
        layer.exl3_mcg = "mcg" in layer.exl3_codebook
        if torch.cuda.is_available():
            from .ops import GEMV_MAX_ROWS, reserve_workspace
            stored = [s.stored_n for s in shard.shards]
            reserve_workspace(shard.shards[0].trellis.device, shard.local_k, sum(stored), len(stored), GEMV_MAX_ROWS)
        # the load targets have served their purpose; weights live in the shard
        for kind in layer.exl3_load_targets:
            layer._parameters.pop(kind, None)
        if self.drafting and isinstance(layer, ParallelLMHead):
            prune_draft_head(layer)

    def apply(self, layer, x, bias=None):
        y = layer.exl3_shard.forward(x, layer.exl3_mcg, layer.exl3_mul1)
        y = y if y.dtype == x.dtype else y.to(x.dtype)
        return y if bias is None else y + bias

    def embedding(self, layer, input_):
        raise NotImplementedError("exl3: this plugin quantises linears only; the input embedding stays dense")


# ---------------------------------------------------------------------------------------------
# KV cache routing (reference plugin.py:586-740)
# ---------------------------------------------------------------------------------------------
class KvRouting:
    """Sends vLLM's per-token-head KV cache traffic on the Triton attention backend to exl3rocm.kv.

    * cache write (``TritonAttentionImpl.do_kv_cache_update``): int8 -> ``kv.reshape_and_cache_int8``;
      int4 -> ``kv.reshape_and_cache`` with the batch's query_start_loc / seq_lens taken from vLLM's
      per-layer attention context (they locate each request's newest positions for the exact rows);
    * attention (the backend module's ``unified_attention``): decode / speculative verify to
      ``kv.attention_int8`` / ``kv.attention``; prefill chunks of at least ``prefill_min_q`` query
      tokens outside graph capture to ``kv.prefill_int8`` / ``kv.prefill`` (the sequences' blocks
      dequantised once to fp16, then vLLM's own fp16 kernel); calls the kernels do not implement
      (``kv.supported``: ALiBi, sinks, softcap, sliding window, non-fp16 q, ...) stay with vLLM;
    * ``TritonAttentionImpl.forward`` records the running layer's name for the duration of the call
      (the int4 exact rows and the centering means are per layer);
    * request slots (the V2 model runner's ``RequestState``): the slot count at construction, a slot's
      exact rows cleared when a new request takes it, and the batch's row -> slot map before each
      forward (``kv.configure_request_slots`` / ``request_added`` / ``set_batch_slots``).

    vLLM's caches keep each row's fp32 scale inline after it; the kernels get the cache and scale
    views' strides (``kv.cache_layout``), so no cache is copied."""

    def __init__(self, ta, modes, kv, get_context=None):
        self.ta, self.kv, self.get_context = ta, kv, get_context
        self.int8 = modes.get("int8")
        self.int4 = modes.get("int4")
        self.none = modes.get("none")
        self.prefill_min_q = int(os.environ.get("EXL3_PTH_PREFILL_MIN_Q", "32"))
        self.layer: Optional[str] = None
        self.descale: dict = {}

    def _ours(self, mode) -> bool:
        return mode is not None and mode in (self.int8, self.int4)

    @staticmethod
    def _rows(cache: torch.Tensor, row_bytes: int) -> torch.Tensor:
        """The [blocks, block_size, heads, row bytes] view of a vLLM cache half (inline scale cut off)."""
        return cache[..., :row_bytes] if cache.shape[-1] > row_bytes else cache

    def _metadata(self, layer_name):
        if not layer_name or self.get_context is None:
            return None
        try:
            return self.get_context(layer_name)[0]
        except Exception:
            return None

    # -- hooks ------------------------------------------------------------------------------------
    def kv_update(self, orig, impl, layer, key, value, kv_cache, slot_mapping):
        mode = getattr(impl, "_kv_quant_mode", None)
        decoder = getattr(getattr(impl, "attn_type", None), "name", "DECODER") in ("DECODER", "ENCODER_DECODER")
        if not (self._ours(mode) and decoder and key.dtype in (torch.float16, torch.bfloat16)
                and key.shape[-1] == self.kv.HEAD_SIZE):
            return orig(impl, layer, key, value, kv_cache, slot_mapping)
        impl._ensure_scale_caches(kv_cache)
        kc, vc = kv_cache.unbind(1)
        name = getattr(layer, "layer_name", None)
        if mode == self.int8:
            self.kv.reshape_and_cache_int8(key, value, self._rows(kc, 128), self._rows(vc, 128),
                                           slot_mapping, impl._k_scale_cache, impl._v_scale_cache)
            return None
        md = self._metadata(name)
        self.kv.reshape_and_cache(key, value, self._rows(kc, 64), self._rows(vc, 64), slot_mapping,
                                  k_scale_cache=impl._k_scale_cache, v_scale_cache=impl._v_scale_cache,
                                  layer_name=name, query_start_loc=getattr(md, "query_start_loc", None),
                                  seq_lens=getattr(md, "seq_lens", None))
        return None

    def attention(self, orig, *args, **kw):
        mode = kw.get("kv_quant_mode")
        if args or not self._ours(mode):
            return orig(*args, **kw)
        capturing = torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()
        long_prefill = int(kw.get("max_seqlen_q", 1)) >= self.prefill_min_q and not capturing
        if not self.kv.supported(kw, prefill=long_prefill):
            return orig(*args, **kw)
        row = 128 if mode == self.int8 else 64
        kw = dict(kw, k=self._rows(kw["k"], row), v=self._rows(kw["v"], row))
        if long_prefill:
            dense = self._dense_kwargs(kw)
            if mode == self.int8:
                return self.kv.prefill_int8(orig, dense)
            return self.kv.prefill(orig, dense, layer_name=self.layer)
        if mode == self.int8:
            return self.kv.attention_int8(**kw)
        return self.kv.attention(**kw, layer_name=self.layer)

    def _dense_kwargs(self, kw) -> dict:
        """vLLM's unified_attention arguments for the fp16 cache the prefill gathers: no quant mode,
        unit descales (one per sequence and KV head, as vLLM passes for an unquantised cache)."""
        seqs, heads = kw["block_table"].shape[0], kw["k"].shape[2]
        key = (kw["q"].device, heads)
        if key not in self.descale:
            self.descale[key] = torch.ones((1, 1), dtype=torch.float32, device=kw["q"].device)
        unit = self.descale[key].expand(seqs, heads)
        return dict(kw, kv_quant_mode=self.none, k_descale=unit, v_descale=unit)

    def forward(self, orig, impl, layer, *args, **kw):
        outer, self.layer = self.layer, getattr(layer, "layer_name", None)
        try:
            return orig(impl, layer, *args, **kw)
        finally:
            self.layer = outer

    # -- installation -------------------------------------------------------------------------------
    def install(self) -> None:
        ta, cls = self.ta, self.ta.TritonAttentionImpl
        inner_attention, inner_update, inner_forward = ta.unified_attention, cls.do_kv_cache_update, cls.forward
        ta.unified_attention = lambda *a, **kw: self.attention(inner_attention, *a, **kw)
        cls.do_kv_cache_update = lambda impl, layer, k, v, cache, slots: self.kv_update(
            inner_update, impl, layer, k, v, cache, slots)
        cls.forward = lambda impl, layer, *a, **kw: self.forward(inner_forward, impl, layer, *a, **kw)
        ta._exl3_kv_routing = self

    def install_request_slots(self, states, runner) -> bool:
        """Feed the exact-row ring from the V2 model runner (None when that runner is absent)."""
        if states is None or runner is None or getattr(states.RequestState, "_exl3_slots", False):
            return False
        kv, rs_cls, mr_cls = self.kv, states.RequestState, runner.GPUModelRunner
        init, add, prep = rs_cls.__init__, rs_cls.add_request, mr_cls.prepare_inputs

        def state_init(st, *a, **k):
            init(st, *a, **k)
            kv.configure_request_slots(st.max_num_reqs)

        def state_add(st, req_id, *a, **k):
            add(st, req_id, *a, **k)
            kv.request_added(st.req_id_to_index[req_id])

        def prepare(runner_self, *a, **k):
            batch = prep(runner_self, *a, **k)
            kv.set_batch_slots(batch.idx_mapping)
            return batch

        rs_cls.__init__, rs_cls.add_request, mr_cls.prepare_inputs = state_init, state_add, prepare
        rs_cls._exl3_slots = True
        return True


def _install_kv_hooks():
    """Install KvRouting on the running vLLM (once).  int8_per_token_head routes on any vLLM that has
    the mode (0.22 here); int4_per_token_head where vLLM defines it (0.28, the reference's).  Returns
    the routing object, or None when the Triton backend or the quant modes are missing."""
    try:
        from vllm.v1.attention.backends import triton_attn as ta
        from vllm.v1.kv_cache_interface import KVQuantMode
    except Exception:
        return None
    if getattr(ta, "_exl3_kv_routing", None) is not None:
        return ta._exl3_kv_routing
    modes = {"int8": getattr(KVQuantMode, "INT8_PER_TOKEN_HEAD", None),
             "int4": getattr(KVQuantMode, "INT4_PER_TOKEN_HEAD", None), "none": KVQuantMode.NONE}
    if modes["int8"] is None and modes["int4"] is None:
        return None
    try:
        from vllm.model_executor.layers.attention.attention import get_attention_context
    except Exception:
        get_attention_context = None
    from . import kv
    routing = KvRouting(ta, modes, kv, get_attention_context)
    routing.install()
    try:
        from vllm.v1.worker.gpu import model_runner, states
    except Exception:
        model_runner = states = None
    routing.install_request_slots(states, model_runner)
    return routing


def register():
    """vllm.general_plugins entry point (runs in every vLLM process)."""
    from . import ops  # noqa: F401  registers torch.ops.exl3rocm.*
    if os.environ.get("EXL3_FP8_EMBEDDING", "1") != "0":
        _install_fp8_embedding_hook()
    if os.environ.get("EXL3_DRAFT_VOCAB_BLOCKS", "640") != "0":
        _install_draft_logits_patch()
    if os.environ.get("EXL3_KV_ROUTING", "1") != "0":
        _install_kv_hooks()
    return None
