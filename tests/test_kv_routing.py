"""KvRouting (exl3rocm.plugin) against a stand-in of vLLM's Triton attention backend, on the CPU.

Every hook of the reference's KV installation (vllm_plugin/exl3rocm/plugin.py:586-740) must forward
what the kernels need: the cache write its cache halves (inline scale cut off), the scale views and,
for int4, the batch's query_start_loc / seq_lens from vLLM's per-layer attention context and the
running layer's name; attention its arguments (decode / verify to the split-KV kernels, long prefill
chunks to the gather + fp16 route with vLLM's unquantised mode and unit descales, anything else to
vLLM); the request-slot hooks the V2 runner's slot count, new requests and the batch's slot map.
"""
from __future__ import annotations

import types

import pytest
import torch

plugin = pytest.importorskip("exl3rocm.plugin", reason="vLLM not importable")


class Mode:
    NONE, INT8, INT4, FP8 = "none", "int8_per_token_head", "int4_per_token_head", "fp8"


def fake_backend():
    calls = []

    def unified_attention(*args, **kw):
        calls.append(("vllm_attention", kw))

    class TritonAttentionImpl:
        def __init__(self, mode, attn_type="DECODER"):
            self._kv_quant_mode = mode
            self.attn_type = types.SimpleNamespace(name=attn_type)
            self._k_scale_cache = self._v_scale_cache = None

        def _ensure_scale_caches(self, kv_cache):
            if self._k_scale_cache is None:
                nb, _, bs, h, _ = kv_cache.shape
                self._k_scale_cache = torch.zeros(nb, bs, h)
                self._v_scale_cache = torch.zeros(nb, bs, h)

        def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
            calls.append(("vllm_update", None))

        def forward(self, layer, query, *rest, **kw):
            calls.append(("vllm_forward", routing_of[0].layer))
            return "out"

    ta = types.SimpleNamespace(unified_attention=unified_attention, TritonAttentionImpl=TritonAttentionImpl)
    routing_of = []
    return ta, calls, routing_of


class FakeKv:
    HEAD_SIZE = 128

    def __init__(self):
        self.calls = []

    def supported(self, kw, prefill=False):
        return kw.get("alibi_slopes") is None and kw["q"].dtype == torch.float16

    def __getattr__(self, name):
        if name in ("reshape_and_cache_int8", "reshape_and_cache", "attention_int8", "attention", "prefill_int8",
                    "prefill", "configure_request_slots", "request_added", "set_batch_slots"):
            return lambda *a, **k: self.calls.append((name, a, k))
        raise AttributeError(name)


def install(get_context=None):
    ta, calls, routing_of = fake_backend()
    kv = FakeKv()
    r = plugin.KvRouting(ta, {"int8": Mode.INT8, "int4": Mode.INT4, "none": Mode.NONE}, kv, get_context)
    r.install()
    routing_of.append(r)
    return ta, calls, kv, r


def cache(row):
    return torch.zeros(6, 2, 16, 2, row + 4, dtype=torch.int8)  # vLLM: [blocks, 2, bs, heads, row + scale]


def test_int8_write_routes_with_the_scale_cut_off():
    ta, calls, kv, _ = install()
    impl = ta.TritonAttentionImpl(Mode.INT8)
    layer = types.SimpleNamespace(layer_name="model.layers.0.self_attn.attn")
    key = torch.zeros(3, 2, 128, dtype=torch.float16)
    slots = torch.arange(3)
    impl.do_kv_cache_update(layer, key, key, cache(128), slots)
    (name, args, _), = kv.calls
    assert name == "reshape_and_cache_int8"
    kc, vc = args[2], args[3]
    assert kc.shape == (6, 16, 2, 128) and kc.stride() == (2 * 16 * 2 * 132, 2 * 132, 132, 1)
    assert args[4] is slots and args[5] is impl._k_scale_cache and args[6] is impl._v_scale_cache
    assert calls == []


def test_int4_write_takes_batch_metadata_and_layer_name():
    md = types.SimpleNamespace(query_start_loc=torch.tensor([0, 3]), seq_lens=torch.tensor([40]))
    seen = []
    ta, calls, kv, _ = install(lambda name: (seen.append(name) or md, None, None, None))
    impl = ta.TritonAttentionImpl(Mode.INT4)
    layer = types.SimpleNamespace(layer_name="model.layers.5.self_attn.attn")
    key = torch.zeros(3, 2, 128, dtype=torch.float16)
    impl.do_kv_cache_update(layer, key, key, cache(64), torch.arange(3))
    (name, args, kw), = kv.calls
    assert name == "reshape_and_cache" and args[2].shape == (6, 16, 2, 64)
    assert kw["layer_name"] == layer.layer_name and seen == [layer.layer_name]
    assert kw["query_start_loc"] is md.query_start_loc and kw["seq_lens"] is md.seq_lens


def test_other_modes_and_encoder_layers_stay_with_vllm():
    ta, calls, kv, _ = install()
    key = torch.zeros(3, 2, 128, dtype=torch.float16)
    ta.TritonAttentionImpl(Mode.FP8).do_kv_cache_update(None, key, key, cache(128), torch.arange(3))
    ta.TritonAttentionImpl(Mode.INT8, "ENCODER_ONLY").do_kv_cache_update(None, key, key, cache(128), torch.arange(3))
    assert [c[0] for c in calls] == ["vllm_update", "vllm_update"] and kv.calls == []


def attn_kw(mode, q_len, row=128, **extra):
    c = cache(row).unbind(1)
    q = torch.zeros(q_len, 10, 128, dtype=torch.float16)
    return dict(q=q, k=c[0], v=c[1], out=torch.empty_like(q), cu_seqlens_q=torch.tensor([0, q_len]),
                max_seqlen_q=q_len, seqused_k=torch.tensor([90]), max_seqlen_k=90, softmax_scale=0.1,
                block_table=torch.zeros(1, 6, dtype=torch.int32), kv_quant_mode=mode,
                k_scale_cache=torch.zeros(6, 16, 2), v_scale_cache=torch.zeros(6, 16, 2), **extra)


def test_attention_routing():
    ta, calls, kv, r = install()
    ta.unified_attention(**attn_kw(Mode.INT8, 1))
    ta.unified_attention(**attn_kw(Mode.INT8, 4))
    ta.unified_attention(**attn_kw(Mode.INT8, 64))
    ta.unified_attention(**attn_kw(Mode.INT4, 1, row=64))
    ta.unified_attention(**attn_kw(Mode.INT8, 1, alibi_slopes=torch.ones(10)))  # unsupported feature
    ta.unified_attention(**attn_kw(Mode.NONE, 1))
    names = [c[0] for c in kv.calls]
    assert names == ["attention_int8", "attention_int8", "prefill_int8", "attention"]
    assert [c[0] for c in calls] == ["vllm_attention", "vllm_attention"]
    assert kv.calls[0][2]["k"].shape == (6, 16, 2, 128) and kv.calls[3][2]["k"].shape == (6, 16, 2, 64)
    orig, dense = kv.calls[2][1]
    assert dense["kv_quant_mode"] == Mode.NONE and dense["k_descale"].shape == (1, 2)
    assert float(dense["v_descale"].min()) == 1.0


def test_forward_records_the_running_layer():
    ta, calls, kv, r = install()
    impl = ta.TritonAttentionImpl(Mode.INT4)
    assert impl.forward(types.SimpleNamespace(layer_name="L7"), None) == "out"
    assert calls == [("vllm_forward", "L7")] and r.layer is None


def test_request_slot_hooks():
    ta, calls, kv, r = install()

    class RequestState:
        def __init__(self, max_num_reqs):
            self.max_num_reqs, self.req_id_to_index = max_num_reqs, {}

        def add_request(self, req_id, *a):
            self.req_id_to_index[req_id] = len(self.req_id_to_index)

    class GPUModelRunner:
        def prepare_inputs(self):
            return types.SimpleNamespace(idx_mapping=torch.tensor([1, 0], dtype=torch.int32))

    states = types.SimpleNamespace(RequestState=RequestState)
    runner = types.SimpleNamespace(GPUModelRunner=GPUModelRunner)
    assert r.install_request_slots(states, runner)
    st = RequestState(8)
    st.add_request("a")
    st.add_request("b")
    GPUModelRunner().prepare_inputs()
    names = [(c[0], c[1]) for c in kv.calls]
    assert names[0] == ("configure_request_slots", (8,))
    assert names[1] == ("request_added", (0,)) and names[2] == ("request_added", (1,))
    assert names[3][0] == "set_batch_slots" and names[3][1][0].tolist() == [1, 0]
    assert not r.install_request_slots(states, runner)  # once only
