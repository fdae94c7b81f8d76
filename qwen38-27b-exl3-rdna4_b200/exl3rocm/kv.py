"""Paged KV cache (int8 and int4 per-token-head) on libexl3b, drop-in for the reference's
``vllm_plugin/exl3rocm/kv_int4.py`` surface and for vLLM's int8 per-token-head write/attention the
reference runs for ``int8_per_token_head``.

* int4: ``reshape_and_cache`` (kv_int4.py:176-213) rotates, quantises and packs K/V rows and keeps
  exact fp16 rows for each request's first 4 and newest 128 positions; ``attention`` (:516-563)
  runs split-KV decode / verify attention with exact-row substitution and un-rotates the output.
  Request slots follow kv_int4.py:63-89 (``configure_request_slots``, ``request_added``,
  ``set_batch_slots``).  The exact rows are kept per request slot (the reference keeps the sinks
  per physical block; for the sequences' first positions the two agree).
* int8: ``reshape_and_cache_int8`` and ``attention_int8`` take the arguments of vLLM's
  per-token-head write and unified attention.

The RHT sign vector is a fixed seeded +-1 vector (``rht_signs``); writes and reads share it, so the
cache is self-consistent.  There is no CPU path: every call runs on the CUDA library.

Centering (kv_int4.py:120-158): with per-layer K/V channel means (``set_kv_means``, or a file named by
EXL3_KV_MEANS in the reference's ``{layer: {"k": [kv_heads, 128], "v": ...}}`` format), the int4 write
adds the rotated-domain biases -(mean @ diag(s) H) before quantising and the attention adds the value
mean back to its output.  Softmax ignores a per-query constant on the keys, so centering changes only
how tight the 4-bit ranges are.  Without means nothing is centred.
"""
from __future__ import annotations

import os

import numpy as np
import torch

from . import _lib

HEAD_SIZE = 128
SINKS = int(os.environ.get("EXL3_KV_INT4_SINKS", "4"))
TAIL = int(os.environ.get("EXL3_KV_INT4_TAIL", "128"))
MAX_ROWS = 32  # query rows (query tokens x GQA heads) one attention call takes per sequence
RHT_SEED = 0x5EED1234

_signs: dict = {}
_means: dict | None = None  # layer name -> {"k": [kv_heads, 128], "v": ...} (cpu fp32)
_bias: dict = {}            # (layer name, device) -> device biases, or None
_exact: dict = {}
_ws: dict = {}
_req = {"slot": None, "rows": 0}


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _capturing() -> bool:
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


def rht_signs(device, d: int = HEAD_SIZE) -> torch.Tensor:
    """The RHT's +-1 vector (fp32 on the device; built on the CPU once, outside graph capture)."""
    key = (d, str(device))
    if key not in _signs:
        bits = np.random.default_rng(RHT_SEED).integers(0, 2, size=d)
        _signs[key] = torch.from_numpy(np.where(bits == 1, 1.0, -1.0).astype(np.float32)).to(device)
    return _signs[key]


def set_kv_means(means: dict | None) -> None:
    """Per-layer channel means {layer_name: {"k": [kv_heads, 128], "v": [kv_heads, 128]}} for the int4
    centering; None clears them (and the biases derived from them)."""
    global _means
    _means = {name: {"k": torch.as_tensor(m["k"], dtype=torch.float32).cpu(),
                     "v": torch.as_tensor(m["v"], dtype=torch.float32).cpu()} for name, m in (means or {}).items()}
    _bias.clear()


def _load_means() -> dict:
    """The means set by set_kv_means, else those of the file EXL3_KV_MEANS names (unset or "0": none)."""
    global _means
    if _means is None:
        path = os.environ.get("EXL3_KV_MEANS", "0")
        set_kv_means(torch.load(path, map_location="cpu") if path != "0" and os.path.exists(path) else {})
    return _means


def layer_bias(name, kv_heads: int, device, d: int = HEAD_SIZE):
    """The layer's centering terms on the device: {"k", "v"}: rotated-domain write biases
    -(mean @ diag(s) H) fp32 [kv_heads, d]; "v_mean": the value mean [kv_heads, d] the attention adds
    back.  None when the layer has no means of this shape.  The first call per layer must be eager."""
    if not name:
        return None
    key = (name, str(device))
    if key not in _bias:
        m = _load_means().get(name)
        if m is None or tuple(m["k"].shape) != (kv_heads, d):
            _bias[key] = None
        else:
            if _capturing():
                raise RuntimeError("exl3rocm.kv: first use of a layer's means during graph capture")
            fwd = rht_signs("cpu", d)[:, None] * _sylvester(d)  # x @ fwd == H (x * s), the write's rotation
            _bias[key] = {"k": (-(m["k"] @ fwd)).to(device), "v": (-(m["v"] @ fwd)).to(device),
                          "v_mean": m["v"].to(device).contiguous()}
    return _bias[key]


def _sylvester(d: int) -> torch.Tensor:
    """Natural-order Sylvester Hadamard matrix of +-1 (H[i, j] = (-1)^popcount(i & j))."""
    h = torch.ones((1, 1), dtype=torch.float32)
    while h.shape[0] < d:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h


# ---------------------------------------------------------------------------------------------
# request slots and exact rows (kv_int4.py:63-118)
# ---------------------------------------------------------------------------------------------
def configure_request_slots(max_reqs: int) -> None:
    """The model runner keeps per-request state in max_reqs fixed slots; slot max_reqs is scratch."""
    _req["rows"] = max_reqs + 1


def _slot_buffer(device):
    if _req["slot"] is None and _req["rows"] > 0:
        _req["slot"] = torch.full((1024,), _req["rows"] - 1, dtype=torch.int32, device=device)
    return _req["slot"]


def set_batch_slots(idx_mapping: torch.Tensor) -> None:
    """batch row -> request slot, in the persistent buffer the captured kernels read."""
    buf = _slot_buffer(idx_mapping.device)
    if buf is None:
        return
    n = idx_mapping.shape[0]
    buf[:n].copy_(idx_mapping)
    buf[n:].fill_(_req["rows"] - 1)


def request_added(idx: int) -> None:
    """A new request took slot idx: forget the previous request's exact rows (tags are positions)."""
    for b in _exact.values():
        b["tag"][idx].fill_(-1)


def exact_buffers(name, heads: int, device, d: int = HEAD_SIZE):
    """Exact fp16 rows of layer `name`: [slots, SINKS + TAIL, heads, d] for K and V plus int32 tags
    [slots, SINKS + TAIL] (-1 = empty).  Allocated on first eager use; None without request slots,
    with SINKS = TAIL = 0, or when first seen during graph capture."""
    if not name or _req["rows"] <= 0 or (SINKS <= 0 and TAIL <= 0):
        return None
    if name not in _exact:
        if _capturing():
            return None
        rows = _req["rows"]
        _exact[name] = {
            "k": torch.zeros((rows, SINKS + TAIL, heads, d), dtype=torch.float16, device=device),
            "v": torch.zeros((rows, SINKS + TAIL, heads, d), dtype=torch.float16, device=device),
            "tag": torch.full((rows, SINKS + TAIL), -1, dtype=torch.int32, device=device)}
    return _exact[name]


def _workspace(device, nbytes: int) -> torch.Tensor:
    key = (torch.device(device).index, _stream(device))
    ws = _ws.get(key)
    if ws is None or ws.numel() < nbytes:
        if _capturing():
            raise RuntimeError("exl3rocm.kv: attention workspace too small during graph capture; "
                               "call reserve_attention_workspace() before capturing")
        _ws[key] = ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
    return ws


def reserve_attention_workspace(device, num_tokens: int, num_q_heads: int, num_seqs: int, num_kv_heads: int,
                                max_seq_len: int) -> None:
    _workspace(device, int(_lib.lib().exl3b_kv_attn_workspace_bytes(num_tokens, num_q_heads, num_seqs,
                                                                     num_kv_heads, max_seq_len)))


def cache_layout(cache: torch.Tensor, scale: torch.Tensor, other: torch.Tensor | None = None,
                 other_scale: torch.Tensor | None = None):
    """The exl3b_kv_layout of a [blocks, block_size, heads, row] cache view and its [blocks, block_size,
    heads] fp32 scale view, any strides with a unit last cache stride: dense caches and vLLM's
    per-token-head caches (scales inline, K and V interleaved per block) alike.  `other` / `other_scale`
    (the V side) must share the strides."""
    assert cache.dim() == 4 and cache.stride(-1) == 1 and scale.dim() == 3 and scale.dtype == torch.float32
    if other is not None:
        assert other.stride() == cache.stride() and other_scale.stride() == scale.stride(), "K and V layouts differ"
    e = cache.element_size()
    return _lib.ctypes.byref(_lib.KvLayout(cache.stride(0) * e, cache.stride(1) * e, cache.stride(2) * e,
                                           scale.stride(0), scale.stride(1), scale.stride(2)))


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return 0
    if t.dtype == torch.bfloat16:
        return 1
    raise TypeError(f"exl3rocm.kv: key/value must be fp16 or bf16, got {t.dtype}")


def _check_rows(t: torch.Tensor, name: str):
    assert t.dim() == 3 and t.shape[-1] == HEAD_SIZE and t.stride(-1) == 1, f"{name}: [tokens, heads, 128]"


# ---------------------------------------------------------------------------------------------
# writes
# ---------------------------------------------------------------------------------------------
def reshape_and_cache_int8(key, value, key_cache, value_cache, slot_mapping, k_scale_cache, v_scale_cache):
    """vLLM int8_per_token_head write (triton_reshape_and_cache_flash.py:139-238)."""
    _check_rows(key, "key")
    _check_rows(value, "value")
    n = min(key.shape[0], slot_mapping.shape[0])
    if n == 0:
        return
    lay = cache_layout(key_cache, k_scale_cache, value_cache, v_scale_cache)
    slots = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
    _lib.call("exl3b_kv_int8_write", key.data_ptr(), value.data_ptr(), _dtype_code(key), n, key.shape[1],
              HEAD_SIZE, key.stride(0), key.stride(1), value.stride(0), value.stride(1), key_cache.data_ptr(),
              value_cache.data_ptr(), k_scale_cache.data_ptr(), v_scale_cache.data_ptr(), slots.data_ptr(),
              key_cache.shape[1], lay, _stream(key.device))


def rope_and_cache_int8(qkv, q_out, num_q_heads, num_kv_heads, positions, cos_sin, key_cache, value_cache,
                        slot_mapping, k_scale_cache, v_scale_cache):
    """Neox RoPE of q (into q_out) and k, then the int8 write of k and v, in one launch: qkv rows
    [T, (q + 2 kv) heads x 128] fp16, positions int64 [T], cos_sin fp32 [max_pos][128]
    (exl3b_kv_int8_write_rope; byte-identical to glue.rope_neox + reshape_and_cache_int8)."""
    assert qkv.dtype == q_out.dtype == torch.float16 and qkv.stride(-1) == 1 and q_out.stride(-1) == 1
    assert positions.dtype == torch.int64 and cos_sin.dtype == torch.float32
    n = min(qkv.shape[0], slot_mapping.shape[0])
    if n == 0:
        return
    lay = cache_layout(key_cache, k_scale_cache, value_cache, v_scale_cache)
    slots = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
    _lib.call("exl3b_kv_int8_write_rope", qkv.data_ptr(), qkv.stride(0), q_out.data_ptr(), q_out.stride(0), n,
              num_q_heads, num_kv_heads, positions.data_ptr(), cos_sin.data_ptr(), cos_sin.shape[0],
              key_cache.data_ptr(), value_cache.data_ptr(), k_scale_cache.data_ptr(), v_scale_cache.data_ptr(),
              slots.data_ptr(), key_cache.shape[1], lay, _stream(qkv.device))


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, *, k_scale_cache, v_scale_cache,
                      layer_name=None, query_start_loc=None, seq_lens=None):
    """int4 write (kv_int4.py:176-213): rotate, clip-search quantise, pack; exact rows when the layer
    has them and the batch metadata (query_start_loc, seq_lens) is given."""
    _check_rows(key, "key")
    _check_rows(value, "value")
    n = min(key.shape[0], slot_mapping.shape[0])
    if n == 0:
        return
    heads = key.shape[1]
    slots = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
    ex = exact_buffers(layer_name, heads, key.device) if query_start_loc is not None else None
    num_seqs = int(seq_lens.shape[0]) if (ex is not None and seq_lens is not None) else 0
    use_ex = ex is not None and num_seqs > 0
    qsl = query_start_loc.to(torch.int32) if use_ex and query_start_loc.dtype != torch.int32 else query_start_loc
    sl = seq_lens.to(torch.int32) if use_ex and seq_lens.dtype != torch.int32 else seq_lens
    bias = layer_bias(layer_name, heads, key.device)
    lay = cache_layout(key_cache, k_scale_cache, value_cache, v_scale_cache)
    _lib.call("exl3b_kv_int4_write", key.data_ptr(), value.data_ptr(), _dtype_code(key), n, heads, HEAD_SIZE,
              key.stride(0), key.stride(1), value.stride(0), value.stride(1), key_cache.data_ptr(),
              value_cache.data_ptr(), k_scale_cache.data_ptr(), v_scale_cache.data_ptr(), slots.data_ptr(),
              key_cache.shape[1], rht_signs(key.device).data_ptr(),
              bias["k"].data_ptr() if bias else None, bias["v"].data_ptr() if bias else None,
              qsl.data_ptr() if use_ex else None, sl.data_ptr() if use_ex else None,
              _req["slot"].data_ptr() if use_ex else None, num_seqs,
              ex["k"].data_ptr() if use_ex else None, ex["v"].data_ptr() if use_ex else None,
              ex["tag"].data_ptr() if use_ex else None, lay, _stream(key.device))


# ---------------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------------
def supported(kw, prefill: bool = False) -> bool:
    """Features the kernels leave out (kv_int4.py:499-504): the caller falls back otherwise.  The
    split-KV decode / verify kernels also take at most MAX_ROWS query rows per sequence and KV head;
    the prefill route (prefill=True: gather, then an fp16 kernel) takes any query length."""
    q = kw["q"]
    return (kw.get("alibi_slopes") is None and kw.get("sinks") is None and not kw.get("softcap")
            and kw.get("qq_bias") is None and kw.get("mm_prefix_range") is None and kw.get("output_scale") is None
            and tuple(kw.get("window_size", (-1, -1)))[0] < 0 and kw.get("causal", True) is True
            and q.dtype == torch.float16 and q.shape[-1] == HEAD_SIZE
            and (prefill or int(kw.get("max_seqlen_q", 1)) * (q.shape[1] // kw["k"].shape[2]) <= MAX_ROWS))


def _attn(kind, q, k, v, out, cu_seqlens_q, max_seqlen_q, seqused_k, block_table, softmax_scale,
          k_scale_cache, v_scale_cache, max_seqlen_k, layer_name):
    T, hq, d = q.shape
    hkv = k.shape[2]
    assert d == HEAD_SIZE and q.is_contiguous() and out.is_contiguous() and q.dtype == torch.float16
    lay = cache_layout(k, k_scale_cache, v, v_scale_cache)
    num_seqs = seqused_k.shape[0]
    max_k = int(max_seqlen_k) if max_seqlen_k is not None else int(block_table.shape[1] * k.shape[1])
    nbytes = int(_lib.lib().exl3b_kv_attn_workspace_bytes(T, hq, num_seqs, hkv, max_k))
    ws = _workspace(q.device, nbytes)
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    sl = seqused_k if seqused_k.dtype == torch.int32 else seqused_k.to(torch.int32)
    qsl = cu_seqlens_q if cu_seqlens_q.dtype == torch.int32 else cu_seqlens_q.to(torch.int32)
    common = (q.data_ptr(), out.data_ptr(), T, hq, hkv, d, k.data_ptr(), v.data_ptr(), k_scale_cache.data_ptr(),
              v_scale_cache.data_ptr(), k.shape[1], bt.data_ptr(), bt.stride(0), sl.data_ptr(), qsl.data_ptr(),
              num_seqs, int(max_seqlen_q), max_k, float(softmax_scale))
    if kind == 8:
        _lib.call("exl3b_kv_int8_attn", *common, ws.data_ptr(), ws.numel(), lay, _stream(q.device))
        return
    ex = _exact.get(layer_name) if layer_name else None
    use_ex = ex is not None and _req["slot"] is not None
    bias = layer_bias(layer_name, hkv, q.device)
    _lib.call("exl3b_kv_int4_attn", *common, rht_signs(q.device).data_ptr(),
              ex["k"].data_ptr() if use_ex else None, ex["v"].data_ptr() if use_ex else None,
              ex["tag"].data_ptr() if use_ex else None, _req["slot"].data_ptr() if use_ex else None,
              bias["v_mean"].data_ptr() if bias else None, ws.data_ptr(), ws.numel(), lay, _stream(q.device))


def attention(*, q, k, v, out, cu_seqlens_q, max_seqlen_q, seqused_k, block_table, softmax_scale,
              k_scale_cache, v_scale_cache, max_seqlen_k=None, layer_name=None, **_):
    """int4 paged decode / verify attention (kv_int4.py:516-563); writes the un-rotated result to out."""
    _attn(4, q, k, v, out, cu_seqlens_q, max_seqlen_q, seqused_k, block_table, softmax_scale, k_scale_cache,
          v_scale_cache, max_seqlen_k, layer_name)


def attention_int8(*, q, k, v, out, cu_seqlens_q, max_seqlen_q, seqused_k, block_table, softmax_scale,
                   k_scale_cache, v_scale_cache, max_seqlen_k=None, **_):
    """int8 per-token-head paged decode / verify attention (vLLM unified attention, 3D split)."""
    _attn(8, q, k, v, out, cu_seqlens_q, max_seqlen_q, seqused_k, block_table, softmax_scale, k_scale_cache,
          v_scale_cache, max_seqlen_k, None)


# ---------------------------------------------------------------------------------------------
# prefill over the quantised caches (reference kv_dequant.py:42-152, kv_int4.py:566-621,
# plugin.py:586-636): gather + dequantise the blocks the batch uses into an fp16 buffer, then an
# fp16 paged attention kernel over it (vLLM's, handed in as `orig`, or torch SDPA without one)
# ---------------------------------------------------------------------------------------------
_gather_bufs: dict = {}


def _gather_buffer(tag, device, n, bs, heads) -> torch.Tensor:
    """Persistent fp16 buffer [>= n][bs][heads][128] (grows, never shrinks: repeated prefill chunks
    with growing context reuse it instead of ratcheting the caching allocator)."""
    key = (tag, str(device), bs, heads)
    buf = _gather_bufs.get(key)
    if buf is None or buf.shape[0] < n:
        grow = max(n, int((buf.shape[0] if buf is not None else 0) * 1.25) + 1)
        buf = torch.empty((grow, bs, heads, HEAD_SIZE), dtype=torch.float16, device=device)
        _gather_bufs[key] = buf
    return buf[:n]


def gather_dequant_int8(cache, scale, blocks, tag="k"):
    """int8 cache rows of `blocks` -> fp16 [n, bs, heads, 128] = q * scale (kv_dequant.py:131-152)."""
    bs, heads = cache.shape[1], cache.shape[2]
    ids = blocks.to(torch.int32).contiguous()
    out = _gather_buffer(tag, cache.device, ids.numel(), bs, heads)
    _lib.call("exl3b_kv_int8_gather", cache.data_ptr(), scale.data_ptr(), bs, heads, HEAD_SIZE, ids.data_ptr(),
              ids.numel(), out.data_ptr(), cache_layout(cache, scale), _stream(cache.device))
    return out


def gather_dequant_int4(cache, scale, blocks, nb, tag="k", exact=None, seq_lens=None):
    """int4 cache rows -> fp16 [n, bs, heads, 128] in the orthonormal rotated domain; with `exact`
    (the layer's exact rows for this side: (rows, tags)) the sequences' exact positions replace the
    quantised ones (kv_dequant.py:80-123 + kv_int4.py:566-594)."""
    bs, heads = cache.shape[1], cache.shape[2]
    ids = blocks.to(torch.int32).contiguous()
    out = _gather_buffer(tag, cache.device, ids.numel(), bs, heads)
    use_ex = exact is not None and seq_lens is not None and _req["slot"] is not None
    sl = seq_lens.to(torch.int32).contiguous() if use_ex else None
    _lib.call("exl3b_kv_int4_gather", cache.data_ptr(), scale.data_ptr(), bs, heads, HEAD_SIZE, ids.data_ptr(),
              ids.numel(), nb, out.data_ptr(), exact[0].data_ptr() if use_ex else None,
              exact[1].data_ptr() if use_ex else None, _req["slot"].data_ptr() if use_ex else None,
              sl.data_ptr() if use_ex else None, cache_layout(cache, scale), _stream(cache.device))
    return out


def _sdpa_paged(q, kd, vd, cu_seqlens_q, seqused_k, nb, softmax_scale, out):
    """Causal GQA attention of each sequence's queries (the last q_len positions) over its nb gathered
    blocks, with torch's scaled_dot_product_attention (fp16 in, fp32 softmax)."""
    qsl = cu_seqlens_q.tolist()
    lens = seqused_k.tolist()
    bs = kd.shape[1]
    for s, L in enumerate(lens):
        q0, q1 = qsl[s], qsl[s + 1]
        if q1 <= q0:
            continue
        ql = q1 - q0
        k = kd[s * nb:(s + 1) * nb].reshape(nb * bs, kd.shape[2], HEAD_SIZE)[:L]
        v = vd[s * nb:(s + 1) * nb].reshape(nb * bs, vd.shape[2], HEAD_SIZE)[:L]
        # query i sits at position L - ql + i and sees keys 0 .. L - ql + i: for a whole prompt (ql == L)
        # that is the plain causal mask, which keeps SDPA on its fused kernels; a chunk after cached
        # context needs the shifted mask
        if ql == L:
            mask, causal = None, True
        else:
            mask = torch.arange(L, device=q.device)[None, :] <= (L - ql + torch.arange(ql, device=q.device))[:, None]
            causal = False
        # SDPA's fused kernels take 4-d [batch, heads, len, dim] inputs with equal head counts (3-d
        # inputs ran its unfused fp32 path: 59 ms per layer for an 8192-token prompt): the KV heads
        # are repeated for their query heads
        G = q.shape[1] // k.shape[1]
        if G > 1:
            k, v = k.repeat_interleave(G, dim=1), v.repeat_interleave(G, dim=1)
        o = torch.nn.functional.scaled_dot_product_attention(
            q[q0:q1].transpose(0, 1).unsqueeze(0), k.transpose(0, 1).unsqueeze(0), v.transpose(0, 1).unsqueeze(0),
            attn_mask=mask, is_causal=causal, scale=softmax_scale)
        out[q0:q1] = o[0].transpose(0, 1).to(out.dtype)


def prefill(orig=None, kw=None, layer_name=None):
    """int4 long prefill chunk (kv_int4.py:596-621): dequantise the sequences' blocks to fp16 in the
    orthonormal rotated domain (exact rows overlaid), attend with an orthonormally rotated q, then
    un-rotate the output.  q.k and p.v are unchanged by the rotation."""
    q, k, v, bt, out = kw["q"], kw["k"], kw["v"], kw["block_table"], kw["out"]
    bs = k.shape[1]
    nb = (int(kw["max_seqlen_k"]) + bs - 1) // bs
    flat = bt[:, :nb].reshape(-1)
    ex = _exact.get(layer_name) if layer_name else None
    kd = gather_dequant_int4(k, kw["k_scale_cache"], flat, nb, "k", (ex["k"], ex["tag"]) if ex else None,
                             kw["seqused_k"])
    vd = gather_dequant_int4(v, kw["v_scale_cache"], flat, nb, "v", (ex["v"], ex["tag"]) if ex else None,
                             kw["seqused_k"])
    s16 = rht_signs(q.device).to(torch.float16)
    qr = torch.empty_like(q)
    _lib.call("exl3b_had128", q.data_ptr(), HEAD_SIZE, qr.data_ptr(), HEAD_SIZE, q.numel() // HEAD_SIZE, HEAD_SIZE,
              s16.data_ptr(), None, 1.0, _stream(q.device))  # H (q * s) / sqrt(128)
    rot = torch.empty_like(q)
    if orig is not None:
        new_bt = torch.arange(flat.numel(), device=bt.device, dtype=bt.dtype).view(bt.shape[0], nb)
        orig(**dict(kw, q=qr, k=kd, v=vd, out=rot, block_table=new_bt, k_scale_cache=None, v_scale_cache=None))
    else:
        _sdpa_paged(qr, kd, vd, kw["cu_seqlens_q"], kw["seqused_k"], nb, kw["softmax_scale"], rot)
    _lib.call("exl3b_had128", rot.data_ptr(), HEAD_SIZE, out.data_ptr(), HEAD_SIZE, q.numel() // HEAD_SIZE,
              HEAD_SIZE, None, s16.data_ptr(), 1.0, _stream(q.device))  # s * H rot / sqrt(128)
    bias = layer_bias(layer_name, k.shape[2], q.device)
    if bias is not None:  # the centering's value mean (kv_int4.py:621), here after the fp16 un-rotation
        g = q.shape[1] // k.shape[2]
        out.add_(bias["v_mean"].repeat_interleave(g, dim=0).to(out.dtype))


def prefill_int8(orig=None, kw=None):
    """int8 long prefill chunk (plugin.py:586-636): dequantise the sequences' blocks to fp16, attend."""
    q, k, v, bt, out = kw["q"], kw["k"], kw["v"], kw["block_table"], kw["out"]
    bs = k.shape[1]
    nb = (int(kw["max_seqlen_k"]) + bs - 1) // bs
    flat = bt[:, :nb].reshape(-1)
    kd = gather_dequant_int8(k, kw["k_scale_cache"], flat, "k")
    vd = gather_dequant_int8(v, kw["v_scale_cache"], flat, "v")
    if orig is not None:
        new_bt = torch.arange(flat.numel(), device=bt.device, dtype=bt.dtype).view(bt.shape[0], nb)
        orig(**dict(kw, k=kd, v=vd, block_table=new_bt, k_scale_cache=None, v_scale_cache=None))
    else:
        _sdpa_paged(q, kd, vd, kw["cu_seqlens_q"], kw["seqused_k"], nb, kw["softmax_scale"], out)
