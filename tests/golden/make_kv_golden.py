"""Generate the int8 / int4 KV-cache golden vectors from the reference's own kernels.

Run once, in a container where the reference checkout and vLLM are present (no GPU needed):

    python tests/golden/make_kv_golden.py <path to a Luke458/qwen38-27b-exl3-rdna4 checkout>

The reference's KV paths are Triton kernels.  This script runs them unmodified under Triton's CPU
interpreter (TRITON_INTERPRET=1) on seeded inputs and writes ``tests/golden/kv_golden.npz``:

* int8 per-token-head, the cache the reference serves with ``--kv-cache-dtype int8_per_token_head``:
  vLLM's own ``triton_reshape_and_cache_flash_per_token_head_quant`` (the write) and
  ``unified_attention`` with ``KVQuantMode.INT8_PER_TOKEN_HEAD`` (decode through the split-KV "3D"
  kernel plus ``reduce_segments``, and a 4-token verify through the 2D kernel), vLLM 0.22 as
  installed in the image (vllm/v1/attention/ops/triton_reshape_and_cache_flash.py:139-317,
  triton_unified_attention.py:179-1060).
* int4 per-token-head: the reference's ``vllm_plugin/exl3rocm/kv_int4.py`` imported by path —
  ``reshape_and_cache`` (:176-213, rotation + clip-search quantiser + exact sink / tail rows) and
  ``attention`` (:516-563, split-KV decode and verify, un-rotation) — for one layer without and one
  with calibrated-style channel means (the centering of :120-158 and the value mean added back, :563).

Two substitutions, both outside the reference's algorithm:
* the RHT sign vector: kv_int4.rht_matrices takes it from vLLM 0.28's ``_get_rht_signs``, which vLLM
  0.22 lacks; the script fills kv_int4's matrix cache with this repository's seeded sign vector
  (exl3rocm.kv.RHT_SEED) and the natural-order Sylvester H128 exactly as rht_matrices builds them;
* the per-layer means come from a seeded generator instead of the packaged kv_means.pt.

The tests never need the reference or vLLM at run time: they read the committed .npz.
"""
from __future__ import annotations

import importlib.util
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "kv_golden.npz")

RHT_SEED = 0x5EED1234  # exl3rocm.kv.RHT_SEED
HKV, HQ, D, BS = 2, 10, 128, 16
SEQ_LENS = (45, 300)  # ragged; the second is longer than the 128-row tail ring
SEED = 20261202


def rht_signs(d: int = D) -> np.ndarray:
    bits = np.random.default_rng(RHT_SEED).integers(0, 2, size=d)
    return np.where(bits == 1, 1.0, -1.0).astype(np.float32)


def sylvester(d: int) -> np.ndarray:
    i = np.arange(d)
    pc = np.vectorize(lambda v: bin(int(v)).count("1"))(i[:, None] & i[None, :])
    return np.where(pc % 2 == 1, -1.0, 1.0).astype(np.float32)


def load_kv_int4(root: str):
    path = os.path.join(root, "vllm_plugin", "exl3rocm", "kv_int4.py")
    spec = importlib.util.spec_from_file_location("ref_kv_int4", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def kv_rows(rng, n, heads):
    """N(0,1) rows with 1 % of the channels (a fixed set per head) scaled by 8, fp16."""
    x = rng.standard_normal((n, heads, D)).astype(np.float32)
    for h in range(heads):
        ch = rng.choice(D, size=max(1, D // 100), replace=False)
        x[:, h, ch] *= 8.0
    return x.astype(np.float16)


def layout(rng):
    """Token -> slot mapping over a shuffled block pool, block table and query metadata."""
    nb_seq = [(L + BS - 1) // BS for L in SEQ_LENS]
    nblocks = sum(nb_seq) + 3  # a few blocks no sequence uses
    perm = rng.permutation(nblocks)
    bt = np.full((len(SEQ_LENS), max(nb_seq)), 0, dtype=np.int32)
    o = 0
    for s, nb in enumerate(nb_seq):
        bt[s, :nb] = perm[o:o + nb]
        o += nb
    slots = np.concatenate([bt[s, np.arange(L) // BS].astype(np.int64) * BS + np.arange(L) % BS
                            for s, L in enumerate(SEQ_LENS)])
    return nblocks, bt, slots


def main(root: str) -> None:
    rng = np.random.default_rng(SEED)
    g: dict[str, np.ndarray] = {}
    nblocks, bt, slots = layout(rng)
    T = int(sum(SEQ_LENS))
    key, val = kv_rows(rng, T, HKV), kv_rows(rng, T, HKV)
    q1 = rng.standard_normal((len(SEQ_LENS), HQ, D)).astype(np.float16)        # decode: 1 token / seq
    q4 = rng.standard_normal((4 * len(SEQ_LENS), HQ, D)).astype(np.float16)    # verify: 4 tokens / seq
    g.update(key=key, value=val, slots=slots, block_table=bt, seq_lens=np.array(SEQ_LENS, np.int32),
             q_decode=q1, q_verify=q4, num_blocks=np.array(nblocks), signs=rht_signs())
    # the write's batch metadata: both sequences in one prefill batch
    qsl_write = np.array([0, SEQ_LENS[0], T], dtype=np.int32)
    g["qsl_write"] = qsl_write
    scale = D ** -0.5

    kt, vt = torch.from_numpy(key), torch.from_numpy(val)
    st = torch.from_numpy(slots)
    btt = torch.from_numpy(bt)
    sl = torch.from_numpy(np.array(SEQ_LENS, np.int32))
    qsl1 = torch.tensor([0, 1, 2], dtype=torch.int32)
    qsl4 = torch.tensor([0, 4, 8], dtype=torch.int32)

    # ---------------- int8: vLLM's own kernels ----------------
    from vllm.v1.attention.ops.triton_reshape_and_cache_flash import \
        triton_reshape_and_cache_flash_per_token_head_quant
    from vllm.v1.attention.ops.triton_unified_attention import unified_attention
    from vllm.v1.kv_cache_interface import KVQuantMode
    kc = torch.zeros((nblocks, BS, HKV, D), dtype=torch.int8)
    vc = torch.zeros_like(kc)
    ks = torch.zeros((nblocks, BS, HKV), dtype=torch.float32)
    vs = torch.zeros_like(ks)
    triton_reshape_and_cache_flash_per_token_head_quant(kt, vt, kc, vc, ks, vs, st)
    g.update(int8_key_cache=kc.numpy(), int8_value_cache=vc.numpy(), int8_k_scale=ks.numpy(),
             int8_v_scale=vs.numpy())
    segs = 16
    for name, q, qsl, mq in (("decode", q1, qsl1, 1), ("verify", q4, qsl4, 4)):
        qt = torch.from_numpy(q)
        out = torch.zeros_like(qt)
        extra = {}
        if mq == 1:  # the split-KV path vLLM takes for decode batches
            extra = dict(seq_threshold_3D=64, num_par_softmax_segments=segs,
                         softmax_segm_output=torch.empty((q.shape[0], HQ, segs, D), dtype=torch.float32),
                         softmax_segm_max=torch.empty((q.shape[0], HQ, segs), dtype=torch.float32),
                         softmax_segm_expsum=torch.empty((q.shape[0], HQ, segs), dtype=torch.float32))
        unified_attention(q=qt, k=kc, v=vc, out=out, cu_seqlens_q=qsl, max_seqlen_q=mq, seqused_k=sl,
                          max_seqlen_k=max(SEQ_LENS), softmax_scale=scale, causal=True, window_size=(-1, -1),
                          block_table=btt, softcap=0.0, q_descale=None, k_descale=None, v_descale=None,
                          kv_quant_mode=KVQuantMode.INT8_PER_TOKEN_HEAD, k_scale_cache=ks, v_scale_cache=vs,
                          **extra)
        g[f"int8_out_{name}"] = out.numpy()

    # ---------------- int4: the reference's kv_int4.py ----------------
    # kv_int4.exact_buffers asks torch whether a CUDA graph is being captured; on a machine without a
    # CUDA driver that query raises instead of answering "no", so answer it here
    torch.cuda.is_current_stream_capturing = lambda: False
    R = load_kv_int4(root)
    s = torch.from_numpy(rht_signs())
    h = torch.from_numpy(sylvester(D))
    fwd, inv = s[:, None] * h, h * s[None, :]
    R._mats[(D, "cpu")] = {"fwd": fwd.half(), "inv_d": (inv / D).half(), "fwd_n": (fwd * D ** -0.5).half(),
                           "inv_n": (inv * D ** -0.5).half()}
    mk = (rng.standard_normal((HKV, D)) * 0.5).astype(np.float32)
    mv = (rng.standard_normal((HKV, D)) * 0.5).astype(np.float32)
    R._means = {"centered": {"k": torch.from_numpy(mk), "v": torch.from_numpy(mv)}}
    g.update(mean_k=mk, mean_v=mv)
    R.configure_request_slots(len(SEQ_LENS))
    R.set_batch_slots(torch.arange(len(SEQ_LENS), dtype=torch.int32))
    g["int4_sinks"], g["int4_tail"] = np.array(R._CFG["sinks"]), np.array(R._CFG["tail"])
    for layer in ("plain", "centered"):
        kc4 = torch.zeros((nblocks, BS, HKV, D // 2), dtype=torch.uint8)
        vc4 = torch.zeros_like(kc4)
        ks4 = torch.zeros((nblocks, BS, HKV), dtype=torch.float32)
        vs4 = torch.zeros_like(ks4)
        R.reshape_and_cache(kt, vt, kc4, vc4, st, k_scale_cache=ks4, v_scale_cache=vs4, layer_name=layer,
                            query_start_loc=torch.from_numpy(qsl_write), seq_lens=sl)
        ex = R._exact[layer]
        p = f"int4_{layer}_"
        bias = R._bias.get((layer, "cpu"))
        if bias is not None:  # the rotated-domain write biases -(mean @ F) the reference computed
            g.update({p + "bias_k": bias["k"].numpy(), p + "bias_v": bias["v"].numpy()})
        g.update({p + "key_cache": kc4.numpy(), p + "value_cache": vc4.numpy(),
                  p + "k_scale_bits": ks4.numpy().view(np.uint32), p + "v_scale_bits": vs4.numpy().view(np.uint32),
                  p + "sink_k": ex["sink_k"].numpy(), p + "sink_v": ex["sink_v"].numpy(),
                  p + "ring_k": ex["ring_k"].numpy(), p + "ring_v": ex["ring_v"].numpy(),
                  p + "ring_tag": ex["tag"].numpy()})
        for name, q, qsl, mq in (("decode", q1, qsl1, 1), ("verify", q4, qsl4, 4)):
            qt = torch.from_numpy(q)
            out = torch.zeros_like(qt)
            R.attention(q=qt, k=kc4, v=vc4, out=out, cu_seqlens_q=qsl, max_seqlen_q=mq, seqused_k=sl,
                        block_table=btt, softmax_scale=scale, k_scale_cache=ks4, v_scale_cache=vs4,
                        layer_name=layer)
            g[p + f"out_{name}"] = out.numpy()
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT}: {len(g)} arrays, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
