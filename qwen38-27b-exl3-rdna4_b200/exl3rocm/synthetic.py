"""A synthetic dense decoder for measuring decode tokens/s through this library alone.

The workload is the 27B-class decoder shape the decode tok/s metric is quoted on: 64 layers,
hidden 5120, 40 q / 8 kv heads of 128, SwiGLU 17408, vocab 151936, RMSNorm, neox RoPE
(theta 1e6), every layer full attention over an int8 paged KV cache.  Weights are seeded random
EXL3 trellis codes (mul1 codebook) at a fixed mixed width: q/k/v and o 4 bits, gate/up 3 bits,
down 4 bits (3.46 bits per weight on average), lm_head 4 bits.  svh carries a 1/sqrt(k) scale so
activations stay O(1) through the layers, as real checkpoints' scales keep them.  The reference's
checkpoint (a hybrid model with linear-attention layers) is not available here; this stands in
for its full-attention layers.

One step (``step``) runs, for M = batch * q_len query rows:
  embed -> 64 x [ rmsnorm -> qkv (one grouped launch) -> rope (q out, k in place) -> int8 KV write
  -> paged int8 attention -> o (+ residual in the epilogue) -> rmsnorm -> gate/up with SiLU * up
  in the epilogue -> down (+ residual in the epilogue) ] -> rmsnorm -> lm_head -> argmax
All buffers are allocated up front, so the step can be captured in a CUDA graph.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import kv, ops
from .glue import rmsnorm, rope_cos_sin, rope_neox

CB = (False, True)  # (mcg, mul1): the reference's production codebook


@dataclass(frozen=True)
class DecoderShape:
    layers: int = 64
    hidden: int = 5120
    q_heads: int = 40
    kv_heads: int = 8
    head: int = 128
    intermediate: int = 17408
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6
    bits_qkv: int = 4
    bits_o: int = 4
    bits_gate_up: int = 3
    bits_down: int = 4
    bits_head: int = 4
    block_size: int = 16

    def weights_per_layer(self) -> int:
        qkv = self.hidden * (self.q_heads + 2 * self.kv_heads) * self.head
        return qkv + self.q_heads * self.head * self.hidden + 3 * self.hidden * self.intermediate

    def layer_bytes(self) -> int:
        """Trellis bytes one layer streams per step."""
        h, d = self.hidden, self.head
        qkv = h * (self.q_heads + 2 * self.kv_heads) * d * self.bits_qkv
        o = self.q_heads * d * h * self.bits_o
        gu = 2 * h * self.intermediate * self.bits_gate_up
        dn = self.intermediate * h * self.bits_down
        return (qkv + o + gu + dn) // 8


class Exl3Weight:
    """One EXL3 matrix k -> n: trellis int16 [k/16][n/16][16K], suh fp16 [k], svh fp16 [n]."""

    def __init__(self, gen: torch.Generator, k: int, n: int, K: int, device):
        codes = torch.randint(0, 65536, (k // 16, n // 16, 16 * K), generator=gen, device=device, dtype=torch.int32)
        self.trellis = codes.to(torch.int16)
        del codes
        self.suh = (torch.randint(0, 2, (k,), generator=gen, device=device) * 2 - 1).to(torch.float16)
        self.svh = ((torch.randint(0, 2, (n,), generator=gen, device=device) * 2 - 1) / math.sqrt(k)).to(torch.float16)
        self.k, self.n, self.K = k, n, K


class Layer:
    def __init__(self, gen, s: DecoderShape, device):
        h, d = s.hidden, s.head
        self.q = Exl3Weight(gen, h, s.q_heads * d, s.bits_qkv, device)
        self.k = Exl3Weight(gen, h, s.kv_heads * d, s.bits_qkv, device)
        self.v = Exl3Weight(gen, h, s.kv_heads * d, s.bits_qkv, device)
        self.o = Exl3Weight(gen, s.q_heads * d, h, s.bits_o, device)
        self.gate = Exl3Weight(gen, h, s.intermediate, s.bits_gate_up, device)
        self.up = Exl3Weight(gen, h, s.intermediate, s.bits_gate_up, device)
        self.down = Exl3Weight(gen, s.intermediate, h, s.bits_down, device)
        self.norm_in = (1.0 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.float16)
        self.norm_post = (1.0 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.float16)


class SyntheticDecoder:
    """Weights, an int8 paged KV cache of `ctx` tokens for each of `batch` sequences, and the
    buffers of one decode step of q_len tokens per sequence (the last q_len positions of ctx)."""

    def __init__(self, shape: DecoderShape, device, batch: int = 1, q_len: int = 1, ctx: int = 32768,
                 seed: int = 0, weights_of: "SyntheticDecoder | None" = None):
        """weights_of: take the weights of another decoder of the same shape (a different batch,
        query length or context over the same model)."""
        s = self.s = shape
        self.device = device = torch.device(device)
        self.batch, self.q_len, self.ctx = batch, q_len, ctx
        M = self.M = batch * q_len
        if M > ops.GEMV_MAX_ROWS:
            raise ValueError(f"decode step of {M} rows: the fused linears take 1..{ops.GEMV_MAX_ROWS}")
        if ctx % s.block_size or q_len > ctx:
            raise ValueError("ctx must be a multiple of the block size and >= q_len")
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        if weights_of is not None:
            assert weights_of.s == s
            self.layers, self.embed = weights_of.layers, weights_of.embed
            self.norm_final, self.head = weights_of.norm_final, weights_of.head
        else:
            self.layers = [Layer(gen, s, device) for _ in range(s.layers)]
            self.embed = (torch.randn(s.vocab, s.hidden, generator=gen, device=device)).to(torch.float16)
            self.norm_final = (1.0 + 0.1 * torch.randn(s.hidden, generator=gen, device=device)).to(torch.float16)
            self.head = Exl3Weight(gen, s.hidden, s.vocab, s.bits_head, device)
        # int8 paged cache: sequence b owns blocks [b * bps, (b + 1) * bps)
        bps = ctx // s.block_size
        nblk = batch * bps
        self.k_cache, self.v_cache, self.k_scale, self.v_scale = [], [], [], []
        for _ in range(s.layers):
            self.k_cache.append(torch.randint(-127, 128, (nblk, s.block_size, s.kv_heads, s.head), generator=gen,
                                              device=device, dtype=torch.int8))
            self.v_cache.append(torch.randint(-127, 128, (nblk, s.block_size, s.kv_heads, s.head), generator=gen,
                                              device=device, dtype=torch.int8))
            self.k_scale.append(torch.rand((nblk, s.block_size, s.kv_heads), generator=gen, device=device) * 0.02)
            self.v_scale.append(torch.rand((nblk, s.block_size, s.kv_heads), generator=gen, device=device) * 0.02)
        self.block_table = torch.arange(nblk, dtype=torch.int32, device=device).view(batch, bps)
        pos = torch.arange(ctx - q_len, ctx, dtype=torch.int64, device=device).repeat(batch)
        self.positions = pos
        seq = torch.arange(batch, dtype=torch.int64, device=device).repeat_interleave(q_len)
        self.slot_mapping = (self.block_table.to(torch.int64)[seq, pos // s.block_size] * s.block_size
                             + pos % s.block_size)
        self.seq_lens = torch.full((batch,), ctx, dtype=torch.int32, device=device)
        self.cu_q = torch.arange(0, batch + 1, dtype=torch.int32, device=device) * q_len
        self.cos_sin = rope_cos_sin(ctx, s.rope_theta, device, s.head)
        # step buffers
        qd, kd = s.q_heads * s.head, s.kv_heads * s.head
        self.residual = torch.empty(M, s.hidden, dtype=torch.float16, device=device)
        self.h = torch.empty(M, s.hidden, dtype=torch.float16, device=device)
        self.qkv = torch.empty(M, qd + 2 * kd, dtype=torch.float16, device=device)
        self.q = torch.empty(M, qd, dtype=torch.float16, device=device)
        self.attn = torch.empty(M, qd, dtype=torch.float16, device=device)
        self.act = torch.empty(M, s.intermediate, dtype=torch.float16, device=device)
        self.logits = torch.empty(M, s.vocab, dtype=torch.float16, device=device)
        self.next_tokens = torch.empty(M, dtype=torch.int64, device=device)
        self.reserve()

    def reserve(self, stream: torch.cuda.Stream | None = None) -> None:
        """Workspaces of every call of the step on `stream` (the current one by default), so that a
        capture on it allocates nothing."""
        s, M, dev = self.s, self.M, self.device
        qd, kd = s.q_heads * s.head, s.kv_heads * s.head
        ctx = torch.cuda.stream(stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream(dev))
        with ctx:
            for k, n, g in ((s.hidden, qd + 2 * kd, 3), (qd, s.hidden, 1), (s.hidden, 2 * s.intermediate, 2),
                            (s.intermediate, s.hidden, 1), (s.hidden, s.vocab, 1)):
                ops.reserve_workspace(dev, k, n, g, M)
            kv.reserve_attention_workspace(dev, M, s.q_heads, self.batch, s.kv_heads, self.ctx)

    def weight_bytes(self) -> int:
        """Trellis bytes streamed per step (all layers and the lm_head)."""
        return self.s.layers * self.s.layer_bytes() + self.s.hidden * self.s.vocab * self.s.bits_head // 8

    def kv_bytes(self) -> int:
        """KV cache bytes the attention reads per step (int8 rows + fp32 scales, K and V)."""
        s = self.s
        return s.layers * self.batch * self.ctx * s.kv_heads * (2 * s.head + 8)

    def layer_forward(self, i: int) -> None:
        s, L = self.s, self.layers[i]
        qd, kd, M = s.q_heads * s.head, s.kv_heads * s.head, self.M
        mcg, mul1 = CB
        rmsnorm(self.residual, L.norm_in, s.eps, out=self.h)
        ops.linear_into(self.h, [L.q.trellis, L.k.trellis, L.v.trellis], [L.q.suh, L.k.suh, L.v.suh],
                        [L.q.svh, L.k.svh, L.v.svh], s.bits_qkv, mcg, mul1, self.qkv)
        rope_neox(self.qkv, self.q, s.q_heads, s.kv_heads, self.positions, self.cos_sin)
        key = self.qkv[:, qd:qd + kd].view(M, s.kv_heads, s.head)
        val = self.qkv[:, qd + kd:].view(M, s.kv_heads, s.head)
        kv.reshape_and_cache_int8(key, val, self.k_cache[i], self.v_cache[i], self.slot_mapping, self.k_scale[i],
                                  self.v_scale[i])
        kv.attention_int8(q=self.q.view(M, s.q_heads, s.head), k=self.k_cache[i], v=self.v_cache[i],
                          out=self.attn.view(M, s.q_heads, s.head), cu_seqlens_q=self.cu_q, max_seqlen_q=self.q_len,
                          seqused_k=self.seq_lens, block_table=self.block_table,
                          softmax_scale=1.0 / math.sqrt(s.head), k_scale_cache=self.k_scale[i],
                          v_scale_cache=self.v_scale[i], max_seqlen_k=self.ctx)
        ops.linear_into(self.attn, [L.o.trellis], [L.o.suh], [L.o.svh], s.bits_o, mcg, mul1, self.residual, ops.Y_ADD)
        rmsnorm(self.residual, L.norm_post, s.eps, out=self.h)
        ops.linear_into(self.h, [L.gate.trellis, L.up.trellis], [L.gate.suh, L.up.suh], [L.gate.svh, L.up.svh],
                        s.bits_gate_up, mcg, mul1, self.act, ops.ACT_SILU_MUL)
        ops.linear_into(self.act, [L.down.trellis], [L.down.suh], [L.down.svh], s.bits_down, mcg, mul1,
                        self.residual, ops.Y_ADD)

    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        """One decode step for the M input tokens (int64 on the device); returns the greedy next tokens
        (self.next_tokens)."""
        s = self.s
        torch.index_select(self.embed, 0, tokens, out=self.residual)
        for i in range(s.layers):
            self.layer_forward(i)
        rmsnorm(self.residual, self.norm_final, s.eps, out=self.h)
        ops.linear_into(self.h, [self.head.trellis], [self.head.suh], [self.head.svh], s.bits_head, *CB, self.logits)
        torch.argmax(self.logits, dim=-1, out=self.next_tokens)
        return self.next_tokens

    def launches_per_step(self) -> int:
        """This library's kernel launches in one step: per layer rmsnorm x2, 4 linears, rope, the KV
        write, the attention and its split combine; then the final norm and the lm_head."""
        return self.s.layers * 10 + 2


def main(argv=None) -> None:
    """python -m exl3rocm.synthetic [--batch B] [--q-len Q] [--ctx N] [--layers L] [--steps S]
    Times CUDA-graph replays of the decode step and prints one JSON line."""
    import argparse
    import json
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--q-len", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    dec = SyntheticDecoder(DecoderShape(layers=a.layers), dev, batch=a.batch, q_len=a.q_len, ctx=a.ctx, seed=2024)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    dec.reserve(st)
    tokens = torch.randint(0, dec.s.vocab, (dec.M,), device=dev)
    with torch.cuda.stream(st):
        dec.step(tokens)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            dec.step(tokens)
            tokens.copy_(dec.next_tokens)
        for _ in range(a.warmup):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(a.steps):
            graph.replay()
        e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    print(json.dumps({"batch": a.batch, "q_len": a.q_len, "ctx": a.ctx, "layers": a.layers, "ms_per_step": ms,
                      "rows_per_s": dec.M / (ms * 1e-3), "weight_bytes": dec.weight_bytes(),
                      "kv_bytes": dec.kv_bytes()}))
    del graph


if __name__ == "__main__":
    main()
