"""A synthetic dense decoder for measuring decode tokens/s through this library alone, on one GPU
or tensor-parallel over several.

The workload is the 27B-class decoder shape the decode tok/s metric is quoted on: 64 layers,
hidden 5120, 40 q / 8 kv heads of 128, SwiGLU 17408, vocab 151936, RMSNorm, neox RoPE
(theta 1e6), every layer full attention over an int8 paged KV cache.  Weights are seeded random
EXL3 trellis codes (mul1 codebook) at a fixed mixed width: q/k/v and o 4 bits, gate/up 3 bits,
down 4 bits (3.46 bits per weight on average), lm_head 4 bits.  svh carries a 1/sqrt(k) scale so
activations stay O(1) through the layers, as real checkpoints' scales keep them.  The reference's
checkpoint (a hybrid model with linear-attention layers) is not available here; this stands in
for its full-attention layers.

One step (``step``) runs, for M = batch * q_len query rows:
  embed -> 64 x [ qkv (one grouped launch, the RMSNorm of its input fused in) -> rope + int8 KV write
  (one launch) -> paged int8 attention + split combine -> o (+ residual in the epilogue) -> gate/up
  (RMSNorm fused in, SiLU * up in the epilogue) -> down (+ residual in the epilogue) ]
  -> lm_head (final RMSNorm fused in) -> argmax
seven of this library's launches per layer.  fused=False runs the same step with separate RMSNorm,
RoPE and KV-write launches (ten per layer), for comparison.  All buffers are allocated up front, so
the step can be captured in a CUDA graph.

The KV cache is int8 (default) or int4 per-token-head (kv="int4": nibble rows, zero point in the
scale word, RHT domain, the exact rows off).  A step of more than 16 rows (batched decode, e.g. 64
sequences) runs its linears through the tcgen05 GEMM (exl3b_gemm) with separate RMSNorm, SiLU * up and
residual adds, since the fused epilogues are those of the 1..16-row GEMV.  ``prefill`` runs one
prompt eagerly through the same layers: GEMM linears, RoPE, the cache write of every prompt token and
the prefill attention over the quantised cache (gather + fp16 attention).

Tensor parallel (tp_size > 1, one process per GPU): every rank draws the whole model from the same
seed, layer by layer, and keeps its shard, so the sharded model is the single-GPU model.  q/k/v
are split by heads and gate/up by columns (no exchange); o and down by their inputs, summed across
ranks inside the GEMV through peer memory (exl3b_linear_tp) with the residual add in the same
epilogue; each rank caches its own KV heads; the lm_head is split in whole 128-column blocks, and
the ranks' (max, index) pairs are all-gathered (NCCL) to pick the next tokens.
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

    def layer_bytes(self) -> int:
        """Trellis bytes one layer streams per step (all ranks together)."""
        h, d = self.hidden, self.head
        qkv = h * (self.q_heads + 2 * self.kv_heads) * d * self.bits_qkv
        o = self.q_heads * d * h * self.bits_o
        gu = 2 * h * self.intermediate * self.bits_gate_up
        dn = self.intermediate * h * self.bits_down
        return (qkv + o + gu + dn) // 8


class Exl3Weight:
    """One EXL3 matrix k -> n: trellis int16 [k/16][n/16][16K], suh fp16 [k], svh fp16 [n]."""

    def __init__(self, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int):
        self.trellis, self.suh, self.svh, self.K = trellis, suh, svh, K
        self.k, self.n = suh.shape[0], svh.shape[0]

    @staticmethod
    def random(gen: torch.Generator, k: int, n: int, K: int, device) -> "Exl3Weight":
        codes = torch.randint(0, 65536, (k // 16, n // 16, 16 * K), generator=gen, device=device, dtype=torch.int32)
        trellis = codes.to(torch.int16)
        del codes
        suh = (torch.randint(0, 2, (k,), generator=gen, device=device) * 2 - 1).to(torch.float16)
        svh = ((torch.randint(0, 2, (n,), generator=gen, device=device) * 2 - 1) / math.sqrt(k)).to(torch.float16)
        return Exl3Weight(trellis, suh, svh, K)

    def columns(self, n0: int, n1: int) -> "Exl3Weight":
        """Output columns [n0, n1) (multiples of 128): a column-parallel shard."""
        return Exl3Weight(self.trellis[:, n0 // 16:n1 // 16].contiguous(), self.suh, self.svh[n0:n1].contiguous(),
                          self.K)

    def rows(self, k0: int, k1: int) -> "Exl3Weight":
        """Input features [k0, k1) (multiples of 128): a row-parallel shard."""
        return Exl3Weight(self.trellis[k0 // 16:k1 // 16].contiguous(), self.suh[k0:k1].contiguous(), self.svh,
                          self.K)


class Layer:
    """One layer's weights, drawn whole (the same draw at every tensor-parallel size) and sharded."""

    def __init__(self, gen, s: DecoderShape, device, tp: int = 1, rank: int = 0):
        h, d = s.hidden, s.head
        qd, kd, it = s.q_heads * d // tp, s.kv_heads * d // tp, s.intermediate // tp
        q = Exl3Weight.random(gen, h, s.q_heads * d, s.bits_qkv, device)
        k = Exl3Weight.random(gen, h, s.kv_heads * d, s.bits_qkv, device)
        v = Exl3Weight.random(gen, h, s.kv_heads * d, s.bits_qkv, device)
        o = Exl3Weight.random(gen, s.q_heads * d, h, s.bits_o, device)
        gate = Exl3Weight.random(gen, h, s.intermediate, s.bits_gate_up, device)
        up = Exl3Weight.random(gen, h, s.intermediate, s.bits_gate_up, device)
        down = Exl3Weight.random(gen, s.intermediate, h, s.bits_down, device)
        if tp == 1:
            self.q, self.k, self.v, self.o, self.gate, self.up, self.down = q, k, v, o, gate, up, down
        else:
            self.q, self.k, self.v = (q.columns(rank * qd, (rank + 1) * qd), k.columns(rank * kd, (rank + 1) * kd),
                                      v.columns(rank * kd, (rank + 1) * kd))
            self.o = o.rows(rank * qd, (rank + 1) * qd)
            self.gate, self.up = gate.columns(rank * it, (rank + 1) * it), up.columns(rank * it, (rank + 1) * it)
            self.down = down.rows(rank * it, (rank + 1) * it)
        self.norm_in = (1.0 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.float16)
        self.norm_post = (1.0 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.float16)


def head_columns(vocab: int, tp: int, rank: int) -> tuple:
    """This rank's lm_head columns: whole 128-column blocks, ceil(blocks / tp) per rank."""
    blocks = vocab // 128
    per = -(-blocks // tp)
    b0, b1 = min(blocks, rank * per), min(blocks, (rank + 1) * per)
    return b0 * 128, b1 * 128


class SyntheticDecoder:
    """Weights, an int8 paged KV cache of `ctx` tokens for each of `batch` sequences, and the
    buffers of one decode step of q_len tokens per sequence (the last q_len positions of ctx).

    tp_size > 1: this rank's shard; `comm` is an exl3rocm.tp.TpComm over the ranks (o and down
    reduce through it) and `group` the process group of the next-token all-gather."""

    def __init__(self, shape: DecoderShape, device, batch: int = 1, q_len: int = 1, ctx: int = 32768,
                 seed: int = 0, weights_of: "SyntheticDecoder | None" = None, tp_size: int = 1, tp_rank: int = 0,
                 comm=None, group=None, fused: bool = True, kv_cache: str = "int8",
                 gemm_linears: bool | None = None):
        """weights_of: take the weights of another decoder of the same shape and sharding (a different
        batch, query length or context over the same model).  kv_cache: "int8" or "int4".
        gemm_linears: run the step's linears through the GEMM route (default: when M > 16)."""
        s = self.s = shape
        self.device = device = torch.device(device)
        self.batch, self.q_len, self.ctx = batch, q_len, ctx
        self.tp, self.rank, self.comm, self.group = tp_size, tp_rank, comm, group
        self.fused = fused
        M = self.M = batch * q_len
        if kv_cache not in ("int8", "int4"):
            raise ValueError(f"kv_cache {kv_cache!r}: int8 or int4")
        self.kv_kind = kv_cache
        # GEMM linears, separate norm / activation / residual adds
        self.batched = M > ops.GEMV_MAX_ROWS if gemm_linears is None else bool(gemm_linears)
        if self.batched and q_len != 1:
            raise ValueError("batched steps are decode steps (q_len 1)")
        if ctx % s.block_size or q_len > ctx:
            raise ValueError("ctx must be a multiple of the block size and >= q_len")
        tp = tp_size
        if tp > 1:
            if comm is None and not self.batched:
                raise ValueError("tensor parallel decode needs a TpComm")
            if s.q_heads % tp or s.kv_heads % tp or (s.intermediate // 128) % tp:
                raise ValueError(f"heads and intermediate blocks must divide by tp {tp}")
            if (s.q_heads * s.head // tp) % 128:
                raise ValueError("row-parallel shards must be whole 128-blocks")
        self.hq, self.hkv = s.q_heads // tp, s.kv_heads // tp
        self.v0, self.v1 = head_columns(s.vocab, tp, tp_rank)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        if weights_of is not None:
            assert weights_of.s == s and weights_of.tp == tp and weights_of.rank == tp_rank
            self.layers, self.embed = weights_of.layers, weights_of.embed
            self.norm_final, self.head = weights_of.norm_final, weights_of.head
        else:
            self.layers = [Layer(gen, s, device, tp, tp_rank) for _ in range(s.layers)]
            self.embed = (torch.randn(s.vocab, s.hidden, generator=gen, device=device)).to(torch.float16)
            self.norm_final = (1.0 + 0.1 * torch.randn(s.hidden, generator=gen, device=device)).to(torch.float16)
            head = Exl3Weight.random(gen, s.hidden, s.vocab, s.bits_head, device)
            self.head = head if tp == 1 else head.columns(self.v0, self.v1)
            del head
        # int8 paged cache: sequence b owns blocks [b * bps, (b + 1) * bps); drawn for all heads and
        # sliced to this rank's, so the cache contents do not depend on the sharding either
        bps = ctx // s.block_size
        nblk = batch * bps
        h0, h1 = tp_rank * self.hkv, (tp_rank + 1) * self.hkv
        self.k_cache, self.v_cache, self.k_scale, self.v_scale = [], [], [], []
        row = s.head if kv_cache == "int8" else s.head // 2
        for _ in range(s.layers):
            for dst, is_rows in ((self.k_cache, True), (self.v_cache, True), (self.k_scale, False),
                                 (self.v_scale, False)):
                if is_rows and kv_cache == "int8":
                    full = torch.randint(-127, 128, (nblk, s.block_size, s.kv_heads, row), generator=gen,
                                         device=device, dtype=torch.int8)
                elif is_rows:  # packed nibbles
                    full = torch.randint(0, 256, (nblk, s.block_size, s.kv_heads, row), generator=gen,
                                         device=device, dtype=torch.int32).to(torch.uint8)
                elif kv_cache == "int8":
                    full = torch.rand((nblk, s.block_size, s.kv_heads), generator=gen, device=device) * 0.02
                else:  # scale word: (fp32 scale & ~0xF) | zero point
                    sc = torch.rand((nblk, s.block_size, s.kv_heads), generator=gen, device=device) * 0.3 + 0.05
                    zp = torch.randint(4, 12, sc.shape, generator=gen, device=device, dtype=torch.int32)
                    full = ((sc.view(torch.int32) & ~0xF) | zp).view(torch.float32)
                    del sc, zp
                dst.append(full if tp == 1 else full[:, :, h0:h1].contiguous())
                del full
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
        qd, kd = self.hq * s.head, self.hkv * s.head
        self.residual = torch.empty(M, s.hidden, dtype=torch.float16, device=device)
        self.h = torch.empty(M, s.hidden, dtype=torch.float16, device=device)
        self.qkv = torch.empty(M, qd + 2 * kd, dtype=torch.float16, device=device)
        self.q = torch.empty(M, qd, dtype=torch.float16, device=device)
        self.attn = torch.empty(M, qd, dtype=torch.float16, device=device)
        self.act = torch.empty(M, s.intermediate // tp, dtype=torch.float16, device=device)
        if self.batched or kv_cache == "int4":
            self.gu = torch.empty(M, 2 * s.intermediate // tp, dtype=torch.float16, device=device)
            self.row_out = torch.empty(M, s.hidden, dtype=torch.float16, device=device)
        self.logits = torch.empty(M, self.v1 - self.v0, dtype=torch.float16, device=device)
        self.next_tokens = torch.empty(M, dtype=torch.int64, device=device)
        if tp > 1:
            self.pick = torch.empty(M, 2, dtype=torch.float32, device=device)
            self.picks = torch.empty(tp * M, 2, dtype=torch.float32, device=device)
        self.reserve()

    def reserve(self, stream: torch.cuda.Stream | None = None) -> None:
        """Workspaces of every call of the step on `stream` (the current one by default), so that a
        capture on it allocates nothing."""
        s, M, dev = self.s, self.M, self.device
        qd, kd, it = self.hq * s.head, self.hkv * s.head, s.intermediate // self.tp
        ctx = torch.cuda.stream(stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream(dev))
        with ctx:
            for k, n, g in ((s.hidden, qd + 2 * kd, 3), (qd, s.hidden, 1), (s.hidden, 2 * it, 2),
                            (it, s.hidden, 1), (s.hidden, self.v1 - self.v0, 1)):
                if self.batched:
                    ops.reserve_gemm_workspace(dev, M, k)
                else:
                    ops.reserve_workspace(dev, k, n, g, M)
            kv.reserve_attention_workspace(dev, M, self.hq, self.batch, self.hkv, self.ctx)

    def weight_bytes(self) -> int:
        """Trellis bytes one step streams, all ranks together (all layers and the lm_head)."""
        return self.s.layers * self.s.layer_bytes() + self.s.hidden * self.s.vocab * self.s.bits_head // 8

    def kv_bytes(self) -> int:
        """KV cache bytes the attention reads per step, all ranks together (K and V rows + fp32 scales)."""
        s = self.s
        row = s.head if self.kv_kind == "int8" else s.head // 2
        return s.layers * self.batch * self.ctx * s.kv_heads * (2 * row + 8)

    def _attention(self, i: int, q: torch.Tensor, out: torch.Tensor, seq_lens, cu_q, max_q: int, max_k: int,
                   block_table=None) -> None:
        s = self.s
        fn = kv.attention_int8 if self.kv_kind == "int8" else kv.attention
        fn(q=q, k=self.k_cache[i], v=self.v_cache[i], out=out, cu_seqlens_q=cu_q, max_seqlen_q=max_q,
           seqused_k=seq_lens, block_table=self.block_table if block_table is None else block_table,
           softmax_scale=1.0 / math.sqrt(s.head), k_scale_cache=self.k_scale[i], v_scale_cache=self.v_scale[i],
           max_seqlen_k=max_k)

    def _write_cache(self, i: int, qkv: torch.Tensor, slots: torch.Tensor) -> None:
        s = self.s
        qd, kd = self.hq * s.head, self.hkv * s.head
        T = qkv.shape[0]
        key = qkv[:, qd:qd + kd].view(T, self.hkv, s.head)
        val = qkv[:, qd + kd:].view(T, self.hkv, s.head)
        if self.kv_kind == "int8":
            kv.reshape_and_cache_int8(key, val, self.k_cache[i], self.v_cache[i], slots, self.k_scale[i],
                                      self.v_scale[i])
        else:
            kv.reshape_and_cache(key, val, self.k_cache[i], self.v_cache[i], slots, k_scale_cache=self.k_scale[i],
                                 v_scale_cache=self.v_scale[i])

    def _large_layer(self, i: int, x_res: torch.Tensor, qkv: torch.Tensor, q: torch.Tensor, attn: torch.Tensor,
                     positions: torch.Tensor, slots: torch.Tensor, attend) -> None:
        """One layer for many rows: RMSNorm, GEMM linears (exl3b_gemm), RoPE, the cache write, attention
        (``attend``), residual adds; under tensor parallelism the row-parallel partial outputs are summed
        with an NCCL all-reduce."""
        s, L = self.s, self.layers[i]
        h = rmsnorm(x_res, L.norm_in, s.eps)
        self._gemm_into(h, [L.q, L.k, L.v], s.bits_qkv, qkv)
        rope_neox(qkv, q, self.hq, self.hkv, positions, self.cos_sin)
        self._write_cache(i, qkv, slots)
        attend(i, q.view(-1, self.hq, s.head), attn.view(-1, self.hq, s.head))
        self._row_add(x_res, attn, L.o, s.bits_o)
        h = rmsnorm(x_res, L.norm_post, s.eps)
        gu = torch.empty(h.shape[0], 2 * L.gate.n, dtype=torch.float16, device=h.device)
        self._gemm_into(h, [L.gate, L.up], s.bits_gate_up, gu)
        act = ops.silu_mul(gu)
        self._row_add(x_res, act, L.down, s.bits_down)

    @staticmethod
    def _gemm_into(x: torch.Tensor, ws: list, K: int, out: torch.Tensor) -> None:
        """The GEMM route (exl3b_gemm) of each weight into its column slice of out."""
        n0 = 0
        for w in ws:
            ops._linear_large(x, w.trellis, w.suh, w.svh, K, *CB, out[:, n0:n0 + w.n])
            n0 += w.n

    def _row_add(self, x_res: torch.Tensor, x: torch.Tensor, w: Exl3Weight, K: int) -> None:
        y = torch.empty(x.shape[0], w.n, dtype=torch.float16, device=x.device)
        self._gemm_into(x, [w], K, y)
        if self.tp > 1:
            torch.distributed.all_reduce(y, group=self.group)
        x_res.add_(y)

    def layer_forward(self, i: int) -> None:
        s, L = self.s, self.layers[i]
        qd, kd, M = self.hq * s.head, self.hkv * s.head, self.M
        if self.batched:
            self._large_layer(i, self.residual, self.qkv, self.q, self.attn, self.positions, self.slot_mapping,
                              lambda j, qq, out: self._attention(j, qq, out, self.seq_lens, self.cu_q, 1, self.ctx))
            return
        if self.kv_kind == "int4":
            self._normed_linear(L.norm_in, [L.q, L.k, L.v], s.bits_qkv, self.qkv)
            rope_neox(self.qkv, self.q, self.hq, self.hkv, self.positions, self.cos_sin)
            self._write_cache(i, self.qkv, self.slot_mapping)
            self._attention(i, self.q.view(M, self.hq, s.head), self.attn.view(M, self.hq, s.head), self.seq_lens,
                            self.cu_q, self.q_len, self.ctx)
            self._row_parallel(self.attn, L.o, s.bits_o)
            self._normed_linear(L.norm_post, [L.gate, L.up], s.bits_gate_up, self.act, ops.ACT_SILU_MUL)
            self._row_parallel(self.act, L.down, s.bits_down)
            return
        mcg, mul1 = CB
        self._normed_linear(L.norm_in, [L.q, L.k, L.v], s.bits_qkv, self.qkv)
        if self.fused:
            kv.rope_and_cache_int8(self.qkv, self.q, self.hq, self.hkv, self.positions, self.cos_sin,
                                   self.k_cache[i], self.v_cache[i], self.slot_mapping, self.k_scale[i],
                                   self.v_scale[i])
        else:
            rope_neox(self.qkv, self.q, self.hq, self.hkv, self.positions, self.cos_sin)
            key = self.qkv[:, qd:qd + kd].view(M, self.hkv, s.head)
            val = self.qkv[:, qd + kd:].view(M, self.hkv, s.head)
            kv.reshape_and_cache_int8(key, val, self.k_cache[i], self.v_cache[i], self.slot_mapping,
                                      self.k_scale[i], self.v_scale[i])
        kv.attention_int8(q=self.q.view(M, self.hq, s.head), k=self.k_cache[i], v=self.v_cache[i],
                          out=self.attn.view(M, self.hq, s.head), cu_seqlens_q=self.cu_q, max_seqlen_q=self.q_len,
                          seqused_k=self.seq_lens, block_table=self.block_table,
                          softmax_scale=1.0 / math.sqrt(s.head), k_scale_cache=self.k_scale[i],
                          v_scale_cache=self.v_scale[i], max_seqlen_k=self.ctx)
        self._row_parallel(self.attn, L.o, s.bits_o)
        self._normed_linear(L.norm_post, [L.gate, L.up], s.bits_gate_up, self.act, ops.ACT_SILU_MUL)
        self._row_parallel(self.act, L.down, s.bits_down)

    def _normed_linear(self, norm_w: torch.Tensor, ws: list, K: int, y: torch.Tensor, flags: int = 0) -> None:
        """y = linear(RMSNorm(residual)): the norm inside the GEMV, or (fused=False) its own launch."""
        args = ([w.trellis for w in ws], [w.suh for w in ws], [w.svh for w in ws], K, *CB, y, flags)
        if self.fused:
            ops.linear_into(self.residual, *args, norm=(norm_w, self.s.eps))
        else:
            rmsnorm(self.residual, norm_w, self.s.eps, out=self.h)
            ops.linear_into(self.h, *args)

    def _row_parallel(self, x: torch.Tensor, w: Exl3Weight, K: int) -> None:
        """residual += x @ W: the residual add in the GEMV epilogue; under tensor parallelism the
        ranks' partial sums are reduced inside the same kernel first."""
        if self.tp == 1:
            ops.linear_into(x, [w.trellis], [w.suh], [w.svh], K, *CB, self.residual, ops.Y_ADD)
        else:
            from .tp import linear_tp
            linear_tp(x, w.trellis, w.suh, w.svh, K, *CB, self.comm, residual=self.residual)

    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        """One decode step for the M input tokens (int64 on the device); returns the greedy next tokens
        (self.next_tokens)."""
        s = self.s
        torch.index_select(self.embed, 0, tokens, out=self.residual)
        for i in range(s.layers):
            self.layer_forward(i)
        if self.batched:
            self.logits.copy_(torch.ops.exl3rocm.linear(rmsnorm(self.residual, self.norm_final, s.eps),
                                                        self.head.trellis, self.head.suh, self.head.svh, s.bits_head,
                                                        *CB))
        else:
            self._normed_linear(self.norm_final, [self.head], s.bits_head, self.logits)
        if self.tp == 1:
            torch.argmax(self.logits, dim=-1, out=self.next_tokens)
        else:
            # each rank's best column, then the best over ranks (the first on ties, as one argmax over
            # the whole vocabulary: ranks hold increasing column ranges)
            val, idx = torch.max(self.logits, dim=-1)
            self.pick[:, 0] = val.float()
            self.pick[:, 1] = (idx + self.v0).float()  # exact: vocab < 2^24
            torch.distributed.all_gather_into_tensor(self.picks, self.pick, group=self.group)
            p = self.picks.view(self.tp, self.M, 2)
            best = torch.argmax(p[:, :, 0], dim=0)
            self.next_tokens.copy_(p[:, :, 1].gather(0, best[None, :])[0].long())
        return self.next_tokens

    def prefill(self, tokens: torch.Tensor) -> torch.Tensor:
        """Prefill of one prompt (tokens int64 [P], P <= ctx) into sequence 0's cache, eagerly: per layer
        RMSNorm, the GEMM linears, RoPE, the cache write of all P tokens, causal prefill attention over
        the quantised cache (kv.prefill_int8 / kv.prefill: the blocks dequantised to fp16 once, then
        fp16 attention), SiLU * up and the residual adds; then the last token's logits.  Returns the
        greedy next token."""
        s, P = self.s, tokens.shape[0]
        if P > self.ctx:
            raise ValueError(f"prompt of {P} tokens for a cache of {self.ctx}")
        dev = self.device
        qd, kd = self.hq * s.head, self.hkv * s.head
        res = torch.index_select(self.embed, 0, tokens)
        qkv = torch.empty(P, qd + 2 * kd, dtype=torch.float16, device=dev)
        q = torch.empty(P, qd, dtype=torch.float16, device=dev)
        attn = torch.empty(P, qd, dtype=torch.float16, device=dev)
        pos = torch.arange(P, dtype=torch.int64, device=dev)
        slots = self.block_table[0].to(torch.int64)[pos // s.block_size] * s.block_size + pos % s.block_size
        seq = torch.tensor([P], dtype=torch.int32, device=dev)
        cu = torch.tensor([0, P], dtype=torch.int32, device=dev)
        bt = self.block_table[:1]

        def attend(i, qq, out):
            kw = dict(q=qq, k=self.k_cache[i], v=self.v_cache[i], out=out, cu_seqlens_q=cu, max_seqlen_q=P,
                      seqused_k=seq, max_seqlen_k=P, block_table=bt, softmax_scale=1.0 / math.sqrt(s.head),
                      k_scale_cache=self.k_scale[i], v_scale_cache=self.v_scale[i])
            if self.kv_kind == "int8":
                kv.prefill_int8(None, kw)
            else:
                kv.prefill(None, kw)

        for i in range(s.layers):
            self._large_layer(i, res, qkv, q, attn, pos, slots, attend)
        last = rmsnorm(res[-1:], self.norm_final, s.eps)
        logits = torch.ops.exl3rocm.linear(last, self.head.trellis, self.head.suh, self.head.svh, s.bits_head, *CB)
        self.prefill_logits = logits
        return torch.argmax(logits, dim=-1)

    def launches_per_step(self) -> int:
        """This library's kernel launches in one step.  int8, 1..16 rows: per layer 4 linears (norms
        fused), rope + KV write, the attention and its split combine, then the lm_head; unfused: 3 more
        per layer, 1 more at the end.  int4 adds a separate RoPE and the q rotation (9 per layer).
        Batched (GEMM) steps: 2 RMSNorms, 7 GEMMs with their had_in, RoPE, write, attention (+ combine,
        + q rotation for int4), SiLU * up per layer; final norm and lm_head."""
        L = self.s.layers
        if self.batched:
            return L * (2 + 2 * 7 + 1 + 1 + (2 if self.kv_kind == "int8" else 3) + 1) + 3
        if self.kv_kind == "int4":
            return L * 9 + 1
        return L * 7 + 1 if self.fused else L * 10 + 2


def main(argv=None) -> None:
    """python -m exl3rocm.synthetic [--batch B] [--q-len Q] [--ctx N] [--layers L] [--steps S]
    Times CUDA-graph replays of the decode step on one GPU and prints one JSON line."""
    import argparse
    import json
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--q-len", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--unfused", action="store_true", help="separate RMSNorm, RoPE and KV-write launches")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    dec = SyntheticDecoder(DecoderShape(layers=a.layers), dev, batch=a.batch, q_len=a.q_len, ctx=a.ctx, seed=2024,
                           fused=not a.unfused)
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
    print(json.dumps({"batch": a.batch, "q_len": a.q_len, "ctx": a.ctx, "layers": a.layers, "fused": dec.fused,
                      "ms_per_step": ms,
                      "rows_per_s": dec.M / (ms * 1e-3), "weight_bytes": dec.weight_bytes(),
                      "kv_bytes": dec.kv_bytes()}))
    del graph


if __name__ == "__main__":
    main()
