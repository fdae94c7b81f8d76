"""Decoder-layer glue on libexl3b: RMSNorm (with the residual add), neox rotary embedding and the
cos/sin table it reads.  The reference leaves these steps to vLLM's own kernels; they are here so
that a decode step (exl3rocm.synthetic) runs on this library alone.  No CPU path.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .ops import _stream

HEAD_SIZE = 128


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = fp16(fp16(v * rsqrt(mean(v^2) + eps)) * weight) per row, v = x, or v = residual = fp16(x +
    residual) (stored back) when a residual is given (vLLM rms_norm / fused_add_rms_norm)."""
    cols = x.shape[-1]
    x2 = x.reshape(-1, cols)
    assert x2.dtype == torch.float16 and x2.stride(-1) == 1 and weight.dtype == torch.float16
    if out is None:
        out = torch.empty((x2.shape[0], cols), dtype=torch.float16, device=x.device)
    o2 = out.view(-1, cols)
    r2 = residual.view(-1, cols) if residual is not None else None
    _lib.call("exl3b_rmsnorm", x2.data_ptr(), x2.stride(0), r2.data_ptr() if r2 is not None else None,
              r2.stride(0) if r2 is not None else 0, weight.data_ptr(), o2.data_ptr(), o2.stride(0), x2.shape[0],
              cols, float(eps), _stream(x.device))
    return out


def rope_cos_sin(max_position: int, theta: float, device, head_size: int = HEAD_SIZE) -> torch.Tensor:
    """fp32 [max_position][head_size]: cos(p f_i) for the head_size / 2 frequencies
    f_i = theta^(-2i / head_size), then sin(p f_i) (vLLM RotaryEmbedding's cos_sin_cache, kept fp32)."""
    half = head_size // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64, device=device) * 2.0 / head_size))
    ang = torch.arange(max_position, dtype=torch.float64, device=device)[:, None] * inv[None, :]
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=1).to(torch.float32).contiguous()


def rope_neox(qkv: torch.Tensor, q_out: torch.Tensor, num_q_heads: int, num_k_heads: int,
              positions: torch.Tensor, cos_sin: torch.Tensor) -> None:
    """Rotate q (written to q_out [T, num_q_heads * 128]) and k (in place) of qkv rows [T, >= (q + k)
    heads * 128] by their positions (int64 [T])."""
    assert qkv.dtype == q_out.dtype == torch.float16 and qkv.stride(-1) == 1 and q_out.stride(-1) == 1
    assert positions.dtype == torch.int64 and positions.is_contiguous() and cos_sin.dtype == torch.float32
    T = qkv.shape[0]
    _lib.call("exl3b_rope_neox", qkv.data_ptr(), qkv.stride(0), q_out.data_ptr(), q_out.stride(0), T, num_q_heads,
              num_k_heads, positions.data_ptr(), cos_sin.data_ptr(), cos_sin.shape[0], _stream(qkv.device))
