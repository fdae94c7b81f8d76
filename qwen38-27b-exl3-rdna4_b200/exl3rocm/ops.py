"""EXL3 linear as opaque torch custom ops over libexl3b (sm_100a), drop-in for the reference's
``vllm_plugin/exl3rocm/ops.py``: same op names and schemas (``exl3rocm::linear`` :65-67,
``exl3rocm::linear_groups`` :106-110), fp16 output of shape ``x.shape[:-1] + (sum n,)``, fake
implementations for tracing.

Routing by the number of rows M (reference ops.py:80-97):
  M <= 16  one fused GEMV launch: had_in -> decode + mma + stream-K reduce + had_out (+ svh)
  M  > 16  exl3b_gemm: had_in into a workspace, then the tcgen05 GEMM whose CTAs decode the trellis
           into shared memory (W never materialised) with had_out + svh in its epilogue; it replaces
           the reference's reconstruct + hgemm route.

The helpers ``decode``, ``reconstruct``, ``reconstruct_slice`` and ``had_r_128`` mirror the fork's
pybind functions the reference tests call (tests/test_gpu_parity.py:101-139).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

GEMV_MAX_ROWS = 16
MAX_GROUPS = 8
X_BF16 = 0x100  # EXL3B_X_BF16: x is bf16, rounded to fp16 inside the kernel
ACT_SILU_MUL = 0x200  # EXL3B_ACT_SILU_MUL: two groups (gate, up) -> fp16(fp16(silu(gate)) * up)
Y_ADD = 0x400  # EXL3B_Y_ADD: y = fp16(y + result), the residual add in the epilogue
RECON_SLICE_N = 17408  # widest model layer, as the reference (ops.py:22-24)

_ws: dict = {}    # (device index, stream handle) -> uint8 workspace (counters zeroed once)
_gws: dict = {}   # (device index, stream handle) -> uint8 workspace of the M > 16 GEMM (A_had)
_wbuf: dict = {}  # device -> fp16 reconstruction buffer (reconstruct / reconstruct_slice)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _cb(mcg: bool, mul1: bool) -> int:
    return 2 if mul1 else (1 if mcg else 0)


def _capturing() -> bool:
    return torch.cuda.is_current_stream_capturing()


# ---------------------------------------------------------------------------------------------
# workspaces, reserved at load time so that graph capture never allocates
# ---------------------------------------------------------------------------------------------
def linear_workspace_bytes(m: int, k: int, groups: int, n_total: int) -> int:
    return int(_lib.lib().exl3b_linear_workspace_bytes(m, k, groups, n_total))


def reserve_workspace(device, k: int, n_total: int, groups: int = 1, m: int = GEMV_MAX_ROWS,
                      stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Grow (never shrink) the linear workspace of (device, stream) to fit one call shape."""
    device = torch.device(device)
    key = (device.index, (stream or torch.cuda.current_stream(device)).cuda_stream)
    need = linear_workspace_bytes(m, k, groups, n_total)
    ws = _ws.get(key)
    if ws is None or ws.numel() < need:
        if _capturing():
            raise RuntimeError("exl3rocm: linear workspace too small during graph capture; "
                               "call reserve_workspace() for this shape before capturing")
        _ws[key] = ws = torch.zeros(need, dtype=torch.uint8, device=device)
    return ws


def workspace_error(device=None) -> int:
    """Kernel error word of the current stream's workspace (0 = none); synchronises."""
    device = torch.device(device or "cuda")
    ws = _ws.get((device.index, _stream(device)))
    if ws is None:
        return 0
    out = _lib.i32(0)
    _lib.call("exl3b_linear_workspace_error", ws.data_ptr(), _lib.ctypes.byref(out), _stream(device))
    return int(out.value)


def gemm_workspace_bytes(m: int, k: int) -> int:
    return int(_lib.lib().exl3b_gemm_workspace_bytes(m, k))


def reserve_gemm_workspace(device, m: int, k: int, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Grow (never shrink) the M > 16 GEMM workspace of (device, stream) to fit m rows of k inputs."""
    device = torch.device(device)
    key = (device.index, (stream or torch.cuda.current_stream(device)).cuda_stream)
    need = gemm_workspace_bytes(m, k)
    ws = _gws.get(key)
    if ws is None or ws.numel() < need:
        if _capturing():
            raise RuntimeError("exl3rocm: GEMM workspace too small during graph capture; "
                               "call reserve_gemm_workspace() for this shape before capturing")
        _gws[key] = ws = torch.zeros(need, dtype=torch.uint8, device=device)
    return ws


def reserve_weight_buffer(device, numel: int) -> None:
    """Grow the shared reconstruction buffer at load time (reference ops.py:52-57)."""
    device = torch.device(device)
    buf = _wbuf.get(device)
    if buf is None or buf.numel() < numel:
        if _capturing():
            raise RuntimeError("exl3rocm: reconstruction buffer too small during graph capture")
        _wbuf[device] = torch.empty(numel, dtype=torch.float16, device=device)


def _weight_buffer(device, numel: int) -> torch.Tensor:
    reserve_weight_buffer(device, numel)
    return _wbuf[torch.device(device)][:numel]


# ---------------------------------------------------------------------------------------------
# the fork's pybind surface, over the C ABI
# ---------------------------------------------------------------------------------------------
def decode(codes: torch.Tensor, out: torch.Tensor, mcg: bool, mul1: bool) -> None:
    """16-bit states -> fp32 copies of the fp16 codebook values (fork ``decode``)."""
    assert codes.is_cuda and codes.is_contiguous() and codes.dtype in (torch.int16, torch.uint16)
    assert out.dtype == torch.float32 and out.is_contiguous() and out.numel() == codes.numel()
    _lib.call("exl3b_decode_states", codes.data_ptr(), out.data_ptr(), codes.numel(), _cb(mcg, mul1),
              _stream(codes.device))


def reconstruct_slice(W: torch.Tensor, trellis: torch.Tensor, K: int, mcg: bool, mul1: bool, n0: int) -> None:
    """Decode columns [n0, n0 + W.shape[1]) of the layer into W (fork ``reconstruct_slice``)."""
    k, n = trellis.shape[0] * 16, trellis.shape[1] * 16
    assert W.dtype == torch.float16 and W.stride(1) == 1 and W.shape[0] == k
    assert trellis.is_contiguous()
    _lib.call("exl3b_dequant", trellis.data_ptr(), k, n, K, _cb(mcg, mul1), n0, n0 + W.shape[1],
              W.data_ptr(), W.stride(0), _stream(W.device))


def reconstruct(W: torch.Tensor, trellis: torch.Tensor, K: int, mcg: bool, mul1: bool) -> None:
    """Decode the whole trellis into fp16 W [k, n] (fork ``reconstruct``)."""
    reconstruct_slice(W, trellis, K, mcg, mul1, 0)


def had_r_128(inp: torch.Tensor, out: torch.Tensor, pre: Optional[torch.Tensor], post: Optional[torch.Tensor],
              scale: float) -> None:
    """out = fp16(H128 fp16(inp * pre) * scale / sqrt(128)) * post per 128 columns (fork ``had_r_128``)."""
    cols = inp.shape[-1]
    i2 = inp if inp.dim() == 2 else inp.reshape(-1, cols)
    o2 = out if out.dim() == 2 else out.view(-1, cols)
    assert inp.dtype == out.dtype == torch.float16 and i2.stride(-1) == 1 and o2.stride(-1) == 1
    _lib.call("exl3b_had128", i2.data_ptr(), i2.stride(0), o2.data_ptr(), o2.stride(0), i2.shape[0], cols,
              pre.data_ptr() if pre is not None else None, post.data_ptr() if post is not None else None,
              float(scale), _stream(inp.device))


def linear_into(x2: torch.Tensor, trellis: list, suh: list, svh: list, K: int, mcg: bool, mul1: bool,
                y: torch.Tensor, flags: int = 0, norm: Optional[tuple] = None) -> None:
    """Fused M <= 16 linear of groups sharing x and K; group i -> its column slice of y.  x2 is fp16,
    or bf16 (rounded to fp16 inside the kernel, as the reference's cast at the op boundary).
    flags: Y_ADD (y += result) or ACT_SILU_MUL (two groups; y receives the activation).
    norm = (weight, eps): x2 is the un-normalised input and the RMSNorm runs inside the kernel."""
    M, k = x2.shape
    ng = len(trellis)
    widths = [int(s.shape[0]) for s in svh]
    ws = reserve_workspace(x2.device, k, sum(widths), ng, max(M, 1))
    st = _stream(x2.device)
    cb = _cb(mcg, mul1) | (X_BF16 if x2.dtype == torch.bfloat16 else 0) | flags
    if ng == 1 and norm is None:
        _lib.call("exl3b_linear", x2.data_ptr(), M, k, trellis[0].data_ptr(), widths[0], K, cb,
                  suh[0].data_ptr(), svh[0].data_ptr(), y.data_ptr(), y.stride(0), ws.data_ptr(), ws.numel(), st)
        return
    vp = _lib.c_vp * ng
    if flags & ACT_SILU_MUL:
        assert ng == 2 and widths[0] == widths[1] and y.shape[1] == widths[0]
        ys = vp(y.data_ptr(), y.data_ptr())
    else:
        cols = [0]
        for w in widths[:-1]:
            cols.append(cols[-1] + w)
        ys = vp(*[y.data_ptr() + 2 * c0 for c0 in cols])
    args = [vp(*[t.data_ptr() for t in trellis]), (_lib.i32 * ng)(*widths), K, cb]
    tail = [vp(*[s.data_ptr() for s in suh]), vp(*[s.data_ptr() for s in svh]), ys, y.stride(0), ws.data_ptr(),
            ws.numel(), st]
    if norm is None:
        _lib.call("exl3b_linear_grouped", x2.data_ptr(), M, k, ng, *args, *tail)
    else:
        w, eps = norm
        assert w.dtype == torch.float16 and w.is_contiguous() and w.shape[0] == k
        _lib.call("exl3b_linear_grouped_rmsnorm", x2.data_ptr(), M, k, ng, *args, w.data_ptr(), float(eps), *tail)


def _prep_x(x: torch.Tensor, k: int, keep_bf16: bool = False) -> torch.Tensor:
    """[M, k] contiguous fp16 (or bf16 when keep_bf16: the m <= 16 kernels round it themselves)."""
    x2 = x.reshape(-1, k)
    if x2.dtype != torch.float16 and not (keep_bf16 and x2.dtype == torch.bfloat16):
        x2 = x2.to(torch.float16)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    return x2


def _linear_large(x2: torch.Tensor, trellis: torch.Tensor, suh, svh, K: int, mcg: bool, mul1: bool,
                  y: torch.Tensor) -> None:
    """M > 16: the tcgen05 GEMM (exl3b_gemm), y a [M, n] view with unit column stride."""
    M, k = x2.shape
    n = svh.shape[0]
    if x2.data_ptr() % 16:
        x2 = x2.clone()
    assert y.stride(1) == 1 and y.data_ptr() % 16 == 0 and y.stride(0) % 8 == 0
    ws = reserve_gemm_workspace(x2.device, M, k)
    _lib.call("exl3b_gemm", x2.data_ptr(), M, k, trellis.data_ptr(), n, K, _cb(mcg, mul1), suh.data_ptr(),
              svh.data_ptr(), y.data_ptr(), y.stride(0), ws.data_ptr(), ws.numel(), _stream(x2.device))


# ---------------------------------------------------------------------------------------------
# the custom ops (reference ops.py:65-180)
# ---------------------------------------------------------------------------------------------
def linear_supported(m: int, k: int, n: int, K: int, mcg: bool, mul1: bool) -> bool:
    """Whether the decode GEMV takes an m x k x n call (exl3b_linear_supported; the reference asks
    exl3_gemv_mr_supported the same, ops.py:83)."""
    return bool(_lib.lib().exl3b_linear_supported(m, k, n, K, _cb(mcg, mul1)))


@torch.library.custom_op("exl3rocm::linear", mutates_args=())
def exl3_linear(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor,
                K: int, mcg: bool, mul1: bool) -> torch.Tensor:
    k = x.shape[-1]
    n = svh.shape[0]
    x2 = _prep_x(x, k, keep_bf16=(x.numel() // max(k, 1)) <= GEMV_MAX_ROWS)
    M = x2.shape[0]
    y = torch.empty((M, n), dtype=torch.float16, device=x.device)
    if M == 0:
        return y.view(*x.shape[:-1], n)
    if M <= GEMV_MAX_ROWS:
        linear_into(x2, [trellis], [suh], [svh], K, mcg, mul1, y)
    else:
        _linear_large(x2, trellis, suh, svh, K, mcg, mul1, y)
    return y.view(*x.shape[:-1], n)


@exl3_linear.register_fake
def _(x, trellis, suh, svh, K, mcg, mul1):
    return x.new_empty((*x.shape[:-1], svh.shape[0]), dtype=torch.float16)


@torch.library.custom_op("exl3rocm::linear_groups", mutates_args=())
def exl3_linear_groups(x: torch.Tensor, trellis: list[torch.Tensor], suh: list[torch.Tensor],
                       svh: list[torch.Tensor], K: list[int], mcg: bool, mul1: bool,
                       ptrs_trellis: Optional[torch.Tensor] = None, ptrs_suh: Optional[torch.Tensor] = None,
                       ptrs_svh: Optional[torch.Tensor] = None) -> torch.Tensor:
    """A fused module made of several checkpoint tensors ("groups"), each with its own K, suh and
    svh; the per-group outputs are concatenated inside the op (reference ops.py:106-119).  The
    device pointer tables ``ptrs_*`` of the reference are accepted and unused: the groups' pointers
    travel by value in the kernel parameters."""
    k = x.shape[-1]
    widths = [int(s.shape[0]) for s in svh]
    x2 = _prep_x(x, k, keep_bf16=(x.numel() // max(k, 1)) <= GEMV_MAX_ROWS)
    M = x2.shape[0]
    if len(trellis) == 1:
        return exl3_linear(x, trellis[0], suh[0], svh[0], K[0], mcg, mul1)
    y = torch.empty((M, sum(widths)), dtype=torch.float16, device=x.device)
    if M == 0:
        return y.view(*x.shape[:-1], y.shape[1])
    n0 = 0
    if M <= GEMV_MAX_ROWS:
        # runs of consecutive groups with equal K share one launch (gate/up, q/k/v)
        i = 0
        while i < len(trellis):
            j = i + 1
            while j < len(trellis) and j - i < MAX_GROUPS and K[j] == K[i]:
                j += 1
            w = sum(widths[i:j])
            linear_into(x2, trellis[i:j], suh[i:j], svh[i:j], K[i], mcg, mul1, y[:, n0:n0 + w])
            n0 += w
            i = j
    else:
        for t, su, sv, kk, w in zip(trellis, suh, svh, K, widths):
            _linear_large(x2, t, su, sv, kk, mcg, mul1, y[:, n0:n0 + w])
            n0 += w
    return y.view(*x.shape[:-1], n0)


@exl3_linear_groups.register_fake
def _(x, trellis, suh, svh, K, mcg, mul1, ptrs_trellis=None, ptrs_suh=None, ptrs_svh=None):
    return x.new_empty((*x.shape[:-1], sum(s.shape[0] for s in svh)), dtype=torch.float16)


# ---------------------------------------------------------------------------------------------
# fused epilogues (no reference counterpart: the reference runs the activation and the residual
# add as separate vLLM ops; its own analysis of fusing them: docs/EFFICIENCY_INVESTIGATION.md:36-66)
# ---------------------------------------------------------------------------------------------
def silu_mul(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """SiluAndMul of [.., 2n] -> [.., n]: fp16(fp16(silu(gate)) * up) (exl3b_silu_mul)."""
    n = x.shape[-1] // 2
    x2 = x.reshape(-1, 2 * n)
    assert x2.dtype == torch.float16 and x2.stride(-1) == 1
    if out is None:
        out = torch.empty((*x.shape[:-1], n), dtype=torch.float16, device=x.device)
    o2 = out.view(-1, n)
    _lib.call("exl3b_silu_mul", x2.data_ptr(), x2.stride(0), o2.data_ptr(), o2.stride(0), x2.shape[0], n,
              _stream(x.device))
    return out


@torch.library.custom_op("exl3rocm::gate_up_silu", mutates_args=())
def exl3_gate_up_silu(x: torch.Tensor, trellis: list[torch.Tensor], suh: list[torch.Tensor],
                      svh: list[torch.Tensor], K: int, mcg: bool, mul1: bool) -> torch.Tensor:
    """silu(x @ gate) * (x @ up) for the two EXL3 groups of a SwiGLU MLP, [.., n] fp16.  M <= 16: one
    launch, the activation in the GEMV epilogue; otherwise the grouped route and exl3b_silu_mul."""
    k = x.shape[-1]
    n = int(svh[0].shape[0])
    assert len(trellis) == 2 and int(svh[1].shape[0]) == n
    x2 = _prep_x(x, k, keep_bf16=(x.numel() // max(k, 1)) <= GEMV_MAX_ROWS)
    M = x2.shape[0]
    y = torch.empty((M, n), dtype=torch.float16, device=x.device)
    if M == 0:
        return y.view(*x.shape[:-1], n)
    if M <= GEMV_MAX_ROWS:
        linear_into(x2, trellis, suh, svh, K, mcg, mul1, y, ACT_SILU_MUL)
    else:
        gu = exl3_linear_groups(x2, trellis, suh, svh, [K, K], mcg, mul1)
        silu_mul(gu, y)
    return y.view(*x.shape[:-1], n)


@exl3_gate_up_silu.register_fake
def _(x, trellis, suh, svh, K, mcg, mul1):
    return x.new_empty((*x.shape[:-1], svh[0].shape[0]), dtype=torch.float16)


@torch.library.custom_op("exl3rocm::linear_add_", mutates_args=("residual",))
def exl3_linear_add_(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
                     mcg: bool, mul1: bool, residual: torch.Tensor) -> None:
    """residual = fp16(residual + x @ W) in place (fp16 [.., n] rows of unit stride).  M <= 16: the
    add runs in the GEMV epilogue; otherwise the linear, then one fp16 add."""
    k = x.shape[-1]
    n = int(svh.shape[0])
    x2 = _prep_x(x, k, keep_bf16=(x.numel() // max(k, 1)) <= GEMV_MAX_ROWS)
    M = x2.shape[0]
    r2 = residual.view(-1, n)
    assert residual.dtype == torch.float16 and r2.shape[0] == M and r2.stride(-1) == 1
    if M == 0:
        return
    if M <= GEMV_MAX_ROWS:
        linear_into(x2, [trellis], [suh], [svh], K, mcg, mul1, r2, Y_ADD)
    else:
        r2.add_(exl3_linear(x2, trellis, suh, svh, K, mcg, mul1))


# ---------------------------------------------------------------------------------------------
# fp8 input embedding (reference vllm_plugin/exl3rocm/ops.py:183-202)
# ---------------------------------------------------------------------------------------------
@torch.library.custom_op("exl3rocm::fp8_embedding", mutates_args=())
def fp8_embedding(weight: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """Rows of a float8_e4m3fn table [vocab, hidden] gathered and cast to fp16 (the checkpoint's
    table has no scale), shape [*ids.shape, hidden], by exl3b_fp8_embedding.  An opaque op, as in the
    reference: a compiler tracing the gather would otherwise materialise a cast copy of the table."""
    if weight.dtype != torch.float8_e4m3fn or weight.dim() != 2 or not weight.is_contiguous():
        raise ValueError(f"exl3rocm::fp8_embedding: contiguous 2-d float8_e4m3fn table, not {weight.dtype} "
                         f"{tuple(weight.shape)}")
    flat = ids.reshape(-1)
    if flat.dtype not in (torch.int32, torch.int64):
        flat = flat.to(torch.int64)
    flat = flat.contiguous()
    out = torch.empty((flat.numel(), weight.shape[1]), dtype=torch.float16, device=weight.device)
    _lib.call("exl3b_fp8_embedding", weight.data_ptr(), weight.shape[0], weight.shape[1], flat.data_ptr(),
              1 if flat.dtype == torch.int64 else 0, flat.numel(), out.data_ptr(), _stream(weight.device))
    return out.view(*ids.shape, weight.shape[1])


@fp8_embedding.register_fake
def _(weight, ids):
    return weight.new_empty((*ids.shape, weight.shape[1]), dtype=torch.float16)
