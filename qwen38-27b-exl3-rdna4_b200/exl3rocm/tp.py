"""Tensor-parallel row-parallel EXL3 linear with the all-reduce inside the kernel.

``TpComm(group, device, max_blocks)`` gives every rank of a process group one zeroed communication
buffer and maps all peers' buffers into this process with CUDA IPC (peer memory over NVLink; no
multicast objects).  ``linear_tp(x_local, trellis, suh, svh, K, mcg, mul1, comm)`` then computes this
rank's k-slice of a row-parallel layer (o_proj, down_proj), exchanges the fp32 partial sums of every
128-column block through the peers' buffers and returns the full output on every rank, the same on
all of them.  It replaces the exl3_gemm + all-reduce pair of a row-parallel layer; the reference
runs no tensor parallelism (``vllm_plugin/exl3rocm/plugin.py:255-257``).

All ranks must call ``linear_tp`` on a TpComm in the same order; calls on one rank are ordered by
its stream.  The kernel's waits for peers give up after about a second and leave an error word in
the workspace (``exl3rocm.ops.workspace_error``).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .ops import GEMV_MAX_ROWS, X_BF16, Y_ADD, _cb, _prep_x, _stream, reserve_workspace


class TpComm:
    def __init__(self, group=None, device=None, max_blocks: int = 40, max_rows: int = GEMV_MAX_ROWS):
        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.tp <= _lib.EXL3B_MAX_TP:
            raise ValueError(f"exl3rocm: tensor-parallel size {self.tp} outside 2..{_lib.EXL3B_MAX_TP}")
        self.device = torch.device(device if device is not None else torch.cuda.current_device())
        L = _lib.lib()
        nbytes = int(L.exl3b_tp_comm_bytes(self.tp, max_blocks, max_rows))
        if nbytes == 0:
            raise ValueError("exl3rocm: bad communication buffer shape")
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)  # zeroed before any peer can see it
        h = (ctypes.c_uint8 * _lib.EXL3B_IPC_HANDLE_BYTES)()
        _lib.check("exl3b_ipc_get_handle", L.exl3b_ipc_get_handle(self.buf.data_ptr(), h))
        handles = [None] * self.tp
        dist.all_gather_object(handles, bytes(h), group=group)
        self.comm = _lib.TpComm(self.tp, self.rank, max_blocks, max_rows)
        self._opened = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                self.comm.buffers[r] = self.buf.data_ptr()
                continue
            ptr = ctypes.c_void_p()
            _lib.check("exl3b_ipc_open_handle", L.exl3b_ipc_open_handle((ctypes.c_uint8 * len(hb)).from_buffer_copy(hb),
                                                                        ctypes.byref(ptr)))
            self.comm.buffers[r] = ptr.value
            self._opened.append(ptr.value)
        dist.barrier(group=group)  # every rank mapped every buffer before the first call

    def close(self):
        L = _lib.lib()
        for ptr in self._opened:
            L.exl3b_ipc_close(ptr)
        self._opened = []


def linear_tp(x: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int, mcg: bool,
              mul1: bool, comm: TpComm, residual: torch.Tensor | None = None) -> torch.Tensor:
    """Full output of a row-parallel EXL3 linear from this rank's input slice x [..., k/tp].  With
    `residual` ([M, n] fp16, unit column stride) the summed result is added into it in place (every
    rank holds the same residual and adds the same sum) and returned."""
    k = x.shape[-1]
    n = svh.shape[0]
    x2 = _prep_x(x, k, keep_bf16=True)
    M = x2.shape[0]
    if not 1 <= M <= GEMV_MAX_ROWS:
        raise ValueError(f"exl3rocm: linear_tp takes 1..{GEMV_MAX_ROWS} rows, got {M}")
    if residual is not None:
        y = residual.view(-1, n)
        assert y.dtype == torch.float16 and y.shape[0] == M and y.stride(-1) == 1
    else:
        y = torch.empty((M, n), dtype=torch.float16, device=x.device)
    ws = reserve_workspace(x.device, k, n, 1, max(M, 1))
    cb = _cb(mcg, mul1) | (X_BF16 if x2.dtype == torch.bfloat16 else 0) | (Y_ADD if residual is not None else 0)
    _lib.call("exl3b_linear_tp", x2.data_ptr(), M, k, trellis.data_ptr(), n, K, cb, suh.data_ptr(),
              svh.data_ptr(), y.data_ptr(), y.stride(0), ws.data_ptr(), ws.numel(), ctypes.byref(comm.comm),
              _stream(x.device))
    return y.view(*x.shape[:-1], n)
