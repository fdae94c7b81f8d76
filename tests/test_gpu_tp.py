"""Row-parallel EXL3 linear with the all-reduce inside the kernel (exl3rocm.tp.linear_tp), on two
GPUs: each rank computes its k-slice and the kernels exchange the fp32 partial sums over peer
memory.  Every rank's output must equal the single-GPU linear of the full weights under the
reference's gates (the fp16 staging is the same; only the fp32 summation order differs), the
ranks' outputs must be identical, and CUDA-graph replays (the call counter lives on the device)
must reproduce the eager result.  Skipped on fewer than two GPUs."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from oracle import exl3_oracle as O

pytestmark = pytest.mark.gpu

GATES = {"normalized_max_abs_err": 3e-3, "normalized_rms_err": 2e-4, "cosine_similarity_min": 0.999999}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stats(got, ref):
    got, ref = got.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    d = got - ref
    scale = np.sqrt(np.mean(ref ** 2)) or 1.0
    return {"normalized_max_abs_err": float(np.abs(d).max() / scale),
            "normalized_rms_err": float(np.sqrt(np.mean(d ** 2)) / scale),
            "cosine_similarity": float(got @ ref / ((np.linalg.norm(got) * np.linalg.norm(ref)) or 1.0))}


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    from exl3rocm import ops
    from exl3rocm.tp import TpComm, linear_tp
    failures = []
    comm = None
    graph = None
    try:
        comm = TpComm(None, dev, max_blocks=40)
        cases = [(1, 5120, 5120, 4), (4, 17408, 5120, 3), (16, 5120, 5120, 2), (1, 17408, 5120, 4)]
        for i, (m, k, n, K) in enumerate(cases):
            rng = np.random.default_rng(100 + i)  # the same full weights on every rank
            tr = O.random_trellis(rng, k // 16, n // 16, K)
            suh = np.sign(rng.standard_normal(k)).astype(np.float16)
            svh = np.sign(rng.standard_normal(n)).astype(np.float16)
            x = (rng.standard_normal((m, k)) * 0.3).astype(np.float16)
            kl = k // world
            sl = slice(rank * kl, (rank + 1) * kl)
            xd = torch.from_numpy(x[:, sl].copy()).to(dev)
            td = torch.from_numpy(tr[rank * kl // 16:(rank + 1) * kl // 16].view(np.int16).copy()).to(dev)
            sd = torch.from_numpy(suh[sl].copy()).to(dev)
            vd = torch.from_numpy(svh).to(dev)
            y = linear_tp(xd, td, sd, vd, K, False, True, comm)
            full = torch.ops.exl3rocm.linear(torch.from_numpy(x).to(dev), torch.from_numpy(tr.view(np.int16)).to(dev),
                                             torch.from_numpy(suh).to(dev), vd, K, False, True)
            torch.cuda.synchronize()
            st = _stats(y.cpu().numpy(), full.cpu().numpy())
            if not (st["normalized_max_abs_err"] <= GATES["normalized_max_abs_err"]
                    and st["normalized_rms_err"] <= GATES["normalized_rms_err"]
                    and st["cosine_similarity"] >= GATES["cosine_similarity_min"]):
                failures.append(f"case {i}: {st}")
            ys = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(ys, y)
            if not all(torch.equal(ys[0], t) for t in ys[1:]):
                failures.append(f"case {i}: ranks differ")
            if ops.workspace_error(dev) != 0:
                failures.append(f"case {i}: workspace error {ops.workspace_error(dev)}")
            if i == len(cases) - 1:
                # graph capture: the call counter advances on the device at every replay
                s = torch.cuda.Stream(dev)
                s.wait_stream(torch.cuda.current_stream(dev))
                ops.reserve_workspace(dev, kl, n, 1, m, stream=s)  # workspaces are per (device, stream)
                with torch.cuda.stream(s):
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=s):
                        yg = linear_tp(xd, td, sd, vd, K, False, True, comm)
                for _ in range(3):
                    graph.replay()
                    torch.cuda.synchronize()
                    if not torch.equal(yg, y):
                        failures.append("graph replay differs from eager")
                        break
        dist.barrier()
    except Exception as e:  # report, then leave in step with the other rank
        failures.append(repr(e))
    finally:
        del graph
        if comm is not None:
            torch.cuda.synchronize()
            dist.barrier()
            comm.close()
        dist.destroy_process_group()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write("\n".join(failures) if failures else "ok")


def test_linear_tp_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = {"NCCL_NVLS_ENABLE": "0"}
    os.environ.update(env)
    torch.multiprocessing.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        msg = (tmp_path / f"rank{r}.txt").read_text()
        assert msg == "ok", msg
