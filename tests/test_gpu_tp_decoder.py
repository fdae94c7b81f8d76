"""The synthetic decode step tensor-parallel over two GPUs (exl3rocm.synthetic with tp_size 2).

Both ranks draw the same seeded model and keep their shards; o and down reduce across the ranks
inside the GEMV (exl3b_linear_tp) with the residual add in the same epilogue, and the next tokens
come from an all-gather of the ranks' (max, index) pairs.  Checks: the gathered logits equal the
single-GPU step of the same model within a tolerance (only the fp32 summation order of o and down
differs), the next tokens are the first argmax of the gathered logits and agree across ranks, and
CUDA-graph replays equal the eager step.  Skipped on fewer than two GPUs.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(layers=2, hidden=512, q_heads=4, kv_heads=2, intermediate=1024, vocab=1024)
LOGIT_NRMS = 2e-3
LOGIT_COS = 0.99999


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    from exl3rocm.synthetic import DecoderShape, SyntheticDecoder
    from exl3rocm.tp import TpComm
    failures, comm, graph = [], None, None
    try:
        comm = TpComm(None, dev, max_blocks=40)
        shape = DecoderShape(**SMALL)
        dec = SyntheticDecoder(shape, dev, batch=2, q_len=1, ctx=256, seed=5, tp_size=world, tp_rank=rank,
                               comm=comm, group=dist.group.WORLD)
        tokens = torch.tensor([17, 901], dtype=torch.int64, device=dev)
        dec.step(tokens)
        nxt = dec.next_tokens.clone()
        parts = [torch.empty_like(dec.logits) for _ in range(world)]
        dist.all_gather(parts, dec.logits)
        full = torch.cat(parts, dim=1).float()
        if not torch.equal(nxt, torch.argmax(full, dim=-1)):
            failures.append(f"next tokens {nxt.tolist()} are not the argmax of the gathered logits")
        nx = [torch.empty_like(nxt) for _ in range(world)]
        dist.all_gather(nx, nxt)
        if not all(torch.equal(nx[0], t) for t in nx[1:]):
            failures.append("ranks picked different next tokens")
        dist.barrier()
        if rank == 0:
            ref_dec = SyntheticDecoder(shape, dev, batch=2, q_len=1, ctx=256, seed=5)
            ref_dec.step(tokens)
            ref = ref_dec.logits.float()
            nrms = float((full - ref).pow(2).mean().sqrt() / ref.pow(2).mean().sqrt())
            cos = float(torch.nn.functional.cosine_similarity(full.flatten(), ref.flatten(), dim=0))
            if not (nrms <= LOGIT_NRMS and cos >= LOGIT_COS):
                failures.append(f"tp logits vs single GPU: nrms {nrms}, cos {cos}")
            del ref_dec
        dist.barrier()
        # graph replay: the fused all-reduce's call counter advances on the device
        eager = dec.logits.clone()
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        dec.reserve(st)
        with torch.cuda.stream(st):
            dec.step(tokens)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                dec.step(tokens)
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            if not torch.equal(dec.logits, eager):
                failures.append("graph replay differs from the eager step")
                break
        dist.barrier()
    except Exception as e:  # report, then leave in step with the other rank
        failures.append(repr(e))
    finally:
        del graph
        torch.cuda.synchronize()
        if comm is not None:
            dist.barrier()
            comm.close()
        dist.destroy_process_group()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write("\n".join(failures) if failures else "ok")


def test_tp_decode_step_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ.update({"NCCL_NVLS_ENABLE": "0"})
    torch.multiprocessing.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        msg = (tmp_path / f"rank{r}.txt").read_text()
        assert msg == "ok", msg
