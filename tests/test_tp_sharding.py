"""Tensor-parallel sharding of EXL3 modules, on the CPU.

* shapes and split rules for the model's modules at TP 2/4/8, and the errors for splits that
  would cut a 128-wide Hadamard block on the k side;
* column-parallel: each rank's columns, computed by the oracle from the rank's slice only, are
  bitwise the matching columns of the unsharded oracle output (``had_out`` never mixes blocks);
* row-parallel: two gloo ranks each compute their partial output from their k-slice, all-reduce
  it, and match the unsharded oracle within the TP gate below;
* failure path: a rank whose load is incomplete makes every rank raise in ``agree_loaded``.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from exl3rocm import sharding as S
from oracle import exl3_oracle as O

# Row-parallel outputs are the fp16 sum of per-rank fp16 partials, each rounded once more than the
# unsharded output: the gate is the single-GPU gate widened by those roundings.
TP_GATE = {"nrms": 1e-3, "cos": 0.99999, "max_abs": 5e-3}

MODEL = {  # the 27B-class layer: (groups, parallel)
    "qkv": ([("q", 4, 5120, 5120), ("k", 4, 5120, 1024), ("v", 4, 5120, 1024)], "column"),
    "o": ([("o", 4, 5120, 5120)], "row"),
    "gate_up": ([("gate", 4, 5120, 17408), ("up", 4, 5120, 17408)], "column"),
    "down": ([("down", 4, 17408, 5120)], "row"),
    "lm_head": ([("lm_head", 6, 5120, 151936)], "column"),
}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_tensors(rng, groups):
    out = []
    for _, K, k, n in groups:
        tr = O.random_trellis(rng, k // 16, n // 16, K)
        suh = np.sign(rng.standard_normal(k)).astype(np.float16)
        svh = np.sign(rng.standard_normal(n)).astype(np.float16)
        out.append((tr, suh, svh))
    return out


def _load(shard, full):
    for g, (tr, suh, svh) in enumerate(full):
        shard.load("trellis", g, torch.from_numpy(tr.view(np.int16)))
        shard.load("suh", g, torch.from_numpy(suh))
        shard.load("svh", g, torch.from_numpy(svh))


def _oracle_forward(shard, x, cb=2):
    """The rank's output computed by the oracle from the rank's stored tensors only."""
    xs = x if shard.parallel != "row" else x[:, shard.shards[0].k0:shard.shards[0].k1]
    ys = []
    for s in shard.shards:
        y = O.linear(xs, s.trellis.numpy().view(np.uint16), s.K, s.suh.numpy(), s.svh.numpy(), cb)
        ys.append(y[:, s.keep0:s.keep1])
    return np.concatenate(ys, axis=1)


# ---- shapes and rules --------------------------------------------------------------------------
@pytest.mark.parametrize("tp", [1, 2, 4, 8])
@pytest.mark.parametrize("mod", list(MODEL))
def test_model_modules_split(mod, tp):
    groups, par = MODEL[mod]
    per_rank = [S.module_shard(groups, par, tp, r) for r in range(tp)]
    for g, (_, K, k, n) in enumerate(groups):
        if par == "row":
            assert [sh.shards[g].k0 for sh in per_rank] == [r * k // tp for r in range(tp)]
            assert all(sh.shards[g].local_k == k // tp and sh.shards[g].local_k % 128 == 0 for sh in per_rank)
            assert all(sh.shapes(g)["trellis"] == (k // tp // 16, n // 16, 16 * K) for sh in per_rank)
        else:
            # every column owned by exactly one rank, in order
            owned = np.concatenate([np.arange(sh.shards[g].c0 + sh.shards[g].keep0,
                                              sh.shards[g].c0 + sh.shards[g].keep1) for sh in per_rank])
            np.testing.assert_array_equal(owned, np.arange(n))
            for sh in per_rank:
                s = sh.shards[g]
                assert s.c0 % 128 == 0 and s.c1 % 128 == 0 and s.stored_n - s.out_n < 256
                assert sh.shapes(g)["svh"] == (s.stored_n,)
    assert per_rank[0].out_sizes == ([n // tp for _, _, _, n in groups] if par != "row" else [n for *_, n in groups])


def test_exact_block_splits_need_no_trim():
    for mod in ("qkv", "gate_up"):
        groups, par = MODEL[mod]
        for r in range(8):
            assert not any(s.trimmed for s in S.module_shard(groups, par, 8, r).shards)
    lm = S.module_shard(*MODEL["lm_head"], 8, 3)
    assert lm.shards[0].trimmed and lm.out_sizes == [151936 // 8]


def test_bad_splits_raise():
    with pytest.raises(NotImplementedError):
        S.module_shard([("o", 4, 5120, 5120)], "row", 3, 0)        # 5120 / 3 cuts a block
    with pytest.raises(NotImplementedError):
        S.module_shard([("d", 4, 17408, 5120)], "row", 16, 0)      # 1088-wide shards: 8.5 blocks
    with pytest.raises(ValueError):
        S.module_shard([("q", 4, 5120, 5120)], "column", 3, 0)     # uneven columns
    with pytest.raises(ValueError):
        S.module_shard([("q", 4, 5120, 5120), ("x", 4, 2048, 128)], "column", 1, 0)  # k differs
    with pytest.raises(ValueError):
        S.rank_range(256, 2, 2)
    sh = S.module_shard([("q", 4, 256, 256)], "column", 2, 0)
    with pytest.raises(ValueError):
        sh.load("trellis", 0, torch.zeros((16, 8, 64), dtype=torch.int16))  # shard-sized, not full
    with pytest.raises(ValueError):
        sh.load("svh", 0, torch.zeros((128,), dtype=torch.float16))


# ---- column-parallel: bitwise the unsharded columns ---------------------------------------------
@pytest.mark.parametrize("tp", [2, 4])
def test_column_parallel_matches_unsharded_bitwise(tp):
    rng = np.random.default_rng(5)
    groups = [("q", 4, 256, 384), ("k", 3, 256, 128), ("v", 5, 256, 256)]  # q splits mid-block at tp 2, 4
    full = _full_tensors(rng, groups)
    x = (rng.standard_normal((2, 256)) * 0.3).astype(np.float16)
    ref = [O.linear(x, tr, K, suh, svh, 2) for (tr, suh, svh), (_, K, _, _) in zip(full, groups)]
    outs = []
    for r in range(tp):
        sh = S.module_shard(groups, "column", tp, r)
        _load(sh, full)
        assert not sh.missing()
        outs.append(_oracle_forward(sh, x))
    c = 0
    for g, (_, _, _, n) in enumerate(groups):
        w = n // tp
        got = np.concatenate([o[:, c:c + w] for o in outs], axis=1)
        np.testing.assert_array_equal(got.view(np.uint16), ref[g].view(np.uint16))
        c += w


# ---- row-parallel over two gloo ranks ------------------------------------------------------------
def _gates(got, ref):
    got, ref = got.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    scale = np.sqrt(np.mean(ref ** 2))
    d = got - ref
    return {"nrms": np.sqrt(np.mean(d ** 2)) / scale, "max_abs": np.abs(d).max() / scale,
            "cos": got @ ref / (np.linalg.norm(got) * np.linalg.norm(ref))}


def _row_worker(rank, world, port, result_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(9)
        groups = [("down", 4, 1024, 256)]
        full = _full_tensors(rng, groups)
        x = (rng.standard_normal((3, 1024)) * 0.3).astype(np.float16)
        sh = S.module_shard(groups, "row", world, rank)
        _load(sh, full)
        S.agree_loaded([sh])
        y = torch.from_numpy(_oracle_forward(sh, x))
        dist.all_reduce(y)  # fp16 sum, as the serving engine's all-reduce after a row-parallel layer
        if rank == 0:
            ref = O.linear(x, *full[0][:1], 4, full[0][1], full[0][2], 2)
            np.save(os.path.join(result_dir, "row.npy"), np.stack([y.numpy(), ref]))
    finally:
        dist.destroy_process_group()


def test_row_parallel_gloo_allreduce(tmp_path):
    torch.multiprocessing.spawn(_row_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    got, ref = np.load(tmp_path / "row.npy")
    st = _gates(got, ref)
    assert st["nrms"] <= TP_GATE["nrms"] and st["cos"] >= TP_GATE["cos"] and st["max_abs"] <= TP_GATE["max_abs"], st


def _fail_worker(rank, world, port, result_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        groups = [("o", 4, 256, 128)]
        rng = np.random.default_rng(3)
        full = _full_tensors(rng, groups)
        sh = S.module_shard(groups, "row", world, rank)
        for kind, t in zip(("trellis", "suh", "svh"), full[0]):
            if rank == 1 and kind == "svh":
                continue  # rank 1's checkpoint lacks a tensor
            sh.load(kind, 0, torch.from_numpy(t.view(np.int16) if kind == "trellis" else t))
        try:
            S.agree_loaded([sh])
            msg = "no error"
        except RuntimeError as e:
            msg = str(e)
        with open(os.path.join(result_dir, f"r{rank}.txt"), "w") as f:
            f.write(msg)
    finally:
        dist.destroy_process_group()


def test_incomplete_load_fails_on_every_rank(tmp_path):
    torch.multiprocessing.spawn(_fail_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        msg = (tmp_path / f"r{r}.txt").read_text()
        assert "ranks [1]" in msg, msg
