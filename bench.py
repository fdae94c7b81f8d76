"""Benchmark of the EXL3 hot path on B200: decode-regime EXL3 linears (M = 1) of one synthetic
27B-class decoder layer, as the serving engine calls them (qkv and gate_up as grouped modules).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--bits 4] [--m 1]

One step = one pass over the seven EXL3 linears of one layer (q, k, v as one 3-group call; o;
gate, up as one 2-group call; down) at M rows.  Steps rotate over layer copies whose total size
is far above the 126 MB L2, so every step streams its weights from HBM.  value = algorithmic
bytes (packed codes + suh + svh + x + y) / device time, summed over all ranks' shards.

N > 1: tensor parallel over N ranks (one process per GPU, NCCL for the plumbing): q/k/v/gate/up
column-parallel (n sharded in 128-column blocks), o/down row-parallel (k sharded) with the
cross-rank sum inside the GEMV over peer memory (--tp-reduce nccl: an NCCL all-reduce of the fp16
output after it, as vLLM's RowParallelLinear does).  Total work is fixed: scaling "strong".
The `decode` key holds whole-model decode tok/s (exl3rocm.synthetic) at the same GPU count.

--impl reference: times the CPU restatement of the reference's oracle (the reference path has no
GPU implementation that runs here; its kernels are HIP/gfx1201) on the host cores, on a bounded
sample of the same workload, and reports the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen38-27b-exl3-rdna4_b200"))
sys.path.insert(0, ROOT)

METRIC = "EXL3 GEMM HBM GB/s (M=1) & TFLOP/s (M=2048); decode tok/s at 1/2/4/8 B200"
HIDDEN, INTER, HEADS, KV_HEADS, HEAD_DIM = 5120, 17408, 40, 8, 128
# (name, k, n, row_parallel) of one decoder layer; q/k/v and gate/up are grouped modules
LAYER = [("q", HIDDEN, HEADS * HEAD_DIM, False), ("k", HIDDEN, KV_HEADS * HEAD_DIM, False),
         ("v", HIDDEN, KV_HEADS * HEAD_DIM, False), ("o", HEADS * HEAD_DIM, HIDDEN, True),
         ("gate", HIDDEN, INTER, False), ("up", HIDDEN, INTER, False), ("down", INTER, HIDDEN, True)]
MODULES = [("qkv", ["q", "k", "v"]), ("o", ["o"]), ("gate_up", ["gate", "up"]), ("down", ["down"])]
L2_BYTES = 126 * 1024 * 1024

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one gemv_kernel launch of the gate_up
# call at K = 4, m = 1 on one GPU, from one ncu capture.  A capture describes the kernel source it was
# taken from: the figure is reported only while the GEMV sources hash to src_sha256, else null.
GEMV_TRAFFIC = {"src_sha256": "21ad7da65f2c47d3f7366a64bc4b5f81466e75f40a268e6243c7d9aa20189913", "bytes": 91791104}


def gemv_source_sha() -> str:
    import hashlib
    h = hashlib.sha256()
    for f in ("exl3b_gemv.cu", "exl3b_common.cuh"):
        with open(os.path.join(ROOT, "qwen38-27b-exl3-rdna4_b200", "csrc", f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def linear_bytes(k: int, n: int, K: int, m: int) -> int:
    """Algorithmic bytes of one EXL3 linear: codes + suh + svh + x + y (fp16)."""
    return k * n * K // 8 + 2 * k + 2 * n + 2 * m * k + 2 * m * n


def shard_shape(k, n, row_parallel, tp, rank):
    if tp == 1:
        return k, n
    if row_parallel:
        assert k % (128 * tp) == 0
        return k // tp, n
    assert n % (128 * tp) == 0
    return k, n // tp


# ---------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except OSError:
            pass
        finally:
            if self.path and os.path.exists(self.path):
                os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------------
# synthetic layer weights (seeded uniform codes, random +-1 signs), generated on the device
# ---------------------------------------------------------------------------------------------
def make_layer(torch, dev, K, tp, rank, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    out = {}
    for name, k, n, rowp in LAYER:
        ks, ns = shard_shape(k, n, rowp, tp, rank)
        tr = torch.randint(-32768, 32768, (ks // 16, ns // 16, 16 * K), generator=g, device=dev,
                           dtype=torch.int32).to(torch.int16)
        suh = (torch.randint(0, 2, (ks,), generator=g, device=dev) * 2 - 1).to(torch.float16)
        svh = (torch.randint(0, 2, (ns,), generator=g, device=dev) * 2 - 1).to(torch.float16)
        out[name] = (tr, suh, svh, ks, ns)
    return out


def run_layer(torch, layer, x, inputs, K, tp, pg, comm=None):
    """One decoder layer's EXL3 linears as the engine calls them: x feeds qkv and gate_up; the
    row-parallel o and down read their own (sharded) inputs.  Under tensor parallelism o and down
    reduce across ranks inside their kernel (comm), or with an NCCL all-reduce after it (no comm).
    Returns the last output."""
    y = None
    for mod, names in MODULES:
        y = run_module(torch, layer, mod, names, x, inputs, K, tp, pg, comm)
    return y


def run_module(torch, layer, mod, names, x, inputs, K, tp, pg, comm=None):
    """One module of run_layer (qkv, o, gate_up or down); returns its output."""
    ops = torch.ops.exl3rocm
    ts = [layer[nm][0] for nm in names]
    su = [layer[nm][1] for nm in names]
    sv = [layer[nm][2] for nm in names]
    kin = layer[names[0]][3]
    xin = x if kin == x.shape[1] and mod in ("qkv", "gate_up") else inputs[kin]
    if tp > 1 and mod in ("o", "down") and comm is not None:
        from exl3rocm.tp import linear_tp
        return linear_tp(xin, ts[0], su[0], sv[0], K, False, True, comm)
    if len(names) == 1:
        y = ops.linear(xin, ts[0], su[0], sv[0], K, False, True)
    else:
        y = ops.linear_groups(xin, ts, su, sv, [K] * len(names), False, True)
    if tp > 1 and mod in ("o", "down"):
        torch.distributed.all_reduce(y, group=pg)
    return y


def layer_bytes(K, m, tp):
    """Algorithmic bytes of the step's modules summed over all tp shards."""
    total = 0
    names = {nm for _, nms in MODULES for nm in nms}
    for name, k, n, rowp in LAYER:
        if name not in names:
            continue
        for r in range(tp):
            ks, ns = shard_shape(k, n, rowp, tp, r)
            total += linear_bytes(ks, ns, K, m)
    return total


# ---------------------------------------------------------------------------------------------
# CPU baseline: the oracle restatement on the host cores (bounded sample)
# ---------------------------------------------------------------------------------------------
def _cpu_slice(args):
    """One worker's share: generate its column slice (untimed), then time the oracle linear on it.
    Returns (start, end) of the timed call on the host's monotonic clock."""
    k, n_cols, K, seed = args
    from oracle import exl3_oracle as O
    rng = np.random.default_rng(seed)
    tr = O.random_trellis(rng, k // 16, n_cols // 16, K)
    suh = np.sign(rng.standard_normal(k)).astype(np.float16)
    svh = np.sign(rng.standard_normal(n_cols)).astype(np.float16)
    x = rng.standard_normal((1, k)).astype(np.float16)
    t0 = time.perf_counter()
    O.linear(x, tr, K, suh, svh, 2)
    return t0, time.perf_counter()


def _cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(K: int, budget_cols: int = 524288) -> dict:
    """Time the oracle's linear (M=1, mul1) on a column sample of gate_proj-shaped weights (k = 5120),
    one slice per host core in a spawn pool, about ten seconds of host work in all; report the
    metric's unit for that sample.  Only the oracle calls are timed: the span from the first worker's
    start to the last worker's end (pool start-up and code generation excluded)."""
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    per = max(128, (budget_cols // cores) // 128 * 128)
    jobs = [(HIDDEN, per, K, 1000 + i) for i in range(cores)]
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        spans = pool.map(_cpu_slice, jobs)
    compute = max(e for _, e in spans) - min(s for s, _ in spans)
    nbytes = sum(linear_bytes(HIDDEN, per, K, 1) for _ in jobs)
    return {"value": nbytes / compute / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "cpu_model": _cpu_model(),
            "sample": f"oracle linear M=1 mul1 K={K}: {cores} x (5120 x {per}) column slices of gate_proj, "
                      f"process pool, {compute:.1f} s of oracle calls (first start to last end)"}


# ---------------------------------------------------------------------------------------------
# paged KV attention (40 q / 8 kv heads, contexts 4k-64k) and prefill (M = 2048)
# ---------------------------------------------------------------------------------------------
KV_HQ, KV_HKV, KV_D, KV_BS = 40, 8, 128, 16


def _flush_l2(torch, buf):
    buf.add_(1)  # a write larger than L2 between timed calls


def bench_kv(torch, dev, kind: int, ctx: int, batch: int, q_len: int, iters: int = 20) -> dict:
    """Decode (q_len 1) or verify attention over an int8 / int4 cache of `batch` sequences of `ctx`
    tokens, 40 q heads / 8 kv heads, head 128, block 16.  K/V are written through the write kernel
    from N(0,1) rows with 1 % of channels x8.  GB/s counts the cache bytes the call must read."""
    from exl3rocm import kv as xkv
    nblk = batch * ((ctx + KV_BS - 1) // KV_BS)
    row_bytes = KV_D if kind == 8 else KV_D // 2
    kc = torch.empty((nblk, KV_BS, KV_HKV, row_bytes), dtype=torch.int8 if kind == 8 else torch.uint8, device=dev)
    vc = torch.empty_like(kc)
    ks = torch.empty((nblk, KV_BS, KV_HKV), dtype=torch.float32, device=dev)
    vs = torch.empty_like(ks)
    g = torch.Generator(device=dev)
    g.manual_seed(31 + ctx + batch)
    bt = torch.randperm(nblk, generator=g, device=dev).to(torch.int32).view(batch, -1)
    ch = torch.randperm(KV_D, generator=g, device=dev)[: max(1, KV_D // 100)]
    if kind == 4:
        xkv.configure_request_slots(batch)
        xkv._req["slot"] = None
        xkv._exact.pop("bench", None)
        xkv.set_batch_slots(torch.arange(batch, dtype=torch.int32, device=dev))
    chunk = 8192
    for s in range(batch):
        if kind == 4:
            xkv.set_batch_slots(torch.tensor([s], dtype=torch.int32, device=dev))  # this sequence's slot
        for t0 in range(0, ctx, chunk):
            n = min(chunk, ctx - t0)
            k = torch.randn((n, KV_HKV, KV_D), generator=g, device=dev)
            v = torch.randn((n, KV_HKV, KV_D), generator=g, device=dev)
            k[..., ch] *= 8
            v[..., ch] *= 8
            pos = torch.arange(t0, t0 + n, device=dev)
            slots = (bt[s, pos // KV_BS].to(torch.int64) * KV_BS + pos % KV_BS)
            if kind == 8:
                xkv.reshape_and_cache_int8(k.half(), v.half(), kc, vc, slots, ks, vs)
            else:
                xkv.reshape_and_cache(k.half(), v.half(), kc, vc, slots, k_scale_cache=ks, v_scale_cache=vs,
                                      layer_name="bench",
                                      query_start_loc=torch.tensor([0, n], dtype=torch.int32, device=dev),
                                      seq_lens=torch.tensor([t0 + n], dtype=torch.int32, device=dev))
    if kind == 4:
        xkv.set_batch_slots(torch.arange(batch, dtype=torch.int32, device=dev))
    T = batch * q_len
    q = torch.randn((T, KV_HQ, KV_D), generator=g, device=dev).half()
    out = torch.empty_like(q)
    qsl = torch.arange(0, T + 1, q_len, dtype=torch.int32, device=dev)
    sl = torch.full((batch,), ctx, dtype=torch.int32, device=dev)
    fn = xkv.attention_int8 if kind == 8 else xkv.attention
    args = dict(q=q, k=kc, v=vc, out=out, cu_seqlens_q=qsl, max_seqlen_q=q_len, seqused_k=sl, block_table=bt,
                softmax_scale=KV_D ** -0.5, k_scale_cache=ks, v_scale_cache=vs, max_seqlen_k=ctx, layer_name="bench")
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB > L2
    fn(**args)
    # one call captured in a CUDA graph, as a serving engine replays its decode step: the timed
    # region then holds the kernels, not the Python wrapper's host work (which at short contexts
    # took longer than the kernels and left the GPU idle inside the eager measurement)
    call, timing = (lambda: fn(**args)), "eager"
    try:
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn(**args)
            with torch.cuda.graph(graph, stream=side):
                fn(**args)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        call, timing = graph.replay, "graph-replayed"
    except Exception:  # a path that cannot be captured is timed eagerly, and the record says so
        torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        _flush_l2(torch, flush)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        call()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = statistics.median(times)
    kv_bytes = batch * ctx * KV_HKV * (2 * row_bytes + 8)
    del kc, vc, ks, vs, flush
    return {"cache": f"int{kind}", "ctx": ctx, "batch": batch, "q_len": q_len, "ms": ms,
            "gb_s": kv_bytes / (ms * 1e-3) / 1e9, "kv_bytes": kv_bytes, "timing": timing}


def bench_kv_write(torch, dev, kind: int, tokens: int, iters: int = 20) -> dict:
    """One cache write of `tokens` K and V rows (8 kv heads x 128, fp16, N(0,1) with 1 % of channels x8)
    into an int8 or int4 paged cache, slots in a random block order.  GB/s counts the fp16 rows read
    and the codes and scales written."""
    from exl3rocm import kv as xkv
    nblk = (tokens + KV_BS - 1) // KV_BS
    row_bytes = KV_D if kind == 8 else KV_D // 2
    kc = torch.zeros((nblk, KV_BS, KV_HKV, row_bytes), dtype=torch.int8 if kind == 8 else torch.uint8, device=dev)
    vc = torch.zeros_like(kc)
    ks = torch.zeros((nblk, KV_BS, KV_HKV), dtype=torch.float32, device=dev)
    vs = torch.zeros_like(ks)
    g = torch.Generator(device=dev)
    g.manual_seed(57 + tokens)
    k = torch.randn((tokens, KV_HKV, KV_D), generator=g, device=dev)
    v = torch.randn((tokens, KV_HKV, KV_D), generator=g, device=dev)
    ch = torch.randperm(KV_D, generator=g, device=dev)[: max(1, KV_D // 100)]
    k[..., ch] *= 8
    v[..., ch] *= 8
    k, v = k.half(), v.half()
    blk = torch.randperm(nblk, generator=g, device=dev)
    pos = torch.arange(tokens, device=dev)
    slots = blk[pos // KV_BS] * KV_BS + pos % KV_BS
    if kind == 8:
        call = lambda: xkv.reshape_and_cache_int8(k, v, kc, vc, slots, ks, vs)
    else:
        xkv.configure_request_slots(1)
        xkv._req["slot"] = None
        xkv._exact.pop("bench_write", None)
        xkv.set_batch_slots(torch.zeros(1, dtype=torch.int32, device=dev))
        qsl = torch.tensor([0, tokens], dtype=torch.int32, device=dev)
        sl = torch.tensor([tokens], dtype=torch.int32, device=dev)
        call = lambda: xkv.reshape_and_cache(k, v, kc, vc, slots, k_scale_cache=ks, v_scale_cache=vs,
                                             layer_name="bench_write", query_start_loc=qsl, seq_lens=sl)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    call()
    ms = _event_ms(torch, call, iters, flush)
    nbytes = tokens * KV_HKV * (2 * 2 * KV_D + 2 * row_bytes + 8)
    del kc, vc, ks, vs, flush
    return {"cache": f"int{kind}", "tokens": tokens, "ms": ms, "gb_s": nbytes / (ms * 1e-3) / 1e9, "bytes": nbytes}


def bench_decode_ceiling(torch, dev, K: int, iters: int = 4000, reps: int = 5) -> dict:
    """exl3b_decode_ceiling: the GEMV's per-tile decode + mma with the trellis resident in shared
    memory (no HBM, no stage hand-offs), one CTA of 16 warps per SM.  Its tile rate, in the GB/s of
    trellis it would consume at K bits, bounds what this decode can stream from HBM."""
    import ctypes
    from exl3rocm import _lib
    L = _lib.lib()
    g = torch.Generator(device=dev)
    g.manual_seed(41 + K)
    tr = torch.randint(-32768, 32768, (8 * 64 * 16 * K,), generator=g, device=dev, dtype=torch.int32).to(torch.int16)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    out = torch.empty(sms * 512, dtype=torch.float32, device=dev)
    ctas = ctypes.c_int(0)
    st = torch.cuda.current_stream().cuda_stream
    call = lambda: L.exl3b_decode_ceiling(K, 2, tr.data_ptr(), iters, out.data_ptr(), ctypes.byref(ctas), st)
    for _ in range(3):
        rc = call()
        assert rc == 0, rc
    ms = _event_ms(torch, call, reps)
    tiles = ctas.value * 16 * iters * 32
    return {"bits": K, "ctas": ctas.value, "ms": ms, "tiles_per_s": tiles / (ms * 1e-3),
            "gb_s": tiles * 32 * K / (ms * 1e-3) / 1e9, "finite": bool(torch.isfinite(out).all().item())}


def _layer_weights(torch, dev, k, n, K, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    tr = torch.randint(-32768, 32768, (k // 16, n // 16, 16 * K), generator=g, device=dev,
                       dtype=torch.int32).to(torch.int16)
    suh = (torch.randint(0, 2, (k,), generator=g, device=dev) * 2 - 1).half()
    svh = (torch.randint(0, 2, (n,), generator=g, device=dev) * 2 - 1).half()
    return g, tr, suh, svh


def _event_ms(torch, fn, iters, flush=None):
    """Median event-timed duration of fn() on the current stream (a write larger than L2 between
    calls when flush is given)."""
    times = []
    for _ in range(iters):
        if flush is not None:
            _flush_l2(torch, flush)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


def _measured_peaks() -> dict:
    """The pool's measured peaks (MEASURED_PEAKS.json), {} when absent."""
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return {}


def bench_prefill(torch, dev, K: int, m: int = 2048, iters: int = 10, peak_tflops: float = 1590.0) -> dict:
    """One gate_up-shaped EXL3 linear (5120 -> 17408) at M rows through the public op (the tcgen05 GEMM
    of exl3b_gemm: had_in, then the trellis decoded into shared memory feeding tcgen05.mma), with the
    L2 flushed before every call.  Beside it, the reference's own route on this GPU's libraries
    (had_in, reconstruct into a dense fp16 W, cuBLAS GEMM, had_out: ops.py:86-97) on the same inputs,
    for comparison only."""
    from exl3rocm import ops as xops
    g, tr, suh, svh = _layer_weights(torch, dev, HIDDEN, INTER, K, 5)
    x = torch.randn((m, HIDDEN), generator=g, device=dev).to(torch.bfloat16)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    op = lambda: torch.ops.exl3rocm.linear(x, tr, suh, svh, K, False, True)
    op()
    ms = _event_ms(torch, op, iters, flush)
    # the dense-W route of the reference, with cuBLAS (not this library's product path)
    w = torch.empty(HIDDEN, INTER, dtype=torch.float16, device=dev)
    xh = torch.empty((m, HIDDEN), dtype=torch.float16, device=dev)
    y = torch.empty((m, INTER), dtype=torch.float16, device=dev)

    def dense_route():
        xops.had_r_128(x.half(), xh, suh, None, 1.0)
        xops.reconstruct(w, tr, K, False, True)
        torch.mm(xh, w, out=y)
        xops.had_r_128(y, y, None, svh, 1.0)
    dense_route()
    ms_dense = _event_ms(torch, dense_route, iters, flush)
    del w, xh, y, flush
    fl = 2.0 * m * HIDDEN * INTER
    tf = fl / (ms * 1e-3) / 1e12
    return {"m": m, "k": HIDDEN, "n": INTER, "bits": K, "ms": ms, "tflops": tf,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak_tflops, "unit": "TFLOP/s",
                         "frac": tf / peak_tflops, "flops_per_call": fl},
            "route": "exl3b_gemm: had_in, then tcgen05 GEMM (cta_group::2) over trellis decoded in shared memory",
            "dense_w_cublas_route": {"ms": ms_dense, "tflops": fl / (ms_dense * 1e-3) / 1e12}}


SWEEP_SHAPES = [("q/o", HIDDEN, HIDDEN), ("k/v", HIDDEN, KV_HEADS * HEAD_DIM), ("gate/up", HIDDEN, INTER),
                ("down", INTER, HIDDEN)]


def bench_sweep(torch, dev, rows=(1, 4, 8, 16, 128, 2048), bits=(2, 3, 4, 5, 6, 8), iters: int = 10) -> list:
    """The M / bit-width sweep on the layer shapes, through the public op, L2 flushed between calls:
    every M at 4 bits on every shape, and every bit width at M = 1 and M = 2048 on gate/up, all in the
    mul1 codebook (the reference's production one), plus a spot check of 3INST (cb0)
    at M = 1 and 2048 on gate/up.  M <= 16 reports GB/s of algorithmic bytes (HBM-bound GEMV), M >= 128
    TFLOP/s (tensor-bound GEMM)."""
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    points = [(nm, k, n, m, 4, "mul1") for nm, k, n in SWEEP_SHAPES for m in rows]
    points += [("gate/up", HIDDEN, INTER, m, K, "mul1") for K in bits if K != 4 for m in (1, 2048)]
    points += [("gate/up", HIDDEN, INTER, m, 4, "3inst") for m in (1, 2048)]
    out = []
    for nm, k, n, m, K, cb in points:
        g, tr, suh, svh = _layer_weights(torch, dev, k, n, K, 7 + k + n + K)
        x = torch.randn((m, k), generator=g, device=dev).to(torch.bfloat16)
        mul1 = cb == "mul1"
        op = lambda: torch.ops.exl3rocm.linear(x, tr, suh, svh, K, False, mul1)
        op()
        ms = _event_ms(torch, op, iters, flush)
        rec = {"shape": nm, "k": k, "n": n, "m": m, "bits": K, "codebook": cb, "ms": ms}
        if m <= 16:
            rec["gb_s"] = linear_bytes(k, n, K, m) / (ms * 1e-3) / 1e9
        else:
            rec["tflops"] = 2.0 * m * k * n / (ms * 1e-3) / 1e12
        out.append(rec)
        del tr, suh, svh, x
    del flush
    return out


def bench_decode(torch, dev, steps: int, warmup: int, ctx: int = 32768,
                 cases=((1, 1), (8, 1), (1, 4)), world: int = 1, rank: int = 0, comm=None, pg=None) -> list:
    """Decode tokens/s of the synthetic 64-layer 27B-class decoder (exl3rocm.synthetic) with an int8
    paged KV cache of ctx tokens per sequence: (batch, q_len) = (1, 1) and (8, 1) decode, (1, 4) a
    4-token speculative verify.  Each step is one CUDA-graph replay of embed -> 64 layers -> lm_head
    -> argmax, fed the previous step's tokens on the device; timed with CUDA events over `steps`
    replays after `warmup`.  e2e adds, every step, the input tokens from pinned host memory and the
    output tokens back to it.  Weights (9.5 GB) and caches exceed L2 many times over.
    world > 1: tensor parallel over the ranks (exl3rocm.synthetic), times as the max over ranks."""
    from exl3rocm.synthetic import DecoderShape, SyntheticDecoder
    shape = DecoderShape()
    out, base = [], None
    for batch, q_len in cases:
        dec = SyntheticDecoder(shape, dev, batch=batch, q_len=q_len, ctx=ctx, seed=2024, weights_of=base,
                               tp_size=world, tp_rank=rank, comm=comm, group=pg)
        base = base or dec
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        dec.reserve(st)
        tokens = torch.randint(0, shape.vocab, (dec.M,), device=dev)
        with torch.cuda.stream(st):
            dec.step(tokens)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                dec.step(tokens)
                tokens.copy_(dec.next_tokens)  # next step's input, on the device
            for _ in range(warmup):
                graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            if world > 1:
                graph.replay()  # untimed: its exchanges line the ranks' streams up
            e0.record(st)
            for _ in range(steps):
                graph.replay()
            e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        # end to end: host tokens in, host tokens out, every step
        t_host = torch.randint(0, shape.vocab, (dec.M,), dtype=torch.int64).pin_memory()
        o_host = torch.empty(dec.M, dtype=torch.int64).pin_memory()
        with torch.cuda.stream(st):
            if world > 1:
                graph.replay()
            e0.record(st)
            for _ in range(steps):
                tokens.copy_(t_host, non_blocking=True)
                graph.replay()
                o_host.copy_(dec.next_tokens, non_blocking=True)
            e1.record(st)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms, e2e_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=pg)
            ms, e2e_ms = float(t[0]), float(t[1])
        wb, kb = dec.weight_bytes(), dec.kv_bytes()
        out.append({"batch": batch, "q_len": q_len, "ctx": ctx, "ms_per_step": ms,
                    "tok_s": batch / (ms * 1e-3) if q_len == 1 else None,
                    "rows_per_s": dec.M / (ms * 1e-3), "e2e_ms_per_step": e2e_ms,
                    "e2e_tok_s": batch / (e2e_ms * 1e-3) if q_len == 1 else None,
                    "weight_bytes": wb, "kv_bytes": kb, "gb_s": (wb + kb) / (ms * 1e-3) / 1e9,
                    "gpu_launches_per_step": dec.launches_per_step(), "tp": world})
        del graph
        if dec is not base:
            del dec
        torch.cuda.empty_cache()
    del base
    torch.cuda.empty_cache()
    return out


def bench_c5(torch, dev, world: int, rank: int, pg, comm=None, iters: int = 3) -> dict:
    """The tensor-parallel workloads: batch-64 decode with an int4 KV cache of 64k tokens per sequence
    (64 layers: 285 GB of cache in all, so from 2 GPUs on), and an 8192-token prefill of one prompt
    into an int4 cache (GEMM linears, the cache write, prefill attention).  Eager steps, event-timed,
    max over ranks."""
    from exl3rocm.synthetic import DecoderShape, SyntheticDecoder
    shape = DecoderShape()
    out = {}

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier(device_ids=[dev.index])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        if world > 1:
            t = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=pg)
            ms = float(t.item())
        return ms

    # prefill: one 8192-token prompt
    dec = None
    try:
        dec = SyntheticDecoder(shape, dev, batch=1, q_len=1, ctx=8192, seed=2024, tp_size=world, tp_rank=rank,
                               comm=comm, group=pg, kv_cache="int4")
        g = torch.Generator(device=dev)
        g.manual_seed(8192)
        prompt = torch.randint(0, shape.vocab, (8192,), generator=g, device=dev)
        ms = timed(lambda: dec.prefill(prompt))
        h, d, it = shape.hidden, shape.head, shape.intermediate
        weights = h * (shape.q_heads + 2 * shape.kv_heads) * d + shape.q_heads * d * h + 3 * h * it
        fl = 2.0 * 8192 * shape.layers * weights  # 2 M k n over one layer's linears, all layers
        out["prefill_8192_int4"] = {"tokens": 8192, "ms": ms, "tok_s": 8192 / (ms * 1e-3), "tp": world,
                                    "linear_tflops": fl / (ms * 1e-3) / 1e12,
                                    "note": "eager; includes RMSNorm, RoPE, the int4 cache write and prefill attention"}
    except Exception as e:  # reported in the line, same on every rank
        out["prefill_8192_int4"] = {"error": repr(e)[:300]}
    del dec
    torch.cuda.empty_cache()
    if world == 1:
        out["decode_b64_int4_64k"] = {"skipped": "64 layers x 64 sequences x 64k tokens of int4 KV need 285 GB: "
                                                 "measured from 2 GPUs on"}
        return out
    try:
        dec = SyntheticDecoder(shape, dev, batch=64, q_len=1, ctx=65536, seed=2024, tp_size=world, tp_rank=rank,
                               group=pg, kv_cache="int4")
        tokens = torch.randint(0, shape.vocab, (64,), device=dev)
        ms = timed(lambda: dec.step(tokens))
        wb, kb = dec.weight_bytes(), dec.kv_bytes()
        out["decode_b64_int4_64k"] = {"batch": 64, "ctx": 65536, "ms_per_step": ms, "tok_s": 64 / (ms * 1e-3),
                                      "tp": world, "weight_bytes": wb, "kv_bytes": kb,
                                      "gb_s": (wb + kb) / (ms * 1e-3) / 1e9,
                                      "note": "eager; linears through exl3b_gemm (64 rows), int4 split-KV attention"}
        del dec
    except Exception as e:
        out["decode_b64_int4_64k"] = {"error": repr(e)[:300]}
    torch.cuda.empty_cache()
    return out


def parity_check(torch, dev, world: int, rank: int, pg, comm) -> dict:
    """Untimed correctness of what the line measures.  One GPU: a small linear and an int8 attention
    against the CPU oracle.  N GPUs: one decoder layer's linears with weights drawn whole and sharded
    (column-parallel outputs gathered, row-parallel ones reduced inside the GEMV) against the
    single-GPU op on the whole weights, and a 2-layer synthetic decode step's logits at TP N against
    the same model on one GPU.  Gates: nRMS <= 1e-3 and cosine >= 0.99999 for a linear; for the logits,
    which pass two layers of fp16 activations whose o / down sums differ in fp32 order and in where the
    residual add rounds (inside the TP epilogue, against after the single-GPU op), nRMS <= 2e-3."""
    def cmp(got, ref, tol=1e-3):
        got, ref = got.double().flatten(), ref.double().flatten()
        e = float((got - ref).pow(2).mean().sqrt() / ref.pow(2).mean().sqrt())
        c = float(torch.nn.functional.cosine_similarity(got, ref, 0))
        return {"nrms": e, "cos": c, "tol": tol, "ok": bool(e <= tol and c >= 0.99999)}

    res = {}
    if world == 1:
        from oracle import exl3_oracle as O
        rng = np.random.default_rng(3)
        k, n, K = 1024, 512, 4
        tr = O.random_trellis(rng, k // 16, n // 16, K)
        suh = np.sign(rng.standard_normal(k)).astype(np.float16)
        svh = np.sign(rng.standard_normal(n)).astype(np.float16)
        for m in (1, 64):
            x = (rng.standard_normal((m, k)) * 0.3).astype(np.float16)
            y = torch.ops.exl3rocm.linear(torch.from_numpy(x).to(dev), torch.from_numpy(tr.view(np.int16)).to(dev),
                                          torch.from_numpy(suh).to(dev), torch.from_numpy(svh).to(dev), K, False, True)
            res[f"linear_m{m}_vs_oracle"] = cmp(y.cpu(), torch.from_numpy(O.linear(x, tr, K, suh, svh, 2)))
    else:
        from exl3rocm.synthetic import DecoderShape, Layer, SyntheticDecoder
        from exl3rocm.tp import linear_tp
        shape = DecoderShape()
        g1, g2 = torch.Generator(device=dev), torch.Generator(device=dev)
        g1.manual_seed(77)
        g2.manual_seed(77)
        full = Layer(g1, shape, dev)
        part = Layer(g2, shape, dev, tp=world, rank=rank)
        gx = torch.Generator(device=dev)
        gx.manual_seed(78)
        x = torch.randn((4, shape.hidden), generator=gx, device=dev).half()
        xi = torch.randn((4, shape.intermediate), generator=gx, device=dev).half()
        for name in ("q", "gate"):  # column-parallel: gather the ranks' columns
            w, wp = getattr(full, name), getattr(part, name)
            ref = torch.ops.exl3rocm.linear(x, w.trellis, w.suh, w.svh, w.K, False, True)
            mine = torch.ops.exl3rocm.linear(x, wp.trellis, wp.suh, wp.svh, wp.K, False, True).contiguous()
            parts = [torch.empty_like(mine) for _ in range(world)]
            torch.distributed.all_gather(parts, mine, group=pg)
            res[f"{name}_column_parallel"] = cmp(torch.cat(parts, 1), ref)
        for name, xin in (("o", x), ("down", xi)):  # row-parallel: the in-kernel reduction
            w, wp = getattr(full, name), getattr(part, name)
            ref = torch.ops.exl3rocm.linear(xin, w.trellis, w.suh, w.svh, w.K, False, True)
            kl = xin.shape[1] // world
            mine = linear_tp(xin[:, rank * kl:(rank + 1) * kl], wp.trellis, wp.suh, wp.svh, wp.K, False, True, comm)
            res[f"{name}_row_parallel"] = cmp(mine, ref)
        del full, part
        small = DecoderShape(layers=2)
        one = SyntheticDecoder(small, dev, batch=2, q_len=1, ctx=1024, seed=5)
        tpd = SyntheticDecoder(small, dev, batch=2, q_len=1, ctx=1024, seed=5, tp_size=world, tp_rank=rank,
                               comm=comm, group=pg)
        tokens = torch.arange(2, device=dev) * 7919
        one.step(tokens)
        tpd.step(tokens)
        lg = tpd.logits.contiguous()
        sizes = [None] * world
        torch.distributed.all_gather_object(sizes, lg.shape[1], group=pg)
        parts = [torch.empty((lg.shape[0], w), dtype=lg.dtype, device=dev) for w in sizes]
        torch.distributed.all_gather(parts, lg, group=pg)
        res["decode_step_logits"] = cmp(torch.cat(parts, 1), one.logits, 2e-3)
        del one, tpd
        torch.cuda.empty_cache()
    res["ok"] = all(v["ok"] for v in res.values())
    return res


# ---------------------------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--bits", type=int, default=4)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-extra", action="store_true", help="skip the KV-attention, prefill and decode legs")
    ap.add_argument("--no-decode", action="store_true", help="skip the whole-model decode tok/s leg")
    ap.add_argument("--tp-reduce", default="fused", choices=["fused", "nccl"],
                    help="row-parallel reduction under --gpus > 1: inside the GEMV kernel over peer memory, "
                         "or an NCCL all-reduce after it")
    ap.add_argument("--modules", default="qkv,o,gate_up,down",
                    help="comma list of the layer's modules a step runs (default: all four)")
    ap.add_argument("--only", default=None,
                    help="run one leg alone and print its record (for profiler captures): "
                         "kv:<8|4>:<ctx>:<batch>:<q_len>, kv_write:<8|4>:<tokens>, ceiling:<K>, prefill:<K>[:<m>]")
    args = ap.parse_args()
    assert args.warmup >= 3, "at least 3 warm-up steps"
    if args.only:
        import torch
        sys.path.insert(0, os.path.join(ROOT, "qwen38-27b-exl3-rdna4_b200"))
        import exl3rocm.ops  # noqa: F401
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        kind, *a = args.only.split(":")
        if kind == "kv":
            rec = bench_kv(torch, dev, *map(int, a), iters=args.steps)
        elif kind == "kv_write":
            rec = bench_kv_write(torch, dev, *map(int, a), iters=args.steps)
        elif kind == "ceiling":
            rec = bench_decode_ceiling(torch, dev, int(a[0]), reps=args.steps)
        elif kind == "prefill":
            rec = bench_prefill(torch, dev, int(a[0]), m=int(a[1]) if len(a) > 1 else 2048, iters=args.steps,
                                peak_tflops=float(_measured_peaks().get("bf16_tflops", 1590.0)))
        else:
            raise SystemExit(f"unknown leg {kind}")
        print(json.dumps({"only": args.only, **rec}))
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    K, M = args.bits, args.m
    global MODULES
    wanted = args.modules.split(",")
    MODULES = [mod for mod in MODULES if mod[0] in wanted]
    assert MODULES, f"no known module in {args.modules}"

    config = {"workload": f"one 27B-class decoder layer's EXL3 linears ({','.join(m_ for m_, _ in MODULES)}), M={M}, "
                          f"{K} bits, mul1 codebook, x bf16 cast to fp16", "model": "synthetic 27B-class layer",
              "hidden": HIDDEN, "intermediate": INTER, "m": M, "bits": K, "tp": world,
              "parallelism": f"tp{world}" if world > 1 else "single",
              "tp_reduce": (args.tp_reduce if world > 1 else None), "l2": "weights rotate over copies > 2x L2"}

    if args.impl == "reference":
        if rank != 0:
            return
        cb = cpu_baseline(K)
        # each "step" of the reference arm is one bounded CPU sample of the workload
        vals = [cb["value"]]
        for _ in range(max(0, min(args.steps, 2) - 1)):
            vals.append(cpu_baseline(K)["value"])
        v = statistics.median(vals)
        line = {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus, "steps": len(vals),
                "warmup": 0, "ms_per_step": None, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "fp16", "data": "synthetic", "config": config,
                "impl": "reference", "cpu_baseline": dict(cb, value=v),
                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
        pg = torch.distributed.group.WORLD
    import exl3rocm.ops  # noqa: F401  registers torch.ops.exl3rocm.*
    from exl3rocm import ops as xops
    comm = None
    if world > 1 and args.tp_reduce == "fused":
        from exl3rocm.tp import TpComm
        comm = TpComm(pg, dev, max_blocks=HIDDEN // 128)

    one = layer_bytes(K, M, 1) // 1
    copies = max(2, int(np.ceil(3 * L2_BYTES * world / max(1, one))))  # per-rank bytes > 3x L2
    layers = [make_layer(torch, dev, K, world, rank, seed=1234 + 17 * c) for c in range(copies)]
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    x = torch.randn((M, HIDDEN), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    inputs = {layers[0][nm][3]: torch.randn((M, layers[0][nm][3]), generator=g, device=dev,
                                           dtype=torch.float32).to(torch.bfloat16) for nm in ("o", "down")}

    # One CUDA graph per layer copy, as a serving engine replays its decode step.  The graphs read
    # the static input x; e2e refreshes x from pinned host memory and reads y back every step.
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    graphs, outs = [], []
    with torch.cuda.stream(stream):
        for lay in layers:
            for mod, names in MODULES:
                xops.reserve_workspace(dev, lay[names[0]][3], sum(lay[nm][4] for nm in names), len(names), 16)
        for i in range(3):
            run_layer(torch, layers[i % copies], x, inputs, K, world, pg, comm)
        stream.synchronize()
        for lay in layers:
            g_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_, stream=stream):
                outs.append(run_layer(torch, lay, x, inputs, K, world, pg, comm))
            graphs.append(g_)
        # each module alone, for the per-call roofline of the dominant kernel (gate_up) and the
        # per-module times that name the step's limiting kernel
        mod_graphs = {}
        for mod, names in MODULES:
            mod_graphs[mod] = []
            for lay in layers:
                g_ = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g_, stream=stream):
                    run_module(torch, lay, mod, names, x, inputs, K, world, pg, comm)
                mod_graphs[mod].append(g_)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[local])

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs[i % copies].replay()
    torch.cuda.synchronize()

    # ---- device-timed region ----
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk, torch.cuda.stream(stream):
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        if world > 1:
            # one more untimed warm-up step: its in-kernel exchange lines the ranks' streams up, so
            # the host-side skew of leaving the barrier stays out of the timed region
            graphs[args.steps % copies].replay()
        t_start.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            graphs[i % copies].replay()
            ev[i][1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = t_start.elapsed_time(t_end)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    step_ms = [a.elapsed_time(b) for a, b in ev]
    ms_per_step = total_ms / args.steps
    total_bytes = layer_bytes(K, M, world)
    value = total_bytes / (ms_per_step * 1e-3) / 1e9
    clocks = clk.summary()

    # ---- per-call timing of each module, graph-replayed (every rank replays the same calls) ----
    lay = layers[0]
    n_calls = 3 * copies
    mod_ms = {}
    for mod, _ in MODULES:
        ms_l = []
        with torch.cuda.stream(stream):
            for i in range(n_calls):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                mod_graphs[mod][i % copies].replay()
                e1.record(stream)
                torch.cuda.synchronize()
                ms_l.append(e0.elapsed_time(e1))
        mod_ms[mod] = statistics.median(ms_l)
    if world > 1:  # the slowest rank's median per module
        t = torch.tensor([mod_ms[m_] for m_, _ in MODULES], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        mod_ms = {m_: float(v) for (m_, _), v in zip(MODULES, t.tolist())}
    limiting = max(mod_ms, key=mod_ms.get)
    modules_line = {"us": {m_: v * 1000 for m_, v in mod_ms.items()}, "limiting_kernel":
                    f"{limiting} (gemv_kernel{', fused TP exchange' if world > 1 and limiting in ('o', 'down') else ''})",
                    "limiting_share_of_module_sum": mod_ms[limiting] / sum(mod_ms.values())}
    gu_bytes = sum(linear_bytes(lay[nm][3], lay[nm][4], K, M) for nm in ("gate", "up"))
    # the roofline kernel is gate_up's; a run without it (--modules) reports its first module's call
    rl_mod = "gate_up" if "gate_up" in mod_ms else MODULES[0][0]
    gu_ms_med = mod_ms[rl_mod]
    if rl_mod != "gate_up":
        gu_bytes = sum(linear_bytes(lay[nm][3], lay[nm][4], K, M) for nm in dict(MODULES)[rl_mod])
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = gu_bytes / (gu_ms_med * 1e-3) / 1e9
    traffic = GEMV_TRAFFIC["bytes"] if (K == 4 and M == 1 and world == 1 and rl_mod == "gate_up" and
                                         gemv_source_sha() == GEMV_TRAFFIC["src_sha256"]) else None

    # ---- end to end: pinned host x -> device, the layer's ops (graph), y -> pinned host ----
    x_host = torch.randn((M, HIDDEN), dtype=torch.float32).to(torch.bfloat16).pin_memory()
    y_host = torch.empty(outs[0].shape, dtype=outs[0].dtype).pin_memory()
    barrier()
    torch.cuda.synchronize()
    e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        if world > 1:
            graphs[0].replay()  # untimed: its exchanges line the ranks' streams up
        e_s.record(stream)
        for i in range(args.steps):
            x.copy_(x_host, non_blocking=True)
            graphs[i % copies].replay()
            y_host.copy_(outs[i % copies], non_blocking=True)
        e_e.record(stream)
        torch.cuda.synchronize()
    e2e_ms = e_s.elapsed_time(e_e)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = total_bytes / (e2e_ms / args.steps * 1e-3) / 1e9
    del graphs, mod_graphs

    extra = {}
    if world == 1 and not args.no_extra:
        cases = [(kind, ctx, b, 1) for kind in (8, 4) for ctx in (4096, 32768, 65536) for b in (1, 8)]
        cases += [(8, 32768, 1, 4), (4, 32768, 1, 4)]  # speculative verify, 4 query tokens
        extra["kv_attention"] = []
        for kind, ctx, b, ql in cases:
            rec = bench_kv(torch, dev, kind, ctx, b, ql)
            rec["roofline"] = {"bound": "hbm", "frac": rec["gb_s"] / hbm_peak, "peak": hbm_peak, "unit": "GB/s"}
            extra["kv_attention"].append(rec)
            torch.cuda.empty_cache()
        extra["kv_write"] = []
        for kind in (8, 4):
            rec = bench_kv_write(torch, dev, kind, 8192)
            rec["roofline"] = {"bound": "hbm", "frac": rec["gb_s"] / hbm_peak, "peak": hbm_peak, "unit": "GB/s"}
            extra["kv_write"].append(rec)
        extra["decode_ceiling"] = []
        for kb in (2, 3, 4, 5, 6, 8):
            rec = bench_decode_ceiling(torch, dev, kb)
            rec["frac_of_hbm"] = rec["gb_s"] / hbm_peak
            if kb == K:
                rec["gemv_gate_up_frac_of_ceiling"] = achieved / rec["gb_s"]
            extra["decode_ceiling"].append(rec)
        extra["prefill_m2048"] = bench_prefill(torch, dev, K, peak_tflops=float(peaks.get("bf16_tflops", 1590.0)))
        extra["sweep"] = bench_sweep(torch, dev)

    if not args.no_extra and not args.no_decode and (world == 1 or comm is not None):
        del layers, outs, inputs
        torch.cuda.empty_cache()
        try:
            extra["decode"] = bench_decode(torch, dev, steps=max(10, args.steps), warmup=args.warmup, world=world,
                                           rank=rank, comm=comm, pg=pg)
        except Exception as e:  # a shape or setup error is the same on every rank: keep the layer line
            extra["decode"] = {"error": repr(e)[:300]}
            torch.cuda.synchronize()
            torch.cuda.empty_cache()

    if not args.no_extra:
        try:
            extra["c5"] = bench_c5(torch, dev, world, rank, pg, comm)
        except Exception as e:
            extra["c5"] = {"error": repr(e)[:300]}
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
    try:
        extra["parity"] = parity_check(torch, dev, world, rank, pg, comm)
    except Exception as e:
        extra["parity"] = {"ok": False, "error": repr(e)[:300]}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(K)

    if world > 1:
        torch.distributed.barrier(device_ids=[local])
        if comm is not None:
            comm.close()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded uniform trellis codes, +-1 signs, x ~ N(0,1) bf16)", "config": config,
        "step_ms_median": statistics.median(step_ms),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": traffic,
                     "kernel": f"{rl_mod} call (gemv_kernel, graph-replayed), median "
                               f"of {n_calls} event-timed calls, {gu_bytes} algorithmic bytes per call",
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one gemv_kernel "
                                       "launch of this call, captured from the current GEMV source" if traffic
                                       else "null: no ncu capture of the current GEMV source",
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks else "fallback 6650"},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": int(x_host.numel() * 2),
                "d2h_bytes_per_step": int(y_host.numel() * 2)},
        "gpu_launches": args.steps * len(MODULES),
        "modules": modules_line,
        "clocks": clocks,
        **extra,
    }
    print(json.dumps(line))


if __name__ == "__main__":
    main()
