"""Tensor-parallel storage of one EXL3 module (a single checkpoint tensor or a fused run of them).

The reference keeps every group whole and raises when vLLM asks for a partition
(``vllm_plugin/exl3rocm/plugin.py:255-257``).  Here each rank keeps only its part:

* column-parallel (qkv, gate_up, lm_head): the output columns ``n`` of every group are split
  evenly over the ranks, as vLLM's ``output_partition_sizes`` says.  ``had_out`` mixes columns
  only inside a 128-wide block, so a rank stores the 128-blocks that cover its columns (trellis
  ``[:, n-tiles, :]`` and the matching ``svh`` run) and, when its range does not start or end on
  a block edge (vocab 151936 over 8 ranks is 18992 = 148.375 blocks), computes the covering
  blocks and keeps its own columns.  ``x`` and ``suh`` are replicated; nothing is exchanged.
* row-parallel (o_proj, down_proj): the input features ``k`` are split in whole 128-blocks
  (trellis ``[k-tiles, :, :]`` and the ``suh`` run), ``x`` arrives already split, and each rank
  returns the partial output ``y_r = had_out(c_r) * svh``.  ``had_out`` is linear and ``svh``
  is diagonal, so the sum over ranks (the all-reduce the caller runs) is the full output, up to
  fp16 rounding of the partials.

The split is contiguous and balanced: rank ``r`` of ``tp`` owns ``[r * size / tp,
(r + 1) * size / tp)``, vLLM's own convention for ``ColumnParallelLinear`` and
``RowParallelLinear``.  Nothing here needs vLLM, so it is tested with gloo ranks on the CPU.
"""
from __future__ import annotations

import bisect
import itertools

from dataclasses import dataclass, field
from typing import Optional, Sequence

import torch

BLOCK = 128  # Hadamard block: the unit every split must respect on the k side
TILE = 16    # trellis tile edge


def rank_range(size: int, tp_size: int, tp_rank: int) -> tuple[int, int]:
    """[start, end) of rank ``tp_rank``'s even share of ``size``; ``size`` must divide evenly."""
    if tp_size < 1 or not 0 <= tp_rank < tp_size:
        raise ValueError(f"exl3rocm: bad tensor-parallel rank {tp_rank} of {tp_size}")
    if size % tp_size:
        raise ValueError(f"exl3rocm: size {size} does not split evenly over {tp_size} ranks")
    per = size // tp_size
    return tp_rank * per, (tp_rank + 1) * per


def covering_blocks(n0: int, n1: int) -> tuple[int, int]:
    """The 128-aligned column range that covers [n0, n1)."""
    return (n0 // BLOCK) * BLOCK, -(-n1 // BLOCK) * BLOCK


@dataclass
class Group:
    """One checkpoint tensor of a module: its name, bits per weight and full (k, n)."""
    name: str
    K: int
    k: int
    n: int


@dataclass
class GroupShard:
    """What one rank stores of one group."""
    K: int
    k0: int            # first input feature held (row-parallel) -- 0 otherwise
    k1: int
    c0: int            # first stored column (128-aligned)
    c1: int            # end of the stored columns (128-aligned)
    keep0: int         # first output column of this rank, relative to c0
    keep1: int         # end of this rank's output columns, relative to c0
    trellis: Optional[torch.Tensor] = None
    suh: Optional[torch.Tensor] = None
    svh: Optional[torch.Tensor] = None

    @property
    def local_k(self) -> int:
        return self.k1 - self.k0

    @property
    def stored_n(self) -> int:
        return self.c1 - self.c0

    @property
    def out_n(self) -> int:
        return self.keep1 - self.keep0

    @property
    def trimmed(self) -> bool:
        return self.keep0 != 0 or self.keep1 != self.stored_n


@dataclass
class ModuleShard:
    """One rank's part of an EXL3 module.

    ``parallel`` is ``"column"``, ``"row"`` or ``"replicated"``.  ``load(kind, g, tensor)`` takes
    the FULL checkpoint tensor of group ``g`` (``kind`` one of trellis / suh / svh) and stores this
    rank's slice; ``tensors()`` lists what ``torch.ops.exl3rocm.linear_groups`` needs.
    """
    groups: list[Group]
    parallel: str
    tp_size: int = 1
    tp_rank: int = 0
    device: torch.device = field(default_factory=lambda: torch.device("cpu"))
    shards: list[GroupShard] = field(init=False)
    loaded: set = field(init=False, default_factory=set)

    def __post_init__(self):
        if self.parallel not in ("column", "row", "replicated"):
            raise ValueError(f"exl3rocm: unknown parallel mode {self.parallel!r}")
        tp, r = (self.tp_size, self.tp_rank) if self.parallel != "replicated" else (1, 0)
        ks = {g.k for g in self.groups}
        if len(ks) != 1:
            raise ValueError(f"exl3rocm: groups of one module differ in k: {sorted(ks)}")
        self.shards = []
        for g in self.groups:
            if g.k % BLOCK or g.n % BLOCK:
                raise ValueError(f"exl3rocm: {g.name} ({g.k}x{g.n}) is not a multiple of {BLOCK}")
            if self.parallel == "row":
                if g.k % (BLOCK * tp):
                    raise NotImplementedError(
                        f"exl3rocm: row-parallel {g.name} needs k={g.k} to split into whole {BLOCK}-blocks "
                        f"over {tp} ranks")
                k0, k1 = rank_range(g.k, tp, r)
                self.shards.append(GroupShard(g.K, k0, k1, 0, g.n, 0, g.n))
            else:
                n0, n1 = rank_range(g.n, tp, r)
                c0, c1 = covering_blocks(n0, n1)
                self.shards.append(GroupShard(g.K, 0, g.k, c0, c1, n0 - c0, n1 - c0))

    # ---- shapes ------------------------------------------------------------------------------
    @property
    def local_k(self) -> int:
        return self.shards[0].local_k

    @property
    def out_sizes(self) -> list[int]:
        """This rank's output width per group (vLLM's output_partition_sizes for the module)."""
        return [s.out_n for s in self.shards]

    def shapes(self, g: int) -> dict:
        s = self.shards[g]
        return {"trellis": (s.local_k // TILE, s.stored_n // TILE, TILE * s.K),
                "suh": (s.local_k,), "svh": (s.stored_n,)}

    # ---- loading -----------------------------------------------------------------------------
    def slice_full(self, kind: str, g: int, full: torch.Tensor) -> torch.Tensor:
        """This rank's slice of a full checkpoint tensor of group ``g``."""
        grp, s = self.groups[g], self.shards[g]
        if kind == "trellis":
            want = (grp.k // TILE, grp.n // TILE, TILE * grp.K)
            if tuple(full.shape) != want:
                raise ValueError(f"exl3rocm: {grp.name}.trellis shape {tuple(full.shape)}, expected {want}")
            return full[s.k0 // TILE:s.k1 // TILE, s.c0 // TILE:s.c1 // TILE, :]
        if kind == "suh":
            if tuple(full.shape) != (grp.k,):
                raise ValueError(f"exl3rocm: {grp.name}.suh shape {tuple(full.shape)}, expected ({grp.k},)")
            return full[s.k0:s.k1]
        if kind == "svh":
            if tuple(full.shape) != (grp.n,):
                raise ValueError(f"exl3rocm: {grp.name}.svh shape {tuple(full.shape)}, expected ({grp.n},)")
            return full[s.c0:s.c1]
        raise ValueError(f"exl3rocm: unknown tensor kind {kind!r}")

    def load(self, kind: str, g: int, full: torch.Tensor) -> None:
        part = self.slice_full(kind, g, full)
        dtype = torch.int16 if kind == "trellis" else torch.float16
        if kind == "trellis" and part.dtype == torch.uint16:
            part = part.view(torch.int16)
        setattr(self.shards[g], kind, part.to(device=self.device, dtype=dtype).contiguous())
        self.loaded.add((kind, g))

    def missing(self) -> list[tuple[str, int]]:
        return [(k, g) for k in ("trellis", "suh", "svh") for g in range(len(self.groups))
                if (k, g) not in self.loaded]

    def tensors(self):
        return ([s.trellis for s in self.shards], [s.suh for s in self.shards],
                [s.svh for s in self.shards], [s.K for s in self.shards])

    # ---- forward -----------------------------------------------------------------------------
    def local_x(self, x: torch.Tensor) -> torch.Tensor:
        """The input this rank's kernels read: row-parallel modules take x's own k-slice when handed
        the full activation (vLLM hands them the already-split one)."""
        if self.parallel == "row" and x.shape[-1] != self.local_k:
            s = self.shards[0]
            return x[..., s.k0:s.k1]
        return x

    def trim(self, y: torch.Tensor) -> torch.Tensor:
        """Drop covering-block columns that belong to a neighbouring rank."""
        if not any(s.trimmed for s in self.shards):
            return y
        parts, c = [], 0
        for s in self.shards:
            parts.append(y[..., c + s.keep0:c + s.keep1])
            c += s.stored_n
        return torch.cat(parts, dim=-1)

    def forward(self, x: torch.Tensor, mcg: bool, mul1: bool) -> torch.Tensor:
        """This rank's output: its columns (column / replicated) or its partial sum (row)."""
        tr, su, sv, Ks = self.tensors()
        y = torch.ops.exl3rocm.linear_groups(self.local_x(x), tr, su, sv, Ks, mcg, mul1)
        return self.trim(y)

    def forward_groups(self, x: torch.Tensor, groups: Sequence[int], mcg: bool, mul1: bool) -> torch.Tensor:
        """The output columns of the listed groups only, concatenated in their order (untrimmed
        shards: the draft head below)."""
        tr, su, sv, Ks = self.tensors()
        return torch.ops.exl3rocm.linear_groups(self.local_x(x), [tr[g] for g in groups], [su[g] for g in groups],
                                                [sv[g] for g in groups], [Ks[g] for g in groups], mcg, mul1)

    def split_columns(self, cuts: Sequence[int]) -> None:
        """Re-store a loaded one-group, untrimmed shard as consecutive column groups cut at ``cuts``
        (absolute output columns, multiples of 128 strictly inside the stored range), each with its
        own contiguous trellis and svh and the shared suh.  The full output (all groups in order) is
        unchanged; the parts replace the original tensors, so no copy outlives the call."""
        if len(self.shards) != 1 or self.shards[0].trimmed or self.parallel == "row":
            raise ValueError("exl3rocm: split_columns takes one untrimmed column group")
        s, g = self.shards[0], self.groups[0]
        bounds = [s.c0, *cuts, s.c1]
        if any(b % BLOCK for b in cuts) or any(a >= b for a, b in zip(bounds, bounds[1:])):
            raise ValueError(f"exl3rocm: cuts {list(cuts)} do not split columns [{s.c0}, {s.c1}) into 128-blocks")
        parts = []
        for a, b in zip(bounds, bounds[1:]):
            tr = s.trellis[:, (a - s.c0) // TILE:(b - s.c0) // TILE, :].contiguous()
            sv = s.svh[a - s.c0:b - s.c0].contiguous()
            parts.append(GroupShard(s.K, s.k0, s.k1, a, b, 0, b - a, tr, s.suh, sv))
        self.shards = parts
        self.groups = [Group(f"{g.name}[{a}:{b}]", g.K, g.k, b - a) for a, b in zip(bounds, bounds[1:])]
        self.loaded = {(k, i) for k in ("trellis", "suh", "svh") for i in range(len(parts))}


def draft_bounds(n: int, draft_blocks: int, tail_blocks: int = 16) -> Optional[tuple[int, int]]:
    """Columns an MTP drafter scores of an n-column lm_head: the first ``draft_blocks`` 128-column
    blocks (BPE ids run roughly by frequency) and the last ``tail_blocks`` (special and chat tokens),
    as (a, b) for the column ranges [0, a) and [b, n); None when that is the whole head (reference
    plugin.py:431-441)."""
    nb = n // BLOCK
    if draft_blocks <= 0 or draft_blocks + tail_blocks >= nb:
        return None
    return draft_blocks * BLOCK, (nb - tail_blocks) * BLOCK


def partition_owners(partitions: Sequence[int], widths: Sequence[int]) -> list[int]:
    """The group each of vLLM's output partitions falls in, given the groups' output widths on this rank.
    Partitions must tile the groups in order, several partitions may share one group (q, k and v of
    in_proj_qkv inside in_proj_qkvz), and none may straddle two."""
    ends = list(itertools.accumulate(widths))
    owners, start = [], 0
    for p in partitions:
        g = bisect.bisect_right(ends, start)
        if p <= 0 or g >= len(ends) or start + p > ends[g]:
            raise ValueError(f"exl3: vLLM output partitions {list(partitions)} do not tile the module's groups "
                             f"{list(widths)}")
        owners.append(g)
        start += p
    if start != (ends[-1] if ends else 0):
        raise ValueError(f"exl3: vLLM output partitions {list(partitions)} cover {start} of the groups' "
                         f"{ends[-1] if ends else 0} columns")
    return owners


def agree_loaded(shards: Sequence[ModuleShard], group=None) -> None:
    """Every rank checks that it holds all its tensors, then the ranks exchange the verdicts (one
    small all-gather on ``group``), so that a rank whose load failed makes all ranks raise here,
    on the host, instead of leaving its peers blocked in the first row-parallel all-reduce."""
    import torch.distributed as dist
    bad = sum(len(s.missing()) for s in shards)
    if group is None and not (dist.is_available() and dist.is_initialized()):
        if bad:
            raise RuntimeError(f"exl3rocm: {bad} EXL3 tensors were never loaded")
        return
    world = dist.get_world_size(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
        else torch.device("cpu")
    mine = torch.tensor([bad], dtype=torch.int64, device=dev)
    every = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(every, mine, group=group)
    failed = [r for r, t in enumerate(every) if int(t.item())]
    if failed:
        raise RuntimeError(f"exl3rocm: ranks {failed} are missing EXL3 tensors "
                           f"({[int(every[r].item()) for r in failed]} missing)")


def module_shard(groups: Sequence[tuple], parallel: str, tp_size: int, tp_rank: int, device=None) -> ModuleShard:
    """``groups`` as the reference's ``[(member_key, K, k, n)]`` list (plugin.py:133-147)."""
    return ModuleShard([Group(*g) for g in groups], parallel, tp_size, tp_rank,
                       torch.device(device) if device is not None else torch.device("cpu"))
