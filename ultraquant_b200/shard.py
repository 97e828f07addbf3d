"""Sharding the quantization of a weight set across GPUs (one process per GPU).

Every unit of the path is independent (SURVEY's multi-GPU analysis): the RHT
is per row, E8 groups (256) and trellis segments (T) lie inside rows because
the padded width is a power of two >= 256.  So a weight set is split by
tensor and, for large tensors, by row block; each rank quantizes its share
with the fused device pipelines and no collective runs on the data path.  The
only exchanges are

* an all-gather of the per-tensor error statistics {sum (A-Ah)^2, sum A^2}
  (weighted NMSE per tensor, whichever ranks held its row blocks), and
* optionally, assembling a tensor's outputs (What, states, scales) on one
  rank with NCCL gathers.

The plan is deterministic (every rank computes it locally) and balances the
ranks by padded weights x trellis cost per weight.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

__all__ = ["TensorSpec", "Shard", "plan", "llama_shapes", "run_shards", "gather_errors", "assemble_rows"]


@dataclass(frozen=True)
class TensorSpec:
    name: str
    rows: int
    cols: int
    L: int = 16
    R: int = 2

    @property
    def padded_cols(self) -> int:
        n = 1
        while n < self.cols:
            n <<= 1
        return n

    def cost(self, rows: int | None = None) -> float:
        """Relative device cost of `rows` rows: padded weights x Viterbi ops/weight."""
        rows = self.rows if rows is None else rows
        ops = 3 * (1 << self.L) + ((1 << self.R) - 1) * (1 << (self.L - self.R))
        return float(rows) * self.padded_cols * ops


@dataclass
class Shard:
    tensor: TensorSpec
    row0: int
    row1: int
    rank: int

    @property
    def rows(self) -> int:
        return self.row1 - self.row0


def plan(specs, world: int, block_rows: int = 512) -> list[Shard]:
    """Assign row blocks of every tensor to ranks, greedily by cost (largest
    blocks first onto the least loaded rank).  Row blocks are multiples of
    `block_rows` (whole trellis segments / E8 groups, since rows are padded to
    a power of two >= 256) except the last block of a tensor."""
    if world < 1:
        raise ValueError("world size must be >= 1")
    blocks = []
    for spec in specs:
        for r0 in range(0, spec.rows, block_rows):
            r1 = min(spec.rows, r0 + block_rows)
            blocks.append((spec.cost(r1 - r0), spec, r0, r1))
    # deterministic: cost desc, then name / row
    blocks.sort(key=lambda b: (-b[0], b[1].name, b[2]))
    load = [0.0] * world
    shards = []
    for c, spec, r0, r1 in blocks:
        rank = min(range(world), key=lambda r: (load[r], r))
        load[rank] += c
        shards.append(Shard(spec, r0, r1, rank))
    shards.sort(key=lambda s: (s.rank, s.tensor.name, s.row0))
    return shards


def llama_shapes(layers: int = 32, hidden: int = 4096, kv: int = 1024, ffn: int = 14336,
                 k_by_type=None, L: int = 16) -> list[TensorSpec]:
    """Llama-shaped linear weight set (out, in).  Default allocation: k=3 on
    ffn_down / attn_q / attn_output, k=2 elsewhere."""
    k_by_type = k_by_type or {"attn_q": 3, "attn_k": 2, "attn_v": 2, "attn_output": 3,
                              "ffn_gate": 2, "ffn_up": 2, "ffn_down": 3}
    shapes = {"attn_q": (hidden, hidden), "attn_k": (kv, hidden), "attn_v": (kv, hidden),
              "attn_output": (hidden, hidden), "ffn_gate": (ffn, hidden), "ffn_up": (ffn, hidden),
              "ffn_down": (hidden, ffn)}
    out = []
    for li in range(layers):
        for typ, (r, c) in shapes.items():
            out.append(TensorSpec(f"blk.{li}.{typ}.weight", r, c, L=L, R=k_by_type[typ]))
    return out


@dataclass
class ShardResult:
    shard: Shard
    What: torch.Tensor
    err: torch.Tensor                     # [2] fp64
    extras: dict = field(default_factory=dict)


def run_shards(shards, rank: int, make_weights, quantize) -> list[ShardResult]:
    """Quantize this rank's shards.  make_weights(spec, row0, row1) -> (W, H)
    on this rank's device; quantize(spec, W, H) -> (What, err[2])."""
    out = []
    for s in shards:
        if s.rank != rank:
            continue
        W, H = make_weights(s.tensor, s.row0, s.row1)
        What, err = quantize(s.tensor, W, H)
        out.append(ShardResult(s, What, err))
    return out


def gather_errors(results, specs, group=None) -> dict:
    """All-gather the per-shard error sums and reduce them per tensor in a
    fixed order (tensor, row0), so every rank gets identical weighted NMSEs."""
    import torch.distributed as dist
    names = {s.name: i for i, s in enumerate(specs)}
    dev = results[0].err.device if results else (torch.device("cuda", torch.cuda.current_device())
                                                 if torch.cuda.is_available() else torch.device("cpu"))
    # rows: (tensor index, row0, sum_err, sum_ref) per shard of this rank
    local = torch.tensor([[names[r.shard.tensor.name], r.shard.row0, float(r.err[0]), float(r.err[1])]
                          for r in results] or [[-1.0, -1.0, 0.0, 0.0]], dtype=torch.float64)
    if dist.is_available() and dist.is_initialized():
        world = dist.get_world_size(group)
        n = torch.tensor([local.shape[0]], dtype=torch.int64, device=dev)
        sizes = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(sizes, n, group=group)
        mx = int(max(int(x) for x in sizes))
        pad = torch.full((mx, 4), -1.0, dtype=torch.float64)
        pad[: local.shape[0]] = local
        pad = pad.to(dev)
        allp = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(allp, pad, group=group)
        rows = torch.cat([p.cpu() for p in allp])
    else:
        rows = local
    rows = rows[rows[:, 0] >= 0]
    order = sorted(range(rows.shape[0]), key=lambda i: (int(rows[i, 0]), int(rows[i, 1])))
    acc: dict = {}
    for i in order:
        name = specs[int(rows[i, 0])].name
        e, a = acc.get(name, (0.0, 0.0))
        acc[name] = (e + float(rows[i, 2]), a + float(rows[i, 3]))
    return {k: (e / a if a else float("nan")) for k, (e, a) in acc.items()}


def assemble_rows(results, spec: TensorSpec, dst_rank: int = 0, group=None):
    """Gather the row blocks of `spec` (What) onto dst_rank; returns the full
    (rows, cols) tensor there and None elsewhere.  Uses point-to-point NCCL /
    gloo sends of each block (the only data-path exchange, on demand)."""
    import torch.distributed as dist
    mine = {r.shard.row0: r for r in results if r.shard.tensor.name == spec.name}
    if not (dist.is_available() and dist.is_initialized()):
        full = torch.empty((spec.rows, spec.cols), dtype=torch.float32)
        for r0, r in mine.items():
            full[r0:r0 + r.shard.rows] = r.What.cpu()
        return full
    rank = dist.get_rank(group)
    blocks = plan_blocks_for(spec, results, group)
    if rank == dst_rank:
        dev = next(iter(mine.values())).What.device if mine else torch.device("cpu")
        full = torch.empty((spec.rows, spec.cols), dtype=torch.float32, device=dev)
        for r0, (r1, owner) in sorted(blocks.items()):
            if owner == rank:
                full[r0:r1] = mine[r0].What
            else:
                buf = torch.empty((r1 - r0, spec.cols), dtype=torch.float32, device=dev)
                dist.recv(buf, src=owner, group=group)
                full[r0:r1] = buf
        return full
    for r0, (r1, owner) in sorted(blocks.items()):
        if owner == rank:
            dist.send(mine[r0].What.contiguous(), dst=dst_rank, group=group)
    return None


def plan_blocks_for(spec, results, group=None) -> dict:
    """row0 -> (row1, owner rank) for all blocks of `spec` (all-gathered)."""
    import torch.distributed as dist
    local = [(r.shard.row0, r.shard.row1, r.shard.rank) for r in results if r.shard.tensor.name == spec.name]
    world = dist.get_world_size(group)
    gathered = [None] * world
    dist.all_gather_object(gathered, local, group=group)
    out = {}
    for lst in gathered:
        for r0, r1, owner in lst:
            out[r0] = (r1, owner)
    return out
