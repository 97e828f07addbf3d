"""Sharding the quantization of a weight set across GPUs (one process per GPU).

Every unit of the path is independent: the RHT
is per row, E8 groups (256) and trellis segments (T) lie inside rows because
the padded width is a power of two >= 256.  So a weight set is split by
tensor and, for large tensors, by row block; each rank quantizes its share
with the fused device pipelines and no collective runs on the data path.  The
only exchanges are

* one all-gather of every rank's packed trellis codes (the L + R(T-1) bits
  of each sequence), per-256 scales and per-block error sums
  {sum (A-Ah)^2, sum A^2} (``quantize_shards`` + ``gather_codes``): after it
  every rank holds every tensor's codes and weighted NMSE; likewise the
  int16 E8 lattice points of the fixed-step recipe and their error sums
  (``quantize_shards_e8`` + ``gather_e8``),
* an all-gather of the error statistics alone (``gather_errors``), and,
  optionally, assembling a tensor's What on one rank (``assemble_rows``),
* for the calibrated E8 step (qlab.py:171-180), whose 600k-vector sample
  spans the whole tensor: a gather of the sampled normalised vectors to one
  rank, which bisects, and a broadcast of the step.

Resumable runs: with a ``BlockStore``, each finished row block's packed
codes, scales and error sums are saved with a completion marker, and a
re-run (at any world size) loads the finished blocks instead of quantizing
them again -- the sharded counterpart of the builders' per-tensor
``OUT.done`` (buildtrellis.py:22-28, 40).

The plan is deterministic (every rank computes it locally) and balances the
ranks by padded weights x trellis cost per weight.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import numpy as np
import torch

__all__ = ["TensorSpec", "Shard", "plan", "llama_shapes", "run_shards", "gather_errors", "assemble_rows",
           "calibrate_e8", "ShardCodes", "PackedTrellis", "quantize_shards", "gather_codes", "shard_words",
           "BlockStore", "ShardE8", "PackedE8", "quantize_shards_e8", "gather_e8", "shard_words_e8"]


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


@dataclass
class ShardCodes:
    """One row block's trellis output on its rank: packed state paths
    (nseq, words) int32 holding uint32 bit strings, per-group scales (float32),
    error sums [sum (A-Ah)^2, sum A^2] (fp64) and, if kept, What."""
    shard: Shard
    codes: torch.Tensor
    sc: torch.Tensor
    err: torch.Tensor
    What: torch.Tensor | None = None


@dataclass
class PackedTrellis:
    """A whole tensor's trellis codes assembled from its row blocks (row
    order): codes (nseq, words), scales (G,), error sums (2,) summed over the
    blocks in row order, and the weighted NMSE."""
    spec: TensorSpec
    codes: torch.Tensor
    sc: torch.Tensor
    err: torch.Tensor
    seg: int
    group: int

    @property
    def wnmse(self) -> float:
        e = self.err.double().cpu()
        return float(e[0] / e[1])


def shard_words(shard: Shard, seg: int = 256, group: int = 256) -> tuple[int, int, int]:
    """32-bit words of a block's packed codes, scales and error sums in the
    gathered buffer (the padded width is a power of two >= seg and group,
    so blocks of whole rows hold whole sequences and scale groups)."""
    t = shard.tensor
    n = t.padded_cols
    if n % seg or n % group:
        raise ValueError(f"{t.name}: padded width {n} is not a multiple of seg {seg} and group {group}")
    nseq = shard.rows * n // seg
    words = (t.L + t.R * (seg - 1) + 31) // 32
    return nseq * words, shard.rows * n // group, 4


class BlockStore:
    """Completion markers of row blocks for resumable sharded runs.

    ``save`` writes a block's packed codes, scales and error sums to
    ``<root>/<tensor>.<row0>-<row1>.npz`` under a temporary name, renames it
    into place and only then appends the block's key to the rank's marker
    file ``<root>/blocks.<rank>.done`` (flushed and synced), so a marker
    always names a complete file.  The key also holds L, R, seg and group,
    so a run with other parameters does not pick up stale blocks.  ``done``
    reads the markers of every rank (a re-run may use another world size).
    ``load`` checks the sizes against the block's plan and returns None for
    a file that does not match (the block is then quantized again)."""

    def __init__(self, root: str, rank: int = 0):
        self.root = root
        self.rank = rank
        os.makedirs(root, exist_ok=True)
        self._keys = None

    @staticmethod
    def key(shard: Shard, seg: int, group: int) -> str:
        t = shard.tensor
        return f"{t.name}:{shard.row0}:{shard.row1}:L{t.L}:R{t.R}:seg{seg}:g{group}"

    def path(self, shard: Shard) -> str:
        name = shard.tensor.name.replace(os.sep, "_")
        return os.path.join(self.root, f"{name}.{shard.row0}-{shard.row1}.npz")

    def _read_keys(self) -> set:
        keys = set()
        for fn in os.listdir(self.root):
            if fn.startswith("blocks.") and fn.endswith(".done"):
                with open(os.path.join(self.root, fn)) as fh:
                    keys.update(ln.strip() for ln in fh if ln.strip())
        return keys

    def done(self, shard: Shard, seg: int = 256, group: int = 256) -> bool:
        if self._keys is None:
            self._keys = self._read_keys()
        return self.key(shard, seg, group) in self._keys

    def save(self, c: ShardCodes, seg: int = 256, group: int = 256) -> None:
        final = self.path(c.shard)
        tmp = final + f".{os.getpid()}.tmp"
        with open(tmp, "wb") as fh:
            np.savez(fh, codes=c.codes.cpu().numpy(), sc=c.sc.cpu().numpy(),
                     err=c.err.to(torch.float64).cpu().numpy())
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, final)
        k = self.key(c.shard, seg, group)
        with open(os.path.join(self.root, f"blocks.{self.rank}.done"), "a") as fh:
            fh.write(k + "\n")
            fh.flush()
            os.fsync(fh.fileno())
        if self._keys is not None:
            self._keys.add(k)

    def load(self, shard: Shard, device, seg: int = 256, group: int = 256) -> ShardCodes | None:
        try:
            with np.load(self.path(shard)) as z:
                codes, sc, err = z["codes"], z["sc"], z["err"]
        except (OSError, KeyError, ValueError):
            return None
        nc, ns, _ = shard_words(shard, seg, group)
        if (codes.dtype != np.int32 or codes.size != nc or sc.dtype != np.float32 or sc.size != ns
                or err.dtype != np.float64 or err.size != 2):
            return None
        return ShardCodes(shard, torch.from_numpy(codes).to(device), torch.from_numpy(sc).to(device),
                          torch.from_numpy(err).to(device))


def quantize_shards(shards, rank: int, weights, seg: int = 256, group: int = 256,
                    keep_what: bool = False, store: BlockStore | None = None, device=None) -> list[ShardCodes]:
    """Quantize this rank's row blocks with the fused device recipe
    (buildtrellis.py:16-20 around trellis.py:62-108) and pack each block's
    state paths.  ``weights(shard) -> (W rows, H)``: device tensors, or host
    tensors (pinned for asynchronous copies), which are copied in.

    The blocks are launched back to back; the bounded-wait status of all of
    them is checked once at the end (one stream synchronisation), before any
    result leaves the rank, and a timed-out wait raises UQError.

    ``store``: blocks it marks done are loaded onto ``device`` (default: the
    current CUDA device, else the CPU) instead of being quantized; the others
    are saved to it after the status check (What is not kept for loaded
    blocks)."""
    from . import _device as D
    from . import _lib, pipeline, trellis
    out = []
    dev = None
    fresh = []
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    for s in shards:
        if s.rank != rank:
            continue
        if store is not None and store.done(s, seg, group):
            c = store.load(s, device, seg, group)
            if c is not None:
                out.append(c)
                continue
        W, H = weights(s)
        if not W.is_cuda:
            W = D.as_device(W)
        dev = W.device
        res = pipeline.quant_trellis_device(W, H, L=s.tensor.L, R=s.tensor.R, seg=seg, scale_group=group,
                                            keep_codes=True, check_errors=False)
        codes = trellis.pack_states(res.states, s.tensor.L, s.tensor.R)
        out.append(ShardCodes(s, codes, res.sc, res.err, res.What if keep_what else None))
        fresh.append(out[-1])
    if dev is not None:
        _lib.check(_lib.load().uq_device_errors(D.stream_handle(dev)), "quantize_shards")
    if store is not None:
        for c in fresh:
            store.save(c, seg, group)
    return out


def _exchange_device(local_dev, world: int, pg=None):
    """Device of the gathered buffer: the rank's blocks' device, or for a
    rank without blocks the current CUDA device under NCCL (which gathers
    device tensors only), else the CPU."""
    if local_dev is not None:
        return local_dev
    import torch.distributed as dist
    if world > 1 and dist.is_available() and dist.is_initialized() and dist.get_backend(pg) == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _exchange_blocks(parts, shards, world: int, words, dev, pg=None):
    """The one all-gather of block payloads.  ``parts[(tensor, row0)]``: this
    rank's blocks as lists of flat 32-bit tensors whose word counts are
    ``words(shard)``; every rank contributes its blocks in plan order, padded
    to the largest rank's size (every rank knows the plan, so no sizes are
    exchanged).  Returns [(shard, [int32 views of its parts])] for every block
    of every rank."""
    import torch.distributed as dist
    by_rank = [[s for s in shards if s.rank == r] for r in range(world)]
    sizes = [sum(sum(words(s)) for s in blk) for blk in by_rank]
    cap = max(sizes) if sizes else 0
    rank = dist.get_rank(pg) if (world > 1 and dist.is_available() and dist.is_initialized()) else 0
    buf = torch.zeros(max(cap, 1), dtype=torch.int32, device=dev)
    off = 0
    for s in by_rank[rank]:
        for p, nw in zip(parts[(s.tensor.name, s.row0)], words(s)):
            buf[off:off + nw] = p.reshape(-1).view(torch.int32)
            off += nw
    if world > 1:
        allb = torch.empty(world * buf.numel(), dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(allb, buf, group=pg)
    else:
        allb = buf
    out = []
    for r in range(world):
        off = r * buf.numel()
        for s in by_rank[r]:
            views = []
            for nw in words(s):
                views.append(allb[off:off + nw])
                off += nw
            out.append((s, views))
    return out


def gather_codes(local, shards, world: int, seg: int = 256, group: int = 256, pg=None) -> dict:
    """All-gather every rank's packed codes, scales and error sums (one
    collective) and assemble them per tensor in row order on every rank.

    ``shards`` is the whole plan (every rank computes it), so each block's
    place in the gathered buffer is known without exchanging sizes; each rank
    contributes its blocks in plan order, padded to the largest rank's size.
    Error sums are added in row order (deterministic on every rank)."""
    dev = _exchange_device(local[0].codes.device if local else None, world, pg)
    parts = {(c.shard.tensor.name, c.shard.row0): [c.codes, c.sc, c.err.to(torch.float64)] for c in local}
    blocks = _exchange_blocks(parts, shards, world, lambda s: shard_words(s, seg, group), dev, pg)
    out = {}
    for s in shards:
        t = s.tensor
        if t.name in out:
            continue
        words = (t.L + t.R * (seg - 1) + 31) // 32
        nseq = t.rows * t.padded_cols // seg
        ng = t.rows * t.padded_cols // group
        out[t.name] = PackedTrellis(t, torch.empty((nseq, words), dtype=torch.int32, device=dev),
                                    torch.empty(ng, dtype=torch.float32, device=dev),
                                    torch.zeros(2, dtype=torch.float64, device=dev), seg, group)
    errs = {}
    for s, (codes, sc, err) in blocks:
        p = out[s.tensor.name]
        q0 = s.row0 * s.tensor.padded_cols // seg
        g0 = s.row0 * s.tensor.padded_cols // group
        p.codes.view(-1)[q0 * p.codes.shape[1]:q0 * p.codes.shape[1] + codes.numel()] = codes
        p.sc[g0:g0 + sc.numel()] = sc.view(torch.float32)
        errs.setdefault(s.tensor.name, []).append((s.row0, err))
    for name, lst in errs.items():
        acc = out[name].err
        for _, e in sorted(lst, key=lambda v: v[0]):
            acc += e.view(torch.float64)
    return out


# ---- E8 lattice points of row-sharded tensors (qlab.py:159-183, fixed step) ----

@dataclass
class ShardE8:
    """One row block's E8 output on its rank: the int16 lattice coordinates
    2p of its padded rotated rows (rows, n) -- the integer "indices" of
    qlab.py:153 -- error sums [sum (A-Ah)^2, sum A^2] (fp64) and, if kept,
    What."""
    shard: Shard
    idx: torch.Tensor
    err: torch.Tensor
    What: torch.Tensor | None = None


@dataclass
class PackedE8:
    """A whole tensor's E8 points assembled from its row blocks (row order):
    idx (rows, n) int16 = 2p, error sums (2,) summed over the blocks in row
    order, the step, and the weighted NMSE."""
    spec: TensorSpec
    idx: torch.Tensor
    err: torch.Tensor
    step: float

    @property
    def wnmse(self) -> float:
        e = self.err.double().cpu()
        return float(e[0] / e[1])


def shard_words_e8(shard: Shard) -> tuple[int, int]:
    """32-bit words of a block's int16 points (two per word: the padded width
    is a power of two) and error sums in the gathered buffer."""
    return shard.rows * shard.tensor.padded_cols // 2, 4


def quantize_shards_e8(shards, rank: int, weights, step: float, group: int = 256,
                       keep_what: bool = False) -> list[ShardE8]:
    """This rank's row blocks through the fixed-step E8 recipe
    (buildalloc.py:21-24 around qlab.py:159-183), keeping the int16 points.
    ``weights(shard) -> (W rows, H)`` as for ``quantize_shards``; one
    bounded-wait check at the end."""
    from . import _device as D
    from . import _lib, pipeline
    out = []
    dev = None
    for s in shards:
        if s.rank != rank:
            continue
        W, H = weights(s)
        if not W.is_cuda:
            W = D.as_device(W)
        dev = W.device
        res = pipeline.quant_step_device(W, H, step, group=group, keep_codes=True, check_errors=False)
        out.append(ShardE8(s, res.idx.reshape(s.rows, s.tensor.padded_cols), res.err,
                           res.What if keep_what else None))
    if dev is not None:
        _lib.check(_lib.load().uq_device_errors(D.stream_handle(dev)), "quantize_shards_e8")
    return out


def gather_e8(local, shards, world: int, step: float, pg=None) -> dict:
    """All-gather every rank's E8 points and error sums (one collective) and
    assemble them per tensor in row order on every rank; error sums are added
    in row order."""
    dev = _exchange_device(local[0].idx.device if local else None, world, pg)
    parts = {(c.shard.tensor.name, c.shard.row0): [c.idx.contiguous(), c.err.to(torch.float64)] for c in local}
    blocks = _exchange_blocks(parts, shards, world, shard_words_e8, dev, pg)
    out = {}
    for s in shards:
        t = s.tensor
        if t.name not in out:
            out[t.name] = PackedE8(t, torch.empty((t.rows, t.padded_cols), dtype=torch.int16, device=dev),
                                   torch.zeros(2, dtype=torch.float64, device=dev), step)
    errs = {}
    for s, (idx, err) in blocks:
        out[s.tensor.name].idx[s.row0:s.row1] = idx.view(torch.int16).reshape(s.rows, s.tensor.padded_cols)
        errs.setdefault(s.tensor.name, []).append((s.row0, err))
    for name, lst in errs.items():
        acc = out[name].err
        for _, e in sorted(lst, key=lambda v: v[0]):
            acc += e.view(torch.float64)
    return out


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


def _device_sample_gn(A: torch.Tensor, vec_ids: torch.Tensor, group: int) -> torch.Tensor:
    from . import _device as D, _lib
    lib = _lib.load()
    out = torch.empty((vec_ids.numel(), 8), dtype=torch.float64, device=A.device)
    if vec_ids.numel():
        ids = vec_ids.to(A.device, torch.int64).contiguous()
        ws = D.workspace(lib.uq_e8_sample_gn_workspace_bytes(A.numel(), group), A.device)
        _lib.check(lib.uq_e8_sample_gn(A.data_ptr(), D.dtype_code(A), A.numel(), group, ids.data_ptr(), ids.numel(),
                                       out.data_ptr(), ws.data_ptr(), ws.numel(), D.stream_handle(A.device)),
                   "e8 sample gn")
    return out


def _device_bisect(sub: torch.Tensor, target_bpw: float) -> float:
    import ctypes
    from . import _device as D, _lib
    lib = _lib.load()
    sub = sub.to(D.device(), torch.float64).contiguous()
    ws = D.workspace(lib.uq_e8_calibrate_sample_workspace_bytes(sub.shape[0]), sub.device)
    step = ctypes.c_double()
    _lib.check(lib.uq_e8_calibrate_sample(sub.data_ptr(), sub.shape[0], float(target_bpw), ctypes.addressof(step),
                                          ws.data_ptr(), ws.numel(), D.stream_handle(sub.device)), "e8 calibration")
    return float(step.value)


def _sample_indices(nvec: int, ns: int):
    import ctypes
    import numpy as np
    from . import _lib
    out = np.empty(ns, dtype=np.int64)
    _lib.check(_lib.load().uq_e8_sample_indices(nvec, ns, out.ctypes.data_as(ctypes.c_void_p)), "e8 sample indices")
    return out


def calibrate_e8(blocks, spec: TensorSpec, target_bpw: float = 2.0, group: int = 256, root: int = 0,
                 sample_gn=None, bisect=None, pg=None) -> float:
    """The calibrated step of q_e8_fast (qlab.py:171-180) for a tensor split by
    row blocks across ranks, equal to the single-process step: every rank draws
    the same sample of vector ids over the whole tensor (RandomState(0).randint
    (0, nvec, ns), ns = min(600000, nvec)), computes the normalised vectors of
    the ids it holds, `root` places them in sample order and bisects, and the
    step is broadcast.  blocks: [(row0, A_block)] of this rank (rows x
    spec.cols, whole groups: spec.cols % group == 0).  sample_gn(A_block, ids)
    -> (k, 8) fp64 and bisect(sub) -> step default to the device kernels."""
    import numpy as np
    import torch.distributed as dist
    if spec.cols % group or group % 8:
        raise ValueError(f"calibrate_e8: row blocks must hold whole groups (cols={spec.cols}, group={group})")
    sample_gn = sample_gn or (lambda A, ids: _device_sample_gn(A, ids, group))
    bisect = bisect or (lambda sub: _device_bisect(sub, target_bpw))
    nvec = spec.rows * spec.cols // 8
    ns = min(600_000, nvec)
    pick = _sample_indices(nvec, ns)
    vpr = spec.cols // 8                         # vectors per row
    pos_l, gn_l = [], []
    for row0, A in blocks:
        v0, v1 = row0 * vpr, (row0 + A.shape[0]) * vpr
        pos = np.flatnonzero((pick >= v0) & (pick < v1))
        if pos.size:
            gn_l.append(sample_gn(A, torch.from_numpy(pick[pos] - v0)).to(torch.float64).cpu())
            pos_l.append(torch.from_numpy(pos))
    pos = torch.cat(pos_l) if pos_l else torch.zeros(0, dtype=torch.int64)
    gn = torch.cat(gn_l) if gn_l else torch.zeros((0, 8), dtype=torch.float64)
    if not (dist.is_available() and dist.is_initialized()):
        sub = torch.empty((ns, 8), dtype=torch.float64)
        sub[pos] = gn
        return float(bisect(sub))
    rank, world = dist.get_rank(pg), dist.get_world_size(pg)
    dev = (torch.device("cuda", torch.cuda.current_device())
           if dist.get_backend(pg) == "nccl" else torch.device("cpu"))
    n = torch.tensor([pos.numel()], dtype=torch.int64, device=dev)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=pg)
    mx = max(int(x) for x in sizes)
    rec = torch.full((max(mx, 1), 9), -1.0, dtype=torch.float64)
    rec[: pos.numel(), 0] = pos.to(torch.float64)  # ids < 2^53: exact
    rec[: pos.numel(), 1:] = gn
    rec = rec.to(dev)
    allr = [torch.empty_like(rec) for _ in range(world)]
    dist.all_gather(allr, rec, group=pg)
    # the root always broadcasts (NaN when the blocks did not cover the
    # sample exactly once), so every rank leaves the collective together
    step = torch.full((1,), float("nan"), dtype=torch.float64, device=dev)
    got = -1
    if rank == root:
        rows = torch.cat([r.cpu() for r in allr])
        rows = rows[rows[:, 0] >= 0]
        got = rows.shape[0]
        ids = rows[:, 0].to(torch.int64)
        if got == ns and torch.unique(ids).numel() == ns:
            sub = torch.empty((ns, 8), dtype=torch.float64)
            sub[ids] = rows[:, 1:]
            step[0] = bisect(sub)
    dist.broadcast(step, src=root, group=pg)
    if step.isnan().item():
        raise RuntimeError(f"calibrate_e8: the ranks' row blocks do not cover the tensor once "
                           f"({got if rank == root else '?'} of {ns} sampled vectors)")
    return float(step.item())
