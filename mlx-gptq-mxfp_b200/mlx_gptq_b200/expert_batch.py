"""Routed expert batches, sharded over the GPUs of one box.

One MoE layer's experts are independent: expert e's Hessian depends only on the rows
routed to it, and its solve only on its own H. A batch is therefore partitioned over
the ranks of a process group (one process per GPU) with no data-path collective until
the end, where one all-gather per output tensor hands every rank the codes and E8M0
scales of every expert (what sequential propagation needs). This is the expert split of
the reference's multi-device mode (mlx_gptq/sequential.py:471-474, 610-626: expert
spans spread over devices), done with one process per GPU and NCCL.

Inside a rank the expert Hessians are one grouped tcgen05 launch per parameter. A
routed distribution is skewed (top-k routing with a Zipf bias gives a handful of
experts nearly every token), so an expert holding most of a rank's rows would leave
most SM pairs idle: its rows are cut into pieces, each piece is a separate work item
of the launch (a "virtual expert"), and the pieces are summed afterwards in a fixed
order. Pieces are laid out first-piece-of-every-expert first, so the summed Hessians
are a view of the launch's output, not a copy.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from . import _lib as L
from .capture import hessian_grouped, hessian_spans, hessian_tile_count, hessian_tiles_per_wave
from .pipeline import lpt_partition

# Solve cost of one weight element in Hessian units (one token x one C^2 multiply-add):
# the groupwise MXFP column loop runs ~1.1e11 elements/s on a B200, the Hessian
# ~8e17 multiply-adds/s, so one element costs about as much as 7,000 Hessian units.
SOLVE_UNITS_PER_ELEM = 7.0e3
# An expert without tokens takes the data-free RTN path (layer.solve_experts), a handful
# of small launches costing about 0.1 ms per parameter on a B200 (measured on the C3
# split): about as much as the Hessians of 30,000 tokens of a 2048/768 expert.
RTN_FALLBACK_UNITS = 1.5e11


def plan_experts(counts, world: int, hess_dims, solve_elems: int) -> list[list[int]]:
    """Longest-processing-time split of experts over `world` ranks: cost(e) =
    counts[e] * sum(C^2 over the expert's Hessians) + SOLVE_UNITS_PER_ELEM * elements
    solved per expert (+ RTN_FALLBACK_UNITS for an expert without tokens). Returns the
    sorted expert list of every rank."""
    per_token = float(sum(c * c for c in hess_dims))
    costs = [float(n) * per_token + SOLVE_UNITS_PER_ELEM * solve_elems + (RTN_FALLBACK_UNITS if int(n) == 0 else 0.0)
             for n in counts]
    return lpt_partition(costs, world)


@dataclass
class PieceLayout:
    """Rows of a set of experts cut into pieces for one grouped Hessian launch.

    Pieces 0 .. n-1 are the first pieces of experts[0 .. n-1]; extra[j] = (expert
    position, piece) for the rest (piece n + j). Gather form (rows named by token ids):
    token_idx int32 [rows] on the device, the rows of piece v at offsets[v] ..
    offsets[v + 1] (offsets int64 [V + 1] on the host), and perm int64 [rows] on the
    device with token_idx = (the source index array)[perm], so a fresh copy of the same
    routing is laid out again with one gather. Span form (each expert's rows one
    contiguous block of X): spans[v] = (first row, rows) of piece v, read in place."""
    n: int
    extra: list[tuple[int, int]]
    offsets: torch.Tensor
    token_idx: torch.Tensor | None = None
    perm: torch.Tensor | None = None
    spans: list[tuple[int, int]] | None = None
    merge: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None  # device (targets, piece_ptr, pieces)

    def merge_plan(self, device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None:
        """The extra pieces grouped by expert, in piece order, as device arrays for
        gq_hessian_merge_pieces (built once; None without extra pieces)."""
        if not self.extra:
            return None
        if self.merge is None or self.merge[0].device != torch.device(device):
            by_expert: dict[int, list[int]] = {}
            for j, (i, _) in enumerate(self.extra):
                by_expert.setdefault(i, []).append(self.n + j)
            targets = sorted(by_expert)
            ptr, pieces = [0], []
            for i in targets:
                pieces += by_expert[i]
                ptr.append(len(pieces))
            mk = lambda v: torch.tensor(v, dtype=torch.int64, device=device)
            self.merge = (mk(targets), mk(ptr), mk(pieces))
        return self.merge


def piece_layout(token_idx: torch.Tensor | None, offsets, experts: list[int], c: int, device,
                 waves: float = 4.0, tiles_per_wave: int | None = None) -> PieceLayout:
    """Cut the experts' rows into pieces of at most P rows, P chosen so that the launch
    has about `waves` waves of equally long work items (each piece runs
    hessian_tile_count(c) tiles over its rows; tiles_per_wave defaults to what `device`
    runs at once). Expert e's rows are token_idx[offsets[e]:offsets[e+1]] (gather
    form) or, with token_idx None, rows offsets[e] .. offsets[e+1] of X (span form)."""
    off = [int(v) for v in offsets]
    rows = [off[e + 1] - off[e] for e in experts]
    tiles = hessian_tile_count(c)
    slots = (hessian_tiles_per_wave(device) if tiles_per_wave is None else tiles_per_wave) * waves
    total = sum(rows)
    cap = max(64, -(-total * tiles // int(max(1, slots)))) if total else 64
    cap = -(-cap // 64) * 64  # whole 64-row steps per piece
    first, rest, extra = [], [], []
    for i, (e, n) in enumerate(zip(experts, rows)):
        k = max(1, -(-n // cap))
        bounds = [off[e] + j * n // k for j in range(k + 1)]
        first.append((bounds[0], bounds[1]))
        for j in range(1, k):
            rest.append((bounds[j], bounds[j + 1]))
            extra.append((i, j))
    spans = first + rest
    lens = torch.tensor([b - a for a, b in spans], dtype=torch.int64)
    new_off = torch.zeros(len(spans) + 1, dtype=torch.int64)
    new_off[1:] = torch.cumsum(lens, 0)
    if token_idx is None:
        return PieceLayout(len(experts), extra, new_off, spans=[(a, b - a) for a, b in spans])
    if spans and int(new_off[-1]):
        perm = torch.cat([torch.arange(a, b, dtype=torch.int64) for a, b in spans if b > a]).to(device)
        tok = token_idx.index_select(0, perm)
    else:
        perm = torch.zeros(0, dtype=torch.int64, device=device)
        tok = torch.zeros(1, dtype=torch.int32, device=device)
    return PieceLayout(len(experts), extra, new_off, token_idx=tok, perm=perm)


@torch.no_grad()
def expert_hessians(X: torch.Tensor, layout: PieceLayout, out: torch.Tensor | None = None) -> torch.Tensor:
    """H [n, C, C] float32 of the layout's experts: one grouped launch over all pieces,
    then one launch adding each expert's extra pieces to its first, in piece order."""
    V = layout.offsets.numel() - 1
    if layout.spans is not None:
        H = hessian_spans(X, layout.spans, H=out)
    else:
        H = hessian_grouped(X, layout.token_idx, layout.offsets, V, H=out)
    plan = layout.merge_plan(H.device)
    if plan is not None:  # every expert's extra pieces onto its first, in piece order, one launch
        t, ptr, pieces = plan
        L.check(L.lib().gq_hessian_merge_pieces(L.ptr(H), H.shape[-1], t.numel(), L.ptr(t), L.ptr(ptr),
                                                L.ptr(pieces), L.stream_ptr(H.device)), "hessian_merge_pieces")
    return H[:layout.n]


def _symmetric_memory():
    """torch's symmetric-memory module when it can map peer buffers here, else None.
    The exchange needs only peer mappings, so its buffers are kept out of NVLink
    multicast objects."""
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    try:
        from torch.distributed import _symmetric_memory as symm
    except ImportError:
        return None
    return symm if hasattr(symm, "empty") and hasattr(symm, "rendezvous") else None


class Exchange:
    """Every rank's expert outputs (leading dim = the rank's experts) handed to every
    rank, one buffer per tensor laid out rank-major: rank r's experts fill slots
    r*m .. r*m + n_r - 1 (m = the largest share), slot_of[e] names expert e's slot and
    expert_order() gives the [E, ...] view in expert order.

    On GPUs that map each other's memory (one process per GPU, NVLink) the buffers are
    symmetric allocations and start() pushes this rank's slab into every peer's
    buffer with copy-engine copies on a side stream, so no SM of any rank works on the
    exchange; wait() closes it with a one-element NCCL all-reduce issued after the
    pushes (a rank passes it only once every rank's pushes have landed) and joins the
    side stream. Elsewhere (host tensors, gloo) start() is an asynchronous
    all_gather_into_tensor into the same layout. A buffer must not be read between a
    start() into it and the wait() that follows, nor written by the caller at all."""

    def __init__(self, shares: list[list[int]], rank: int, group, device, push: bool | None = None):
        self.shares, self.rank, self.group = shares, rank, group
        self.world = len(shares)
        self.m = max(len(s) for s in shares)
        self.slot_of = {}
        for r, sh in enumerate(shares):
            for i, e in enumerate(sh):
                self.slot_of[e] = r * self.m + i
        self.E = len(self.slot_of)
        self.device = torch.device(device)
        self.order = torch.tensor([self.slot_of[e] for e in range(self.E)], dtype=torch.long, device=self.device)
        if push is None:
            push = self.device.type == "cuda" and self.world > 1 and _symmetric_memory() is not None
        self.push = push
        self.side = torch.cuda.Stream(device=self.device) if push else None
        self.peers = {}  # buffer data_ptr -> the buffer as mapped on every rank
        self.flag = torch.zeros(1, dtype=torch.int32, device=self.device) if push else None
        self.pending = []

    def buffer(self, tail, dtype) -> torch.Tensor:
        """A rank-major output buffer [world * m, *tail] (symmetric when pushing)."""
        shape = (self.world * self.m,) + tuple(tail)
        if not self.push:
            return torch.empty(shape, dtype=dtype, device=self.device)
        symm = _symmetric_memory()
        t = symm.empty(shape, dtype=dtype, device=self.device)
        h = symm.rendezvous(t, self.group.group_name)
        self.peers[t.data_ptr()] = [t if p == self.rank else h.get_buffer(p, shape, dtype)
                                    for p in range(self.world)]
        return t

    def start(self, t: torch.Tensor, out: torch.Tensor) -> None:
        """Hand this rank's t [n_r, ...] to every rank's out (a buffer() of the same tail)."""
        import torch.distributed as dist

        lo = self.rank * self.m
        if self.push:
            self.side.wait_stream(torch.cuda.current_stream(self.device))  # t is complete
            with torch.cuda.stream(self.side):
                for dst in self.peers[out.data_ptr()]:
                    dst[lo:lo + t.shape[0]].copy_(t)
            t.record_stream(self.side)
            return
        pad = t
        if t.shape[0] != self.m:
            pad = torch.zeros((self.m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
            pad[: t.shape[0]].copy_(t)
        work = dist.all_gather_into_tensor(out, pad.contiguous(), group=self.group, async_op=True)
        self.pending.append((work, pad))

    def wait(self) -> None:
        import torch.distributed as dist

        if self.push:
            with torch.cuda.stream(self.side):
                dist.all_reduce(self.flag, group=self.group, async_op=True).wait()
            torch.cuda.current_stream(self.device).wait_stream(self.side)
            return
        for work, _ in self.pending:
            work.wait()
        self.pending = []

    def expert_order(self, out: torch.Tensor) -> torch.Tensor:
        """out [world * m, ...] -> [E, ...] in expert order (a gather: a new tensor)."""
        return out.index_select(0, self.order)
