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

from dataclasses import dataclass

import torch

from . import _lib as L
from .capture import hessian_grouped, hessian_spans, hessian_tile_count, hessian_tiles_per_wave
from .pipeline import lpt_partition

# Solve cost of one weight element in Hessian units (one token x one C^2 multiply-add):
# the groupwise MXFP column loop runs ~1.1e11 elements/s on a B200, the Hessian
# ~8e17 multiply-adds/s, so one element costs about as much as 7,000 Hessian units.
SOLVE_UNITS_PER_ELEM = 7.0e3


def plan_experts(counts, world: int, hess_dims, solve_elems: int) -> list[list[int]]:
    """Longest-processing-time split of experts over `world` ranks: cost(e) =
    counts[e] * sum(C^2 over the expert's Hessians) + SOLVE_UNITS_PER_ELEM * elements
    solved per expert. Returns the sorted expert list of every rank."""
    per_token = float(sum(c * c for c in hess_dims))
    costs = [float(n) * per_token + SOLVE_UNITS_PER_ELEM * solve_elems for n in counts]
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


class Exchange:
    """All-gather of per-rank expert outputs (leading dim = the rank's experts) into
    expert order on every rank: one padded all_gather_into_tensor per tensor, issued
    asynchronously; a side stream waits for each gather and reorders its result while
    the caller's stream goes on with the work that follows; wait() joins the side
    stream."""

    def __init__(self, shares: list[list[int]], rank: int, group, device):
        self.shares, self.rank, self.group = shares, rank, group
        self.m = max(len(s) for s in shares)
        order = [e for s in shares for e in s]
        self.E = len(order)
        # position of expert e's slab in the gathered [world * m] buffer
        slot = []
        for r, s in enumerate(shares):
            slot += [r * self.m + i for i in range(len(s))]
        self.src = torch.tensor(slot, dtype=torch.long, device=device)
        self.dst = torch.tensor(order, dtype=torch.long, device=device)
        dev = torch.device(device)
        self.side = torch.cuda.Stream(device=dev) if dev.type == "cuda" else None
        self.pending = []

    def start(self, t: torch.Tensor, out: torch.Tensor) -> None:
        """Gather this rank's t [n_r, ...] from every rank into out [E, ...] (expert order)."""
        import torch.distributed as dist

        world = len(self.shares)
        pad = t
        if t.shape[0] != self.m:
            pad = torch.zeros((self.m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
            pad[: t.shape[0]].copy_(t)
        buf = torch.empty((world * self.m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        work = dist.all_gather_into_tensor(buf, pad.contiguous(), group=self.group, async_op=True)
        if self.side is None:  # host tensors (gloo): reorder in wait()
            self.pending.append((work, buf, out, pad))
            return
        self.side.wait_stream(torch.cuda.current_stream(t.device))  # out and the index arrays are ready
        with torch.cuda.stream(self.side):
            work.wait()  # the side stream waits for the gather, the caller's does not
            out.index_copy_(0, self.dst, buf.index_select(0, self.src))
        self.pending.append((None, buf, out, pad))  # buffers live until the caller's stream has joined

    def wait(self) -> None:
        if self.side is not None:
            torch.cuda.current_stream(self.side.device).wait_stream(self.side)
        for work, buf, out, _ in self.pending:
            if work is not None:
                work.wait()
                out.index_copy_(0, self.dst, buf.index_select(0, self.src))
        self.pending = []
