"""Calibration input capture and the Hessian accumulation (tensor cores).

Mirrors mlx_gptq/capture.py of the reference: ``Stash`` (add / add_sampled /
nbytes / hessian / clear) and ``CaptureManager`` (nn.Linear pre-hooks with
same-input dedup, fused-expert interception of ``F.linear`` by weight-slice
data pointer, unrouted-expert backfill, token statistics). Differences, all on
the B200 side of the boundary:

* stashes keep their rows on the device they were produced on by default
  (``stash_device=None``) instead of copying every batch to host memory; pass
  ``stash_device="cpu"`` for the reference's memory profile;
* ``Stash.hessian`` forms H = X^T X in float32 with the tcgen05 kernel instead of
  float32 ``addmm`` per 65,536-row chunk (capture.py:68-76);
* ``CaptureManager.expert_hessians`` builds every expert's Hessian of a fused
  parameter in one grouped launch.
"""

from __future__ import annotations

import contextlib
import logging
import re
import threading
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch.overrides import TorchFunctionMode

from . import _lib as L

log = logging.getLogger(__name__)

# 3D expert parameter names understood, per the transformers fused layout (capture.py:30)
FUSED_EXPERT_PARAMS = ("gate_up_proj", "gate_proj", "up_proj", "down_proj")


def hessian_tile_count(c: int) -> int:
    """Output tiles of the Hessian kernel for c features (see hessian_accumulate's `tiles`)."""
    return int(L.lib().gq_hessian_tile_count(int(c)))


def hessian_tiles_per_wave(device=None) -> int:
    """Output tiles the Hessian kernel runs at once on `device`."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return int(L.lib().gq_hessian_concurrent_tiles(torch.cuda.get_device_properties(dev).multi_processor_count))


@torch.no_grad()
def hessian_accumulate(X: torch.Tensor, H: torch.Tensor, alpha: float = 1.0, beta: float = 1.0,
                       status: torch.Tensor | None = None, tiles: tuple[int, int] | None = None) -> torch.Tensor:
    """H = beta * H + alpha * X^T X for bf16 rows X [n, c] and float32 H [c, c], both on
    the same CUDA device. Returns H. With tiles=(begin, end) only the blocks of those
    output tiles (of hessian_tile_count(c)) are written, bit-identical to a full call.
    status: int32 device word for the kernel's bounded waits; default: the device's
    library status word, read by the solvers (and Stash.hessian) before H is used."""
    L.require_cuda(X, H)
    if X.dtype != torch.bfloat16:
        raise ValueError("X must be bfloat16 (the capture dtype)")
    if X.dim() != 2 or H.shape != (X.shape[1], X.shape[1]) or H.dtype != torch.float32:
        raise ValueError("shapes: X [n, c] bf16, H [c, c] float32")
    if X.stride(1) != 1 or X.stride(0) % 8 or X.data_ptr() % 16:
        X = X.contiguous()
        if X.stride(0) % 8 or X.data_ptr() % 16:
            raise ValueError("X rows must be 16-byte aligned (in_features % 8 == 0)")
    if H.stride(1) != 1 or H.stride(0) % 4 or H.data_ptr() % 16:
        raise ValueError("H must be row-major, 16-byte aligned, row stride % 4 == 0")
    n, c = X.shape
    if status is None:
        status = L.status_word(X.device)
    if tiles is None:
        L.check(L.lib().gq_hessian_bf16(L.ptr(X), n, c, X.stride(0), L.ptr(H), H.stride(0), float(alpha),
                                        float(beta), L.ptr(status), L.stream_ptr(X.device)), "hessian")
    else:
        L.check(L.lib().gq_hessian_bf16_range(L.ptr(X), n, c, X.stride(0), L.ptr(H), H.stride(0), float(alpha),
                                              float(beta), int(tiles[0]), int(tiles[1]), L.ptr(status),
                                              L.stream_ptr(X.device)), "hessian")
    return H


@torch.no_grad()
def hessian_from_rows(X: torch.Tensor) -> torch.Tensor:
    """H = X^T X (float32) for device-resident bf16 rows X [n, c]."""
    c = X.shape[1]
    H = torch.empty(c, c, dtype=torch.float32, device=X.device)
    hessian_accumulate(X, H, 1.0, 0.0)
    L.raise_on_device_timeout(X.device)
    return H


@torch.no_grad()
def hessian_grouped(X: torch.Tensor, token_idx: torch.Tensor, offsets: torch.Tensor, num_experts: int,
                    H: torch.Tensor | None = None, alpha: float = 1.0, beta: float = 0.0) -> torch.Tensor:
    """Per-expert H[e] = beta*H[e] + alpha * X[rows_e]^T X[rows_e] in one launch, with
    rows_e = token_idx[offsets[e]:offsets[e+1]] (the per-expert stashes of the reference's
    capture, as token indices into the layer input X bf16 [n, c] instead of row copies).
    offsets: int64 [E+1] (any device). Returns H float32 [E, c, c]."""
    L.require_cuda(X)
    if X.dtype != torch.bfloat16 or X.dim() != 2:
        raise ValueError("X must be bfloat16 [n, c]")
    n, c = X.shape
    if X.stride(1) != 1 or X.stride(0) % 8 or X.data_ptr() % 16:
        X = X.contiguous()
    off_host = offsets.detach().to("cpu", torch.int64).contiguous()
    if off_host.numel() != num_experts + 1:
        raise ValueError("offsets must have num_experts + 1 entries")
    off_dev = off_host.to(X.device)
    idx = token_idx.to(X.device, torch.int32).contiguous()
    if H is None:
        H = torch.empty(num_experts, c, c, dtype=torch.float32, device=X.device)
    lib = L.lib()
    ws_bytes = lib.gq_hessian_grouped_workspace_size(off_host.data_ptr(), num_experts, c)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=X.device)
    L.check(lib.gq_hessian_grouped_bf16(L.ptr(X), n, c, X.stride(0), L.ptr(idx), L.ptr(off_dev),
                                        off_host.data_ptr(), num_experts, L.ptr(H), float(alpha), float(beta),
                                        L.ptr(ws), ws.numel(), L.ptr(L.status_word(X.device)),
                                        L.stream_ptr(X.device)), "hessian_grouped")
    return H


@torch.no_grad()
def hessian_spans(X: torch.Tensor, spans, H: torch.Tensor | None = None, alpha: float = 1.0,
                  beta: float = 0.0) -> torch.Tensor:
    """Per-expert H[e] = beta*H[e] + alpha * X[a:a+k]^T X[a:a+k] for spans[e] = (a, k), in one
    launch, reading the rows in place (an expert's stash as one contiguous block of
    rows). X: bf16 [n, c] on a CUDA device. Returns H float32 [E, c, c]."""
    L.require_cuda(X)
    if X.dtype != torch.bfloat16 or X.dim() != 2:
        raise ValueError("X must be bfloat16 [n, c]")
    if X.stride(1) != 1 or X.stride(0) % 8 or X.data_ptr() % 16:
        X = X.contiguous()
    n, c = X.shape
    sp = torch.tensor([[int(a), int(k)] for a, k in spans], dtype=torch.int64).reshape(-1, 2).contiguous()
    E = sp.shape[0]
    if H is None:
        H = torch.empty(E, c, c, dtype=torch.float32, device=X.device)
    lib = L.lib()
    ws = torch.empty(lib.gq_hessian_spans_workspace_size(sp.data_ptr(), E, c), dtype=torch.uint8, device=X.device)
    L.check(lib.gq_hessian_spans_bf16(L.ptr(X), n, c, X.stride(0), sp.data_ptr(), E, L.ptr(H), float(alpha),
                                      float(beta), L.ptr(ws), ws.numel(), L.ptr(L.status_word(X.device)),
                                      L.stream_ptr(X.device)), "hessian_spans")
    return H


class Stash:
    """Captured input rows for one logical weight matrix (capture.py:33-79)."""

    def __init__(self, name: str, in_features: int, device=None):
        self.name = name
        self.in_features = in_features
        self.device = device  # None: keep rows where they were produced
        self.chunks: list[torch.Tensor] = []
        self.tokens = 0

    def add(self, x: torch.Tensor):
        rows = x.detach().reshape(-1, x.shape[-1])
        if rows.shape[-1] != self.in_features:
            raise RuntimeError(
                f"stash {self.name}: got rows of dim {rows.shape[-1]}, expected {self.in_features}")
        dev = rows.device if self.device is None else torch.device(self.device)
        same = dev == rows.device and rows.dtype == torch.bfloat16
        self.chunks.append(rows.clone() if same else rows.to(dev, torch.bfloat16))
        self.tokens += rows.shape[0]

    def rows(self, device) -> torch.Tensor:
        """All stashed rows as one bf16 [tokens, in_features] tensor on `device`."""
        if not self.chunks:
            return torch.empty(0, self.in_features, dtype=torch.bfloat16, device=device)
        return torch.cat([c.to(device) for c in self.chunks], dim=0)

    def add_sampled(self, x: torch.Tensor, max_rows: int):
        """Deterministic, evenly spaced sample of input rows (capture.py:52-63)."""
        rows = x.detach().reshape(-1, x.shape[-1])
        if rows.shape[0] > max_rows:
            idx = torch.linspace(0, rows.shape[0] - 1, steps=max_rows, device=rows.device).long()
            rows = rows.index_select(0, idx)
        self.add(rows)

    def nbytes(self) -> int:
        return sum(c.numel() * 2 for c in self.chunks)

    @torch.no_grad()
    def hessian(self, device, chunk_rows: int = 65536, tiles: tuple[int, int] | None = None) -> torch.Tensor:
        """H = X^T X in float32 on `device` (a CUDA device). With tiles=(begin, end)
        only those output tiles are formed and the rest of H is zero."""
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("mlx_gptq_b200 forms Hessians on CUDA devices only")
        H = torch.empty(self.in_features, self.in_features, dtype=torch.float32, device=device)
        if tiles is not None:
            H.zero_()
        beta = 0.0
        for c in self.chunks:
            for i in range(0, c.shape[0], chunk_rows):
                x = c[i:i + chunk_rows]
                if x.shape[0] == 0:
                    continue
                xd = x.to(device, torch.bfloat16, non_blocking=True)
                hessian_accumulate(xd, H, 1.0, beta, tiles=tiles)
                beta = 1.0
        if beta == 0.0 and tiles is None:
            H.zero_()
        L.raise_on_device_timeout(device)
        return H

    def clear(self):
        self.chunks.clear()


@dataclass
class LinearTask:
    """A plain nn.Linear to quantize; `name` is layer-relative (capture.py:82-87)."""
    name: str
    module: torch.nn.Module
    stash_key: str  # owner stash (may belong to a sibling with the same input)


@dataclass
class FusedExpertTask:
    """One fused 3D expert parameter [E, out, in] to quantize per expert (capture.py:90-97)."""
    module_name: str
    param_name: str
    param: torch.nn.Parameter
    num_experts: int
    stash_keys: list = field(default_factory=list)  # one per expert


class SegmentStore:
    """Rows captured from one sort-based expert module (experts.py), kept where the
    layer runs: the module inputs [tokens, in], the activations that feed
    down_proj [slots, inter] in expert order per batch, and each slot's global
    token id. Buffers are sized once from `reserve_tokens` (tokens per layer) and
    grow by doubling otherwise; the forward writes its activations straight into
    them."""

    def __init__(self, num_experts: int, reserve_tokens: int | None = None, device=None):
        self.E = num_experts
        self.reserve = reserve_tokens
        self.device = None if device is None else torch.device(device)  # None: where the rows are produced
        self.inputs = self.acts = self.tok = None
        self.n_tok = self.n_slot = 0
        self.batch_counts: list[list[int]] = []
        self.counts = [0] * num_experts
        self._pending = None  # activation slice handed to the running forward

    @staticmethod
    def _grow(buf, used: int, need: int, row_shape, dtype, device, hint):
        if buf is not None and buf.shape[0] >= need:
            return buf
        cap = max(need, hint or 0, 2 * (buf.shape[0] if buf is not None else 0))
        new = torch.empty((cap,) + tuple(row_shape), dtype=dtype, device=device)
        if buf is not None and used:
            new[:used].copy_(buf[:used])
        return new

    def _slot_hint(self, slots: int, tokens: int):
        """Slots per layer expected from the reservation (tokens x slots per token)."""
        return None if self.reserve is None else self.reserve * max(1, -(-slots // max(1, tokens)))

    def acts_out(self, slots: int, tokens: int, inter: int, dtype, device) -> torch.Tensor | None:
        """Where the forward should write this batch's activation rows (None when the
        store keeps its rows on another device: add() copies them there)."""
        if self.device is not None and torch.device(device) != self.device:
            return None
        self.acts = self._grow(self.acts, self.n_slot, self.n_slot + slots, (inter,), dtype, device,
                               self._slot_hint(slots, tokens))
        self._pending = self.acts[self.n_slot:self.n_slot + slots]
        return self._pending

    def add(self, hidden: torch.Tensor, tok: torch.Tensor, counts, acts: torch.Tensor):
        T, S = hidden.shape[0], tok.shape[0]
        dev = hidden.device if self.device is None else self.device
        self.inputs = self._grow(self.inputs, self.n_tok, self.n_tok + T, hidden.shape[1:], hidden.dtype, dev,
                                 self.reserve)
        self.inputs[self.n_tok:self.n_tok + T].copy_(hidden)
        self.tok = self._grow(self.tok, self.n_slot, self.n_slot + S, (), torch.int32, dev, self._slot_hint(S, T))
        self.tok[self.n_slot:self.n_slot + S].copy_(tok + self.n_tok)
        if acts is not None and (self._pending is None or acts.data_ptr() != self._pending.data_ptr()):
            self.acts = self._grow(self.acts, self.n_slot, self.n_slot + S, acts.shape[1:], acts.dtype, dev, None)
            self.acts[self.n_slot:self.n_slot + S].copy_(acts)
        self._pending = None
        self.batch_counts.append(list(counts))
        for e, n in enumerate(counts):
            self.counts[e] += n
        self.n_tok += T
        self.n_slot += S

    def slot_experts(self, device) -> torch.Tensor:
        E = self.E
        return torch.cat([torch.repeat_interleave(torch.arange(E, device=device), torch.tensor(c, device=device),
                                                  output_size=sum(c)) for c in self.batch_counts])

    def nbytes(self) -> int:
        return sum(x.numel() * x.element_size() for x in (self.inputs, self.acts, self.tok) if x is not None)


class _BatchInputs:
    """Tensors stashed during the current forward batch, by identity: a module that
    reads a tensor a sibling already stashed shares the sibling's stash. The tensors
    are held until the batch ends, so an id() cannot be reused meanwhile."""

    def __init__(self):
        self._owner: dict[int, tuple[torch.Tensor, str]] = {}

    def claim(self, x: torch.Tensor, key: str) -> str | None:
        """None if x is new in this batch (it is now `key`'s); otherwise the key of
        the stash that already holds x."""
        hit = self._owner.get(id(x))
        if hit is not None and hit[0] is x:
            return hit[1]
        self._owner[id(x)] = (x, key)
        return None

    def clear(self) -> None:
        self._owner.clear()


class _ExpertRouter(TorchFunctionMode):
    """Active during capture: every F.linear whose weight is one registered expert
    slice (matched by data pointer, capture.py:192-207) adds its input rows to that
    expert's stash before the call runs."""

    def __init__(self, table: dict[int, "Stash"]):
        super().__init__()
        self.table = table

    def _stash_for(self, w):
        if not isinstance(w, torch.Tensor) or w.dim() != 2:
            return None
        st = self.table.get(w.data_ptr())
        return st if st is not None and w.shape[-1] == st.in_features else None

    def __torch_function__(self, func, types, args=(), kwargs=None):
        if func is F.linear and len(args) >= 2:
            st = self._stash_for(args[1])
            if st is not None:
                st.add(args[0])
        return func(*args, **(kwargs or {}))


def _expert_activation(tasks: dict, e: int, rows: torch.Tensor) -> torch.Tensor | None:
    """silu(x W_gate^T) * (x W_up^T) for expert e, from a fused gate_up parameter or
    separate gate / up parameters; None if the module has neither."""
    if "gate_up_proj" in tasks:
        w = tasks["gate_up_proj"].param[e]
        gate, up = F.linear(rows.to(w.device, w.dtype), w).chunk(2, dim=-1)
    elif "gate_proj" in tasks and "up_proj" in tasks:
        wg, wu = tasks["gate_proj"].param[e], tasks["up_proj"].param[e]
        x = rows.to(wg.device, wg.dtype)
        gate, up = F.linear(x, wg), F.linear(x, wu)
    else:
        return None
    return F.silu(gate) * up


class CaptureManager:
    """Owns all stashes and hooks for one decoder layer (capture.py:100-343).

    Same discovery, routing and dedup rules as the reference: nn.Linear modules
    not matching `exclude_regex` with in_features % group_size == 0 become
    LinearTasks; 3D parameters named in FUSED_EXPERT_PARAMS become
    FusedExpertTasks with one stash per expert; q/k/v (gate/up) fed the same
    tensor in one batch share one stash; fused experts are captured from the
    ``F.linear`` calls whose weight is one expert's slice."""

    def __init__(self, layer: torch.nn.Module, exclude_regex, group_size: int, stash_device=None,
                 reserve_tokens: int | None = None):
        self.layer = layer
        self.stash_device = stash_device
        self.stashes: dict[str, Stash] = {}
        self.linear_tasks: list[LinearTask] = []
        self.fused_tasks: list[FusedExpertTask] = []
        self._hooks = []
        self._ptr_registry: dict[int, str] = {}
        self._batch = _BatchInputs()
        self._fused_modules: dict[str, torch.nn.Module] = {}
        self._fused_input_stashes: dict[str, Stash] = {}
        self.fallback_experts: dict[str, str] = {}
        self._segments: dict[str, SegmentStore] = {}  # sort-based expert modules
        self.reserve_tokens = reserve_tokens
        self._segment_modules: set[str] = set()
        self._slot_experts: dict[tuple[str, str], torch.Tensor] = {}
        self._slot_lock = threading.Lock()
        self.global_tokens: dict[str, int] | None = None  # summed over data-parallel ranks
        self._exit_stack: contextlib.ExitStack | None = None
        excl = re.compile(exclude_regex) if exclude_regex else None
        seen = set()
        for name, mod in layer.named_modules():
            if isinstance(mod, torch.nn.Linear):
                if excl and excl.search(name):
                    continue
                if mod.in_features % group_size:
                    log.warning("skipping %s: in_features %d not divisible by group %d (stays unquantized)",
                                name, mod.in_features, group_size)
                    continue
                self.linear_tasks.append(LinearTask(name, mod, stash_key=name))
                continue
            for pname, p in mod.named_parameters(recurse=False):
                if p.dim() != 3 or pname not in FUSED_EXPERT_PARAMS or (name, pname) in seen:
                    continue
                seen.add((name, pname))
                if p.shape[-1] % group_size:
                    log.warning("skipping fused %s.%s: in dim %d not divisible by group %d",
                                name, pname, p.shape[-1], group_size)
                    continue
                task = FusedExpertTask(name, pname, p, p.shape[0])
                for e in range(p.shape[0]):
                    key = f"{name}.{pname}::e{e}"
                    task.stash_keys.append(key)
                    self.stashes[key] = Stash(key, p.shape[-1], stash_device)
                    self._ptr_registry[p.data_ptr() + e * p.stride(0) * p.element_size()] = key
                self.fused_tasks.append(task)
                self._fused_modules[name] = mod
                if pname in ("gate_up_proj", "gate_proj", "up_proj"):
                    self._fused_input_stashes.setdefault(name, Stash(f"{name}::all_inputs", p.shape[-1],
                                                                     stash_device))
        for t in self.linear_tasks:
            self.stashes.setdefault(t.name, Stash(t.name, t.module.in_features, stash_device))

    # ---- capture taps (the reference's hooks: capture.py:167-207) ----
    def _linear_tap(self, task: LinearTask):
        """Forward pre-hook of one nn.Linear: stash its input, unless a sibling read the
        very same tensor earlier in this batch (q/k/v, gate/up), in which case the task
        adopts the sibling's stash and nothing is copied."""
        def tap(mod, args, kwargs):
            x = args[0] if args else kwargs["input"]
            owner = self._batch.claim(x, task.stash_key)
            if owner is None:
                self.stashes[task.stash_key].add(x)
            else:
                task.stash_key = owner
        return tap

    def _fused_sample_tap(self, module_name: str):
        """Forward pre-hook of a fused-expert module: keep 64 evenly spaced rows of its
        input per batch, the activation-aware fallback for experts no token reaches."""
        sample = self._fused_input_stashes[module_name]

        def tap(mod, args, kwargs):
            sample.add_sampled(args[0] if args else kwargs["hidden_states"], 64)
        return tap

    def _make_segment_sink(self, module_name: str):
        tasks = [t for t in self.fused_tasks if t.module_name == module_name]
        E = tasks[0].num_experts
        store = self._segments.setdefault(module_name, SegmentStore(E, self.reserve_tokens, self.stash_device))

        def sink(hidden, tok, counts, acts):
            store.add(hidden.detach(), tok, counts, acts)
            for t in tasks:
                for e, n in enumerate(counts):
                    self.stashes[t.stash_keys[e]].tokens += n
        sink.acts_out = store.acts_out
        return sink

    def __enter__(self):
        from .experts import uses_grouped

        stack = contextlib.ExitStack()
        for t in self.linear_tasks:
            stack.callback(t.module.register_forward_pre_hook(self._linear_tap(t), with_kwargs=True).remove)
        routed = set()  # experts whose rows arrive through a sort-based forward, not F.linear
        for name, module in self._fused_modules.items():
            if name in self._fused_input_stashes:
                stack.callback(module.register_forward_pre_hook(self._fused_sample_tap(name),
                                                                with_kwargs=True).remove)
            if uses_grouped(module):
                module._gq_sink = self._make_segment_sink(name)
                self._segment_modules.add(name)
                stack.callback(module.__dict__.pop, "_gq_sink", None)
                routed.update(k for t in self.fused_tasks if t.module_name == name for k in t.stash_keys)
        table = {ptr: self.stashes[k] for ptr, k in self._ptr_registry.items() if k not in routed}
        if table:
            stack.enter_context(_ExpertRouter(table))
        stack.callback(self._batch.clear)
        self._exit_stack = stack
        return self

    def __exit__(self, *exc):
        stack, self._exit_stack = self._exit_stack, None
        if stack is not None:
            stack.close()
        return False

    def begin_batch(self):
        """A new forward batch: input identities from the previous one no longer dedup."""
        self._batch.clear()

    def tokens(self, key: str) -> int:
        """Rows captured for a stash: this process's, or the sum over data-parallel
        ranks after sync_token_counts."""
        if self.global_tokens is not None:
            return self.global_tokens[key]
        return self.stashes[key].tokens

    def sync_token_counts(self, group, device):
        """Sum every stash's row count over the ranks of `group` (each rank captured its
        own calibration windows); the local counts stay in Stash.tokens."""
        import torch.distributed as dist

        keys = sorted(self.stashes)
        t = torch.tensor([self.stashes[k].tokens for k in keys], dtype=torch.int64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        self.global_tokens = dict(zip(keys, t.tolist()))

    # ---- diagnostics ----
    def total_stash_bytes(self) -> int:
        seg = sum(st.nbytes() for st in self._segments.values())
        return sum(s.nbytes() for s in self.stashes.values()) + seg

    def expert_token_stats(self):
        """param -> (min, median, max, zero_count) of tokens per expert (capture.py:242-251)."""
        out = {}
        for t in self.fused_tasks:
            counts = sorted(self.tokens(k) for k in t.stash_keys)
            out[f"{t.module_name}.{t.param_name}"] = (counts[0], counts[len(counts) // 2], counts[-1],
                                                      sum(1 for c in counts if c == 0))
        return out

    @torch.no_grad()
    def backfill_unrouted_experts(self):
        """Experts that no calibration token reached get real inputs instead of a zero
        Hessian (capture.py:253-326): their input-side stashes receive the module's
        sampled input rows, and their down_proj stash the activations those rows
        produce through the expert's own gate/up weights. Returns module -> experts."""
        done = {}
        for module_name, tasks in self._fused_tasks_by_module().items():
            sample = self._fused_input_stashes.get(module_name)
            feeder = next((tasks[n] for n in ("gate_up_proj", "gate_proj", "up_proj") if n in tasks), None)
            if sample is None or sample.tokens == 0 or feeder is None:
                continue
            missing = [e for e, key in enumerate(feeder.stash_keys) if self.tokens(key) == 0]
            for e in missing:
                self._backfill_expert(tasks, e, sample)
            if missing:
                done[module_name] = missing
        return done

    def _fused_tasks_by_module(self) -> dict[str, dict[str, FusedExpertTask]]:
        out: dict[str, dict[str, FusedExpertTask]] = {}
        for t in self.fused_tasks:
            out.setdefault(t.module_name, {})[t.param_name] = t
        return out

    def _backfill_expert(self, tasks: dict[str, FusedExpertTask], e: int, sample: Stash) -> None:
        for pname, task in tasks.items():
            if pname == "down_proj":
                continue
            key = task.stash_keys[e]
            for rows in sample.chunks:
                self.stashes[key].add(rows)
            self.fallback_experts[key] = "all_expert_inputs"
        down = tasks.get("down_proj")
        if down is None:
            return
        key = down.stash_keys[e]
        for rows in sample.chunks:
            act = _expert_activation(tasks, e, rows)
            if act is None:
                break
            self.stashes[key].add(act)
        if self.stashes[key].tokens:
            self.fallback_experts[key] = "all_expert_inputs"

    def check_capture_happened(self):
        """capture.py:328-337: fused experts must have gone through F.linear."""
        for t in self.fused_tasks:
            if all(self.tokens(k) == 0 for k in t.stash_keys):
                raise RuntimeError(
                    f"No tokens captured for fused experts {t.module_name}.{t.param_name}. "
                    "The model is probably not using the eager experts implementation; "
                    "load it with experts_implementation='eager'.")

    def drop_all(self):
        for s in self.stashes.values():
            s.clear()
        for s in self._fused_input_stashes.values():
            s.clear()
        self._segments.clear()
        self._slot_experts.clear()

    # ---- rows of one expert, wherever they were captured ----
    def _segment_rows(self, task: FusedExpertTask, experts, device):
        """(X, idx, counts) covering the segment-captured rows of `experts`, expert
        by expert in capture order (batch, then slot): idx int32 rows of X, counts
        per expert. None if the task was captured through F.linear."""
        st = self._segments.get(task.module_name)
        if st is None or st.n_slot == 0:
            return None
        key = (task.module_name, str(torch.device(device)))  # one copy per device (threads per device)
        with self._slot_lock:
            se = self._slot_experts.get(key)
            if se is None:
                se = self._slot_experts[key] = st.slot_experts(device)
        counts = [st.counts[e] for e in experts]
        S = st.n_slot
        pos = torch.full((st.E,), len(experts), dtype=torch.int64, device=device)
        pos[torch.tensor(experts, dtype=torch.int64, device=device)] = torch.arange(len(experts), device=device)
        order = torch.argsort(pos[se] * S + torch.arange(S, device=device))[:sum(counts)]
        if task.param_name == "down_proj":  # rows kept on another device move once, here
            return st.acts[:S].to(device), order.to(torch.int32), counts
        return st.inputs[:st.n_tok].to(device), st.tok[:S].to(device)[order], counts

    @torch.no_grad()
    def expert_rows(self, task: FusedExpertTask, expert: int, device) -> torch.Tensor:
        """All captured input rows of one expert (bf16 [n, in]) on `device`."""
        st = self.stashes[task.stash_keys[expert]]
        chunks = [c.to(device) for c in st.chunks]
        seg = self._segment_rows(task, [expert], device)
        if seg is not None:
            X, idx, _ = seg
            chunks.insert(0, X.index_select(0, idx.long()))
        if not chunks:
            return torch.empty(0, task.param.shape[-1], dtype=torch.bfloat16, device=device)
        return torch.cat(chunks, 0)

    # ---- Hessians on the tensor cores ----
    @torch.no_grad()
    def expert_hessians(self, task: FusedExpertTask, device, experts=None, timer=None) -> torch.Tensor:
        """H [len(experts), C, C] float32 for the given experts of a fused task, one
        grouped launch over their rows (token indices into the captured module
        inputs, or this share's activation blocks, plus any stashed rows)."""
        experts = list(range(task.num_experts)) if experts is None else list(experts)
        C = task.param.shape[-1]
        real = [e for e in experts if e is not None]  # None: a padding slot (H = 0)
        seg = self._segment_rows(task, real, device)
        parts, idx_parts, counts, base = [], [], [], 0
        seg_off, j = 0, 0
        if seg is not None:
            X0, idx0, seg_counts = seg
            parts.append(X0)
            base = X0.shape[0]
        for e in experts:
            n = 0
            if e is None:
                counts.append(0)
                continue
            if seg is not None and seg_counts[j]:
                idx_parts.append(idx0[seg_off:seg_off + seg_counts[j]])
                seg_off += seg_counts[j]
                n += seg_counts[j]
            j += 1
            for c in self.stashes[task.stash_keys[e]].chunks:
                parts.append(c.to(device))
                idx_parts.append(torch.arange(base, base + c.shape[0], dtype=torch.int32, device=device))
                base += c.shape[0]
                n += c.shape[0]
            counts.append(n)
        X = (parts[0] if len(parts) == 1 else torch.cat(parts, 0)) if parts else \
            torch.zeros(1, C, dtype=torch.bfloat16, device=device)
        offsets = torch.zeros(len(experts) + 1, dtype=torch.int64)
        offsets[1:] = torch.cumsum(torch.tensor(counts, dtype=torch.int64), 0)
        idx = torch.cat(idx_parts) if idx_parts else torch.zeros(1, dtype=torch.int32, device=device)
        if timer is not None:
            timer("expert_rows")
        return hessian_grouped(X, idx, offsets, len(experts))
