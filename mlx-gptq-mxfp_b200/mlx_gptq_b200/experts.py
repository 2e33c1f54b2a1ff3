"""Sort-based forward of the transformers fused-expert MLP, with device-side capture.

The eager expert loop of transformers >= 5 (e.g. Qwen3MoeExperts.forward) builds a
one-hot [tokens, top_k, E] mask and calls torch.where on one expert's slice per
iteration: one device->host synchronisation per expert per batch. This forward
computes the same thing with one sort of the routed slots:

* slots are ordered by (expert, top-k position, token), which is exactly the row
  order torch.where gives the eager loop, so every expert GEMM sees the same input
  rows and the results are bit-identical;
* the elementwise work runs once over all slots instead of once per expert, and
  the output is accumulated in k rounds that add each token's contributions in
  ascending expert order, the order of the eager loop's per-expert index_add_;
* the expert GEMMs are one grouped launch each (no per-shape cuBLAS heuristic
  query for every new token count), and two host reads of counts per batch
  replace one synchronisation per expert.

When a CaptureManager is active it receives, per batch, the module input (the
gate/up rows are `hidden_states[tok]`: stored as token indices, not copies), the
sorted token indices, the per-expert counts and the activation rows that feed
down_proj (one tensor in expert order), i.e. exactly the rows the reference's
F.linear interception stashes (capture.py:192-207), without per-expert copies.
"""

from __future__ import annotations

import types

import torch
import torch.nn.functional as F

# expert classes whose eager forward is: gate_up = F.linear(x[tok], gate_up_proj[e]);
# h = act_fn(gate) * up; y = F.linear(h, down_proj[e]) * w; out.index_add_(0, tok, y)
GROUPED_EXPERT_CLASSES = {"Qwen3MoeExperts", "Qwen2MoeExperts", "MixtralExperts", "OlmoeExperts",
                          "Qwen3VLMoeTextExperts", "Qwen3OmniMoeThinkerTextExperts"}


def supports_grouped(module: torch.nn.Module) -> bool:
    return (type(module).__name__ in GROUPED_EXPERT_CLASSES
            and isinstance(getattr(module, "gate_up_proj", None), torch.Tensor)
            and isinstance(getattr(module, "down_proj", None), torch.Tensor)
            and module.gate_up_proj.dim() == 3
            and not getattr(module, "has_bias", False) and not getattr(module, "is_transposed", False))


def _count(idx: torch.Tensor, n: int) -> torch.Tensor:
    """Histogram of idx over [0, n) without a host synchronisation."""
    return torch.zeros(n, dtype=torch.int64, device=idx.device).index_add_(
        0, idx, torch.ones_like(idx, dtype=torch.int64))


@torch.no_grad()
def route(top_k_index: torch.Tensor, num_experts: int):
    """Slots of one batch ordered by (expert, top-k position, token).

    Returns (tok, pos, counts, counts_dev): token and top-k position of each
    ordered slot (int64, on the device), the per-expert slot counts as a host list
    and as a device tensor. Slots routed to index num_experts (dropped) are left out."""
    T, k = top_k_index.shape
    dev = top_k_index.device
    E = num_experts
    e = top_k_index.reshape(-1).long().clamp(0, E)
    j = torch.arange(k, device=dev).repeat(T)
    t = torch.arange(T, device=dev).repeat_interleave(k)
    order = torch.argsort(e * (k * T) + j * T + t)
    counts_dev = _count(e, E + 1)[:E]
    counts = counts_dev.tolist()
    order = order[:sum(counts)]
    return t[order], j[order], counts, counts_dev


def _token_ranks(tok: torch.Tensor, T: int) -> torch.Tensor:
    """For slots already ordered by (expert, ...): the rank of each slot among its
    token's slots in ascending expert order (0 for the lowest expert)."""
    S = tok.shape[0]
    ar = torch.arange(S, device=tok.device)
    order = torch.argsort(tok * S + ar)  # by token, then by expert
    counts = _count(tok, T)
    starts = torch.cumsum(counts, 0) - counts
    ranks = torch.empty_like(ar)
    ranks[order] = ar - starts[tok[order]]
    return ranks


def _expert_gemm(x: torch.Tensor, w: torch.Tensor, counts: list, offs: torch.Tensor) -> torch.Tensor:
    """y[rows of e] = x[rows of e] @ w[e]^T for row blocks in expert order.

    One grouped GEMM launch (torch._grouped_mm) on CUDA bf16; otherwise one mm per
    expert into a shared output. Both produce the F.linear result row for row
    (checked bit for bit against the eager loop by the tests)."""
    S = x.shape[0]
    if x.is_cuda and x.dtype == torch.bfloat16 and hasattr(torch, "_grouped_mm") and S > 0:
        return torch._grouped_mm(x, w.transpose(1, 2), offs=offs)
    y = torch.empty(S, w.shape[1], dtype=x.dtype, device=x.device)
    off = 0
    for e, n in enumerate(counts):
        if n:
            torch.mm(x[off:off + n], w[e].t(), out=y[off:off + n])
            off += n
    return y


def grouped_experts_forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                            top_k_weights: torch.Tensor) -> torch.Tensor:
    """Drop-in for the eager fused-expert forward (bound to the module as `forward`).

    Same arithmetic as the eager loop, batched across experts: each expert's two
    GEMMs cover contiguous row blocks of shared buffers (the same F.linear
    operands, row for row); SiLU(gate)·up and the routing-weight product run once
    over all slots (elementwise, so per element identical); the output is
    accumulated with k index_add_ rounds, round r adding every token's r-th
    lowest-expert contribution, which is the order in which the eager loop's
    per-expert index_add_ reaches each token."""
    E = self.num_experts
    T, k = top_k_index.shape
    tok, pos, counts, counts_dev = route(top_k_index, E)
    S = tok.shape[0]
    offs = torch.cumsum(counts_dev, 0).to(torch.int32)
    x = hidden_states.index_select(0, tok)
    gu = _expert_gemm(x, self.gate_up_proj, counts, offs)
    del x
    gate, up = gu.chunk(2, dim=-1)
    sink = getattr(self, "_gq_sink", None)
    h_out = sink.acts_out(S, T, self.down_proj.shape[-1], hidden_states.dtype, hidden_states.device) if sink is not None else None
    h = torch.mul(self.act_fn(gate), up, out=h_out) if h_out is not None else self.act_fn(gate) * up
    del gu, gate, up
    y = _expert_gemm(h, self.down_proj, counts, offs)
    y = y * top_k_weights[tok, pos, None]
    out = torch.zeros_like(hidden_states)
    y = y.to(out.dtype)
    ranks = _token_ranks(tok, T)
    by_rank = torch.argsort(ranks * S + torch.arange(S, device=tok.device))
    per_rank = _count(ranks, k).tolist()
    off = 0
    for n in per_rank:  # round r: every token's r-th lowest-expert contribution, one per token
        if n:
            sel = by_rank[off:off + n]
            out.index_add_(0, tok.index_select(0, sel), y.index_select(0, sel))
            off += n
    if sink is not None:
        sink(hidden_states, tok, counts, h)
    return out


def install_grouped_experts(model: torch.nn.Module) -> int:
    """Bind the sort-based forward to every supported expert module; returns how many."""
    n = 0
    for m in model.modules():
        if supports_grouped(m):
            m.forward = types.MethodType(grouped_experts_forward, m)
            n += 1
    return n


def uses_grouped(module: torch.nn.Module) -> bool:
    f = module.__dict__.get("forward")
    return getattr(f, "__func__", None) is grouped_experts_forward
