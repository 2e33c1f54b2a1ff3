"""Sort-based forward of the transformers fused-expert MLP, with device-side capture.

The eager expert loop of transformers >= 5 (e.g. Qwen3MoeExperts.forward) builds a
one-hot [tokens, top_k, E] mask and calls torch.where on one expert's slice per
iteration: one device->host synchronisation per expert per batch. This forward
computes the same thing with one sort of the routed slots:

* slots are ordered by (expert, top-k position, token), which is exactly the row
  order torch.where gives the eager loop, so every F.linear sees the same input
  matrix and the results are bit-identical;
* experts run in ascending order and add into the output with index_add_ like the
  eager loop, so each token's contributions are summed in the same order;
* one host read of the per-expert counts per batch instead of one per expert.

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


@torch.no_grad()
def route(top_k_index: torch.Tensor, num_experts: int):
    """Slots of one batch ordered by (expert, top-k position, token).

    Returns (tok, pos, counts): token and top-k position of each ordered slot
    (int64, on the device) and the per-expert slot counts (host list)."""
    T, k = top_k_index.shape
    dev = top_k_index.device
    e = top_k_index.reshape(-1).long()
    j = torch.arange(k, device=dev).repeat(T)
    t = torch.arange(T, device=dev).repeat_interleave(k)
    valid = e < num_experts  # an index equal to num_experts marks a dropped slot
    key = torch.where(valid, e * (k * T) + j * T + t, torch.full_like(e, num_experts * k * T))
    order = torch.argsort(key)
    counts = torch.bincount(e[valid], minlength=num_experts)[:num_experts]
    counts_h = counts.tolist()
    n = sum(counts_h)
    order = order[:n]
    return t[order], j[order], counts_h


def grouped_experts_forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                            top_k_weights: torch.Tensor) -> torch.Tensor:
    """Drop-in for the eager fused-expert forward (bound to the module as `forward`)."""
    E = self.num_experts
    tok, pos, counts = route(top_k_index, E)
    out = torch.zeros_like(hidden_states)
    sink = getattr(self, "_gq_sink", None)
    x = hidden_states.index_select(0, tok)
    acts = None
    if sink is not None:
        acts = torch.empty(tok.shape[0], self.down_proj.shape[-1], dtype=hidden_states.dtype,
                           device=hidden_states.device)
    off = 0
    for e in range(E):
        n = counts[e]
        if n == 0:
            continue
        sl = slice(off, off + n)
        gate, up = F.linear(x[sl], self.gate_up_proj[e]).chunk(2, dim=-1)
        h = self.act_fn(gate) * up
        if acts is not None:
            acts[sl] = h
        y = F.linear(h, self.down_proj[e])
        y = y * top_k_weights[tok[sl], pos[sl], None]
        out.index_add_(0, tok[sl], y.to(out.dtype))
        off += n
    if sink is not None:
        sink(hidden_states, tok, counts, acts)
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
