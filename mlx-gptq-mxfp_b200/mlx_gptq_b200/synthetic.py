"""Seeded synthetic inputs for the benchmark configurations.

There is no public dataset for this path: the configurations are defined by shapes and
value distributions, and every tensor here is drawn from its own seeded generator on the
device (float32, rounded once to bf16, round-to-nearest-even), so every process, rank and
run sees the same inputs.

  C1  dense linear, affine 4-bit g64: W [4096, 4096] ~ N(0, 0.02) (seed 0);
      X [524288, 4096] ~ N(0, 1) with 16 outlier channels x20 (seed 1)
  C2  dense MLP sweep, MXFP4 safe-scale-search: gate/up [11008, 4096], down [4096, 11008]
      ~ N(0, 0.02); X [131072, K] Student-t(4) with 1% of channels x30
  C3  MoE expert batch, MXFP4 groupwise: 128 experts, gate_up [1536, 2048] (= [gate; up])
      and down [2048, 768] ~ N(0, 0.02) (seed 0); X [524288, 2048] ~ N(0, 1) (seed 1);
      router logits N(0, 1) (seed 2) plus a Zipf(1.1) bias -1.1 * ln(rank_e), rank a
      seed-3 permutation of 1..128, top-8; down inputs silu(x Wg^T) * (x Wu^T) per slot
  C4  attention projections, MXFP8 groupwise: q [4096, 2048], k / v [512, 2048],
      o [2048, 4096] ~ N(0, 0.02); X [262144, K] ~ N(0, 1) x LogNormal(0, 0.5) per channel
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

_CHUNK = 16384  # rows generated per call (bounds the float32 staging buffer)


def _gen(seed: int, device) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(int(seed))


def weights_bf16(shape, seed: int, device, std: float = 0.02) -> torch.Tensor:
    """N(0, std) weights, bf16."""
    return (torch.randn(*shape, generator=_gen(seed, device), device=device) * std).to(torch.bfloat16)


def _rows(n: int, k: int, seed: int, device, draw) -> tuple[torch.Tensor, torch.Generator]:
    g = _gen(seed, device)
    out = torch.empty(n, k, dtype=torch.bfloat16, device=device)
    for i in range(0, n, _CHUNK):
        m = min(_CHUNK, n - i)
        out[i:i + m] = draw(g, m).to(torch.bfloat16)
    return out, g


def _scale_channels(X: torch.Tensor, idx: torch.Tensor, factor: float) -> None:
    X[:, idx] = (X[:, idx].float() * factor).to(torch.bfloat16)


def outlier_normal_bf16(n: int, k: int, seed: int, device, n_outliers: int = 16,
                        factor: float = 20.0) -> torch.Tensor:
    """C1 activations: N(0, 1) with `n_outliers` random channels scaled by `factor`."""
    X, g = _rows(n, k, seed, device, lambda g, m: torch.randn(m, k, generator=g, device=device))
    _scale_channels(X, torch.randperm(k, generator=g, device=device)[:n_outliers], factor)
    return X


def student_t_bf16(n: int, k: int, seed: int, device, outlier_frac: float = 0.01,
                   factor: float = 30.0) -> torch.Tensor:
    """C2 activations: i.i.d. Student-t with 4 degrees of freedom (z / sqrt(chi2_4 / 4),
    chi2_4 = -2 ln(u1 u2)), with round(outlier_frac * k) channels scaled by `factor`."""
    def draw(g, m):
        z = torch.randn(m, k, generator=g, device=device)
        u = torch.rand(2, m, k, generator=g, device=device).clamp_(min=1e-12)
        return z / torch.sqrt(-2.0 * torch.log(u[0] * u[1]) / 4.0)

    X, g = _rows(n, k, seed, device, draw)
    _scale_channels(X, torch.randperm(k, generator=g, device=device)[:max(1, round(outlier_frac * k))], factor)
    return X


def lognormal_channels_bf16(n: int, k: int, seed: int, device, sigma: float = 0.5) -> torch.Tensor:
    """C4 activations: N(0, 1) times a per-channel LogNormal(0, sigma) scale."""
    g = _gen(seed, device)
    scale = torch.exp(sigma * torch.randn(k, generator=g, device=device))
    out = torch.empty(n, k, dtype=torch.bfloat16, device=device)
    for i in range(0, n, _CHUNK):
        m = min(_CHUNK, n - i)
        out[i:i + m] = (torch.randn(m, k, generator=g, device=device) * scale).to(torch.bfloat16)
    return out


@dataclass
class Routing:
    """Top-k routing of `tokens` tokens over E experts, grouped by expert.

    token_idx: int32 [slots] on the device, token of every routed slot, expert by expert
    (tokens ascending inside an expert); slot_expert: int64 [slots] on the device;
    counts: int64 [E] on the host; offsets: int64 [E + 1] on the host; bias_scale: the
    factor the Zipf bias was scaled by so that at least one expert gets no token."""
    token_idx: torch.Tensor
    slot_expert: torch.Tensor
    counts: torch.Tensor
    offsets: torch.Tensor
    bias_scale: float

    @property
    def zero_experts(self) -> list[int]:
        return [e for e, c in enumerate(self.counts.tolist()) if c == 0]


def zipf_routing(tokens: int, experts: int, topk: int, device, logit_seed: int = 2, rank_seed: int = 3,
                 zipf: float = 1.1, require_zero: bool = True) -> Routing:
    """C3 router: logits N(0, 1) plus the bias -zipf * ln(rank_e) (rank_e a permutation of
    1..E), top-k (the softmax is monotone, so top-k of the logits). If no expert gets zero
    tokens and require_zero, the bias is scaled by 1.1, 1.2, 1.3, ... until one does."""
    rank = torch.randperm(experts, generator=_gen(rank_seed, device), device=device).double() + 1.0
    bias = -zipf * torch.log(rank)
    for scale in [1.0 + 0.1 * i for i in range(31)]:
        g = _gen(logit_seed, device)
        top = torch.empty(tokens, topk, dtype=torch.int64, device=device)
        for i in range(0, tokens, _CHUNK * 4):
            m = min(_CHUNK * 4, tokens - i)
            logits = torch.randn(m, experts, generator=g, device=device) + (scale * bias).float()
            top[i:i + m] = logits.topk(topk, dim=1).indices
        counts = torch.bincount(top.reshape(-1), minlength=experts)
        if not require_zero or int((counts == 0).sum()) > 0:
            break
    flat = top.reshape(-1)
    order = torch.argsort(flat * tokens + torch.arange(flat.numel(), device=device) // topk)
    token_idx = (order // topk).to(torch.int32)
    counts_h = counts.cpu()
    offsets = torch.zeros(experts + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts_h, 0)
    return Routing(token_idx, flat[order], counts_h, offsets, scale)


@torch.no_grad()
def expert_down_inputs(X: torch.Tensor, gate_up: torch.Tensor, routing: Routing) -> torch.Tensor:
    """bf16 [slots, I]: silu(x W_gate^T) * (x W_up^T) for every routed slot, expert by
    expert in routing order (gate_up [E, 2I, H] bf16, gate rows first)."""
    E, two_i, _ = gate_up.shape
    inter = two_i // 2
    out = torch.empty(routing.token_idx.numel(), inter, dtype=torch.bfloat16, device=X.device)
    off = routing.offsets.tolist()
    for e in range(E):
        a, b = off[e], off[e + 1]
        if a == b:
            continue
        h = F.linear(X.index_select(0, routing.token_idx[a:b].long()), gate_up[e])
        out[a:b] = F.silu(h[:, :inter]) * h[:, inter:]
    return out


# ---------------------------------------------------------------------------
# configuration records
# ---------------------------------------------------------------------------
C1 = dict(rows=4096, cols=4096, tokens=524288, outliers=16, factor=20.0, bits=4, group=64)
C2 = dict(hidden=4096, inter=11008, tokens=131072)
C3 = dict(experts=128, hidden=2048, inter=768, tokens=524288, topk=8)
C4 = dict(hidden=2048, q=4096, kv=512, o_in=4096, tokens=262144)


def c1_inputs(device, tokens: int = C1["tokens"]):
    W = weights_bf16((C1["rows"], C1["cols"]), 0, device)
    X = outlier_normal_bf16(tokens, C1["cols"], 1, device, C1["outliers"], C1["factor"])
    return W, X


def c2_inputs(seed: int, device, tokens: int = C2["tokens"]):
    h, i = C2["hidden"], C2["inter"]
    return {"X_gu": student_t_bf16(tokens, h, seed + 1000, device),
            "X_down": student_t_bf16(tokens, i, seed + 2000, device),
            "gate": weights_bf16((i, h), seed, device), "up": weights_bf16((i, h), seed + 1, device),
            "down": weights_bf16((h, i), seed + 2, device)}


def c3_inputs(device, tokens: int = C3["tokens"], experts: int = C3["experts"]):
    """(X, gate_up [E, 2I, H], down [E, H, I], routing, down inputs [slots, I])."""
    h, i = C3["hidden"], C3["inter"]
    X = _rows(tokens, h, 1, device, lambda g, m: torch.randn(m, h, generator=g, device=device))[0]
    gate_up = weights_bf16((experts, 2 * i, h), 0, device)
    down = weights_bf16((experts, h, i), 10, device)
    routing = zipf_routing(tokens, experts, C3["topk"], device)
    return X, gate_up, down, routing, expert_down_inputs(X, gate_up, routing)


def c4_inputs(device, tokens: int = C4["tokens"]):
    h = C4["hidden"]
    return {"X_qkv": lognormal_channels_bf16(tokens, h, 1, device),
            "X_o": lognormal_channels_bf16(tokens, C4["o_in"], 2, device),
            "q_proj": weights_bf16((C4["q"], h), 0, device), "k_proj": weights_bf16((C4["kv"], h), 1, device),
            "v_proj": weights_bf16((C4["kv"], h), 2, device), "o_proj": weights_bf16((h, C4["o_in"]), 3, device)}


def hessian_flop(n: int, c: int) -> float:
    """Algorithmic FLOP of one H = X^T X (the reference's full product)."""
    return 2.0 * n * c * c


__all__ = ["weights_bf16", "outlier_normal_bf16", "student_t_bf16", "lognormal_channels_bf16", "zipf_routing",
           "Routing", "expert_down_inputs", "c1_inputs", "c2_inputs", "c3_inputs", "c4_inputs", "hessian_flop",
           "C1", "C2", "C3", "C4"]
