"""Calibration input stashes and the Hessian accumulation (tensor cores).

Mirrors ``Stash`` of mlx_gptq/capture.py (add / add_sampled / nbytes / hessian
/ clear). ``Stash.hessian`` forms H = X^T X in float32 with the tcgen05 kernel
of libgptq_b200.so instead of float32 ``addmm`` per 65,536-row chunk
(capture.py:68-76); ``hessian_from_rows`` is the same kernel on rows that are
already in device memory.
"""

from __future__ import annotations

import torch

from . import _lib as L


@torch.no_grad()
def hessian_accumulate(X: torch.Tensor, H: torch.Tensor, alpha: float = 1.0, beta: float = 1.0,
                       status: torch.Tensor | None = None) -> torch.Tensor:
    """H = beta * H + alpha * X^T X for bf16 rows X [n, c] and float32 H [c, c], both on
    the same CUDA device. Returns H."""
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
    L.check(L.lib().gq_hessian_bf16(L.ptr(X), n, c, X.stride(0), L.ptr(H), H.stride(0), float(alpha),
                                    float(beta), L.ptr(status), L.stream_ptr(X.device)), "hessian")
    return H


@torch.no_grad()
def hessian_from_rows(X: torch.Tensor) -> torch.Tensor:
    """H = X^T X (float32) for device-resident bf16 rows X [n, c]."""
    c = X.shape[1]
    H = torch.empty(c, c, dtype=torch.float32, device=X.device)
    return hessian_accumulate(X, H, 1.0, 0.0)


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
                                        L.ptr(ws), ws.numel(), None, L.stream_ptr(X.device)), "hessian_grouped")
    return H


class Stash:
    """Captured input rows for one logical weight matrix (capture.py:33-79)."""

    def __init__(self, name: str, in_features: int):
        self.name = name
        self.in_features = in_features
        self.chunks: list[torch.Tensor] = []
        self.tokens = 0

    def add(self, x: torch.Tensor):
        rows = x.detach().reshape(-1, x.shape[-1])
        if rows.shape[-1] != self.in_features:
            raise RuntimeError(
                f"stash {self.name}: got rows of dim {rows.shape[-1]}, expected {self.in_features}")
        self.chunks.append(rows.to("cpu", torch.bfloat16))
        self.tokens += rows.shape[0]

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
    def hessian(self, device, chunk_rows: int = 65536) -> torch.Tensor:
        """H = X^T X in float32 on `device` (a CUDA device)."""
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("mlx_gptq_b200 forms Hessians on CUDA devices only")
        H = torch.empty(self.in_features, self.in_features, dtype=torch.float32, device=device)
        beta = 0.0
        for c in self.chunks:
            for i in range(0, c.shape[0], chunk_rows):
                x = c[i:i + chunk_rows]
                if x.shape[0] == 0:
                    continue
                xd = x.to(device, torch.bfloat16, non_blocking=True)
                hessian_accumulate(xd, H, 1.0, beta)
                beta = 1.0
        if beta == 0.0:
            H.zero_()
        return H

    def clear(self):
        self.chunks.clear()
