"""Solving several weight matrices that share one Hessian.

The reference caches one Hessian per stash and reuses it for every linear fed
by the same input (q/k/v, gate/up: mlx_gptq/capture.py:167-178 dedup and the
hess_cache of mlx_gptq/sequential.py:479-487). Here the shared work is done
once: dead-column handling and the damped 32x32 block factors for MXFP. Each
matrix then gets one column-loop launch that writes the artifact form directly:
nibble-packed E2M1 codes (MXFP4) or E4M3 bytes (MXFP8), E8M0 scales, and W_dq in
the model dtype for the re-forward.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib as L
from .gptq import _not_pd_error

MX_GROUP_SIZE = 32


@dataclass
class MxfpFactors:
    """Per-Hessian state shared by every matrix solved against it."""
    H: torch.Tensor      # [B, C, C] float32 (dead-column diagonals set to 1)
    dead: torch.Tensor   # [B, C] uint8
    U: torch.Tensor      # [B, C/32, 32, 32] float32
    info: torch.Tensor   # [B, C/32] int32


@dataclass
class MxfpSolution:
    codes: torch.Tensor   # mxfp4: [B, R, C/2] packed nibbles; mxfp8: [B, R, C] E4M3 bytes
    scales: torch.Tensor  # [B, R, C/32] uint8 E8M0
    w_dq: torch.Tensor    # [B, R, C] wdq_dtype
    rel_err: torch.Tensor | None


@torch.no_grad()
def mxfp_factors(H: torch.Tensor, damp: float = 0.01) -> MxfpFactors:
    """Dead columns (gptq.py:216-222, in place on H) + block factors (gptq.py:99-100)."""
    L.require_cuda(H)
    if H.dim() == 2:
        H = H.unsqueeze(0)
    B, C, _ = H.shape
    if C % MX_GROUP_SIZE:
        raise ValueError(f"in_features {C} not divisible by group {MX_GROUP_SIZE}")
    lib, stream = L.lib(), L.stream_ptr(H.device)
    dead = torch.empty(B, C, dtype=torch.uint8, device=H.device)
    L.check(lib.gq_dead_columns(L.ptr(H), B, C, L.ptr(dead), stream), "dead columns")
    U = torch.empty(B, C // 32, 32, 32, dtype=torch.float32, device=H.device)
    info = torch.empty(B, C // 32, dtype=torch.int32, device=H.device)
    L.check(lib.gq_mx_prepare_hinv(L.ptr(H), B, C, float(damp), L.ptr(U), L.ptr(info), None, stream),
            "mx prepare_hinv")
    return MxfpFactors(H, dead, U, info)


@torch.no_grad()
def solve_mxfp_packed(W: torch.Tensor, f: MxfpFactors, mode: str = "mxfp4", algorithm: str = "auto",
                      wdq_dtype: torch.dtype = torch.bfloat16, want_rel: bool = True,
                      check_info: bool = True) -> MxfpSolution:
    """MXFP GPTQ of W [B, R, C] (or [R, C]) against shared factors, artifact outputs."""
    if mode not in ("mxfp4", "mxfp8"):
        raise ValueError(f"not a microscaling mode: {mode}")
    if algorithm == "auto":
        algorithm = "safe-scale-search" if mode == "mxfp4" else "groupwise"
    if algorithm not in ("groupwise", "safe-scale-search"):
        raise ValueError(f"unsupported MXFP GPTQ algorithm: {algorithm}")
    L.require_cuda(W, f.H)
    if W.dim() == 2:
        W = W.unsqueeze(0)
    W = L.aligned(W)
    B, R, C = W.shape
    assert f.H.shape == (B, C, C)
    dev = W.device
    lib, stream = L.lib(), L.stream_ptr(dev)
    ncode = C // 2 if mode == "mxfp4" else C
    codes = torch.empty(B, R, ncode, dtype=torch.uint8, device=dev)
    scales = torch.empty(B, R, C // 32, dtype=torch.uint8, device=dev)
    w_dq = torch.empty(B, R, C, dtype=wdq_dtype, device=dev)
    rel = torch.empty(B, dtype=torch.float32, device=dev) if want_rel else None
    ws = torch.empty(lib.gq_gptq_mxfp_workspace_size(B, R, C) if want_rel else 0, dtype=torch.uint8, device=dev)
    q_ptr, qp_ptr = (None, L.ptr(codes)) if mode == "mxfp4" else (L.ptr(codes), None)
    L.check(lib.gq_gptq_mxfp(L.ptr(W), L.DTYPE_CODE[W.dtype], L.ptr(f.H), L.ptr(f.U), L.ptr(f.dead),
                             L.ptr(f.info), B, R, C, L.MODE_CODE[mode],
                             L.GQ_MX_SAFE_SCALE_SEARCH if algorithm == "safe-scale-search" else L.GQ_MX_GROUPWISE,
                             q_ptr, qp_ptr, L.ptr(scales), L.ptr(w_dq), L.DTYPE_CODE[wdq_dtype], L.ptr(rel),
                             L.ptr(ws), ws.numel(), stream), "gptq mxfp")
    if check_info:
        L.raise_on_device_timeout(dev)  # the Hessian behind f finished every wait
        failed = f.info != 0
        if bool(failed.any()):
            raise _not_pd_error(f.H, failed.any(dim=1), B)
    return MxfpSolution(codes, scales, w_dq, rel)


@torch.no_grad()
def solve_experts(W: torch.Tensor, H: torch.Tensor, counts, mode: str = "mxfp4", algorithm: str = "auto",
                  wdq_dtype: torch.dtype = torch.bfloat16, want_rel: bool = True, damp: float = 0.01,
                  check_info: bool = True) -> MxfpSolution:
    """A routed expert batch W [E, R, C] against its per-expert Hessians H [E, C, C]
    (mode mxfp4 / mxfp8): one factor launch and one column-loop launch for all experts;
    experts that received no token (counts[e] == 0) get data-free RTN instead
    (rtn_quantize_mxfp, grid.py:142-151), not GPTQ against an all-zero H, which would
    zero them (gptq.py:216-222)."""
    f = mxfp_factors(H, damp)
    sol = solve_mxfp_packed(W, f, mode, algorithm, wdq_dtype, want_rel, check_info=check_info)
    empty = [e for e, c in enumerate(list(counts)) if int(c) == 0]
    if empty:
        # pinned and non-blocking: the index upload does not make the host wait for the GPU
        idx = torch.tensor(empty, dtype=torch.long).pin_memory().to(W.device, non_blocking=True)
        We = L.aligned(W.index_select(0, idx))
        n, R, C = We.shape
        q = torch.empty(n, R, C, dtype=torch.uint8, device=W.device)
        codes = torch.empty((n,) + tuple(sol.codes.shape[1:]), dtype=torch.uint8, device=W.device) \
            if mode == "mxfp4" else q
        scales = torch.empty(n, R, C // MX_GROUP_SIZE, dtype=torch.uint8, device=W.device)
        dq = torch.empty(n, R, C, dtype=torch.float32, device=W.device)
        qp_ptr = L.ptr(codes) if mode == "mxfp4" else None
        L.check(L.lib().gq_rtn_mxfp(L.ptr(We), L.DTYPE_CODE[We.dtype], n * R, C, L.MODE_CODE[mode], L.ptr(q), qp_ptr,
                                    L.ptr(scales), L.ptr(dq), L.GQ_F32, L.stream_ptr(W.device)), "rtn fallback")
        sol.codes.index_copy_(0, idx, codes)
        sol.scales.index_copy_(0, idx, scales)
        sol.w_dq.index_copy_(0, idx, dq.to(sol.w_dq.dtype))
        if sol.rel_err is not None:
            Wf = We.float()
            rel = (dq - Wf).flatten(1).norm(dim=1) / Wf.flatten(1).norm(dim=1).clamp_min(1e-12)
            sol.rel_err.index_copy_(0, idx, rel)
    return sol
