"""Batched GPTQ solver on B200, with the reference's Python API.

Mirrors mlx_gptq/gptq.py of the reference: ``solve_gptq`` / ``gptq_quantize``
on W [B, out, in] and H [B, in, in] (any scale of X^T X), MLX affine grid or the
native MXFP4 / MXFP8 grids, same defaults, same ownership (``solve_gptq`` keeps
W intact and mutates the caller's H on dead columns; ``gptq_quantize``
overwrites W), same errors (AssertionError on shapes, ValueError on a bad
mode/algorithm/group, RuntimeError when H is not positive definite after the
damping escalation). All compute runs in libgptq_b200.so on the tensors' CUDA
device and stream.
"""

from __future__ import annotations

import logging

import torch

from . import _lib as L
from .grid import MX_GROUP_SIZE

log = logging.getLogger(__name__)


def _not_pd_error(H: torch.Tensor, failed: torch.Tensor, B: int) -> RuntimeError:
    """The diagnostics of gptq.py:53-63 for the failed batch items."""
    bad = H[failed]
    diag = bad.diagonal(dim1=-2, dim2=-1)
    return RuntimeError(
        "Hessian not positive definite after damping escalation; "
        f"batch={B} failed={int(failed.sum())} "
        f"nonfinite={int((~torch.isfinite(bad)).sum())} "
        f"diag_min={float(diag.min())} diag_max={float(diag.max())} "
        f"value_min={float(bad.min())} value_max={float(bad.max())}"
    )


_FACTOR_BLOCK = 64  # column block of gq_prepare_hinv


@torch.no_grad()
def _prepare_hinv(H: torch.Tensor, damp: float, max_attempts: int = 6) -> torch.Tensor:
    """gptq.py:27-66: upper Cholesky factor of (H + damp*mean(diag)*I)^-1, batched,
    damping escalated x10 for failing items (6 attempts)."""
    if max_attempts != 6:
        raise ValueError("the GPU factorization implements max_attempts=6")
    B, C, _ = H.shape
    dev = L.require_cuda(H)
    Hc = L.aligned(H.float())
    Hf = Hc
    if C % _FACTOR_BLOCK:
        # The factorization works on 64-column blocks: embed H in a block-diagonal matrix
        # whose extra diagonal is mean(diag H), so the damping mean (and lambda) is that
        # of H and the upper factor of the inverse is block-diagonal, U = U'[:C, :C].
        Cp = -(-C // _FACTOR_BLOCK) * _FACTOR_BLOCK
        Hf = torch.zeros(B, Cp, Cp, dtype=torch.float32, device=dev)
        Hf[:, :C, :C] = Hc
        m = Hc.diagonal(dim1=-2, dim2=-1).mean(-1)
        Hf[:, C:, C:].diagonal(dim1=-2, dim2=-1).copy_(m.unsqueeze(-1).expand(B, Cp - C))
    Cf = Hf.shape[-1]
    U = torch.empty(B, Cf, Cf, dtype=torch.float32, device=dev)
    info = torch.empty(B, dtype=torch.int32, device=dev)
    used = torch.empty(B, dtype=torch.float32, device=dev)
    ws = torch.empty(L.lib().gq_prepare_hinv_workspace_size(B, Cf), dtype=torch.uint8, device=dev)
    L.raise_on_device_timeout(dev)  # a Hessian formed on this device finished every wait
    st = L.lib().gq_prepare_hinv(L.ptr(Hf), B, Cf, float(damp), L.ptr(U), L.ptr(info), L.ptr(used),
                                 L.ptr(ws), ws.numel(), L.ptr(L.status_word(dev)), L.stream_ptr(dev))
    if st == L.GQ_ERR_NOT_PD:
        raise _not_pd_error(Hc, info != 0, B)
    L.check(st, "_prepare_hinv")
    L.raise_on_device_timeout(dev)  # the factor's tensor-core GEMMs finished every wait
    esc = used > damp
    if bool(esc.any()):
        log.warning("cholesky failed for %d/%d matrices, damp -> %.3g", int(esc.sum()), B, float(used.max()))
    return U if Cf == C else U[:, :C, :C].contiguous()


def _dead_columns(H: torch.Tensor) -> torch.Tensor:
    B, C, _ = H.shape
    dead = torch.empty(B, C, dtype=torch.uint8, device=H.device)
    L.check(L.lib().gq_dead_columns(L.ptr(H), B, C, L.ptr(dead), L.stream_ptr(H.device)), "dead columns")
    return dead


@torch.no_grad()
def _solve_mxfp(W_src: torch.Tensor, H: torch.Tensor, mode: str, damp: float, algorithm: str,
                W_out: torch.Tensor | None, want_rel: bool, dead: torch.Tensor,
                q_packed: torch.Tensor | None = None, wdq_dtype: torch.dtype = torch.float32):
    """gptq.py:69-180 on the GPU. W_src: original weights (any float dtype)."""
    if algorithm not in ("groupwise", "safe-scale-search"):
        raise ValueError(f"unsupported MXFP GPTQ algorithm: {algorithm}")
    B, R, C = W_src.shape
    dev = W_src.device
    G = C // MX_GROUP_SIZE
    lib, stream = L.lib(), L.stream_ptr(dev)
    U = torch.empty(B, G, 32, 32, dtype=torch.float32, device=dev)
    info = torch.empty(B, G, dtype=torch.int32, device=dev)
    L.check(lib.gq_mx_prepare_hinv(L.ptr(H), B, C, float(damp), L.ptr(U), L.ptr(info), None, stream),
            "mx prepare_hinv")
    q = torch.empty(B, R, C, dtype=torch.uint8, device=dev)
    scales = torch.empty(B, R, G, dtype=torch.uint8, device=dev)
    if W_out is None:
        W_out = torch.empty(B, R, C, dtype=wdq_dtype, device=dev)
    rel = torch.empty(B, dtype=torch.float32, device=dev) if want_rel else None
    ws = torch.empty(lib.gq_gptq_mxfp_workspace_size(B, R, C) if want_rel else 0, dtype=torch.uint8, device=dev)
    L.check(lib.gq_gptq_mxfp(L.ptr(W_src), L.DTYPE_CODE[W_src.dtype], L.ptr(H), L.ptr(U), L.ptr(dead),
                             L.ptr(info), B, R, C, L.MODE_CODE[mode],
                             L.GQ_MX_SAFE_SCALE_SEARCH if algorithm == "safe-scale-search" else L.GQ_MX_GROUPWISE,
                             L.ptr(q), L.ptr(q_packed), L.ptr(scales), L.ptr(W_out), L.DTYPE_CODE[W_out.dtype],
                             L.ptr(rel), L.ptr(ws), ws.numel(), stream), "gptq mxfp")
    L.raise_on_device_timeout(dev)  # a Hessian formed on this device finished every wait
    failed_groups = info != 0
    if bool(failed_groups.any()):
        raise _not_pd_error(H, failed_groups.any(dim=1), B)
    return q, scales, None, W_out, rel


@torch.no_grad()
def _solve_affine(W: torch.Tensor, W_orig: torch.Tensor | None, H: torch.Tensor, bits: int, group_size: int,
                  damp: float, clip: str, storage_dtype: torch.dtype, block_size: int, want_rel: bool):
    """gptq.py:229-272 on the GPU. W: float32 working weights (dead columns zeroed),
    overwritten with W_dq."""
    if clip not in L.CLIP_CODE:
        raise ValueError(f"unsupported clip method {clip}")
    if storage_dtype not in L.DTYPE_CODE:
        raise ValueError(f"unsupported storage dtype {storage_dtype}")
    B, R, C = W.shape
    dev = W.device
    lib, stream = L.lib(), L.stream_ptr(dev)
    U = _prepare_hinv(H, damp)
    q = torch.empty(B, R, C, dtype=torch.uint8, device=dev)
    ng = C // group_size
    scales = torch.empty(B, R, ng, dtype=storage_dtype, device=dev)
    biases = torch.empty(B, R, ng, dtype=storage_dtype, device=dev)
    rel = torch.empty(B, dtype=torch.float32, device=dev) if want_rel else None
    ws = torch.empty(lib.gq_gptq_affine_workspace_size(B, R, C, group_size, block_size), dtype=torch.uint8,
                     device=dev)
    L.check(lib.gq_gptq_affine(L.ptr(W), L.ptr(W_orig), L.DTYPE_CODE[W_orig.dtype] if W_orig is not None else 0,
                               L.ptr(U), B, R, C, bits, group_size, block_size, L.CLIP_CODE[clip],
                               L.DTYPE_CODE[storage_dtype], L.ptr(q), L.ptr(scales), L.ptr(biases), L.ptr(rel),
                               L.ptr(ws), ws.numel(), L.ptr(L.status_word(dev)), stream), "gptq affine")
    L.raise_on_device_timeout(dev)  # the trailing updates finished every wait
    return q, scales, biases, W, rel


def _check_args(W: torch.Tensor, H: torch.Tensor, group_size: int, mode: str):
    assert W.dim() == 3 and H.dim() == 3
    B, R, C = W.shape
    assert H.shape == (B, C, C)
    assert C % group_size == 0, f"in_features {C} not divisible by group {group_size}"
    if mode in ("mxfp4", "mxfp8") and group_size != MX_GROUP_SIZE:
        raise ValueError(f"{mode} requires group size {MX_GROUP_SIZE}")
    if mode not in ("affine", "mxfp4", "mxfp8"):
        raise ValueError(f"unsupported quantization mode: {mode}")
    if H.dtype != torch.float32:
        raise ValueError("H must be float32")


@torch.no_grad()
def gptq_quantize(W: torch.Tensor, H: torch.Tensor, bits: int, group_size: int, damp: float = 0.01,
                  clip: str = "mse", storage_dtype: torch.dtype = torch.bfloat16, block_size: int = 128,
                  mode: str = "affine", mxfp_algorithm: str = "auto"):
    """gptq.py:183-272. W [B, out, in] float32 is overwritten with W_dq; H [B, in, in]
    float32 gets unit diagonals on dead columns. Returns (q, scales, biases|None, W, None)."""
    _check_args(W, H, group_size, mode)
    L.require_cuda(W, H)
    if W.dtype != torch.float32 or not W.is_contiguous() or W.data_ptr() % 16:
        raise ValueError("gptq_quantize works in place on a contiguous float32 W")
    if not H.is_contiguous():
        raise ValueError("H must be contiguous (it is updated in place)")
    B, R, C = W.shape
    dead = _dead_columns(H)
    if mode in ("mxfp4", "mxfp8"):
        if mxfp_algorithm == "auto":
            mxfp_algorithm = "safe-scale-search" if mode == "mxfp4" else "groupwise"
        q, s, _, _, _ = _solve_mxfp(W, H, mode, damp, mxfp_algorithm, W, False, dead)
        return q, s, None, W, None
    L.check(L.lib().gq_prepare_weights(L.ptr(W), L.GQ_F32, L.ptr(dead), B, R, C, L.ptr(W),
                                       L.stream_ptr(W.device)), "prepare weights")
    q, s, b, W, _ = _solve_affine(W, None, H, bits, group_size, damp, clip, storage_dtype, block_size, False)
    return q, s, b, W, None


@torch.no_grad()
def solve_gptq(W_orig: torch.Tensor, H: torch.Tensor, bits: int, group_size: int, damp: float = 0.01,
               clip: str = "mse", storage_dtype: torch.dtype = torch.bfloat16, mode: str = "affine",
               mxfp_algorithm: str = "auto"):
    """gptq.py:275-302: keeps W_orig intact, returns (q, scales, biases|None, W_dq float32,
    rel_err [B]) with rel_err = ||W_dq - W_orig||_F / ||W_orig||_F."""
    _check_args(W_orig, H, group_size, mode)
    L.require_cuda(W_orig, H)
    if not H.is_contiguous():
        raise ValueError("H must be contiguous (it is updated in place)")
    if W_orig.dtype not in L.DTYPE_CODE:
        W_orig = W_orig.float()
    W0 = L.aligned(W_orig)
    B, R, C = W0.shape
    dead = _dead_columns(H)
    if mode in ("mxfp4", "mxfp8"):
        if mxfp_algorithm == "auto":
            mxfp_algorithm = "safe-scale-search" if mode == "mxfp4" else "groupwise"
        return _solve_mxfp(W0, H, mode, damp, mxfp_algorithm, None, True, dead)
    W = torch.empty(B, R, C, dtype=torch.float32, device=W0.device)
    L.check(L.lib().gq_prepare_weights(L.ptr(W0), L.DTYPE_CODE[W0.dtype], L.ptr(dead), B, R, C, L.ptr(W),
                                       L.stream_ptr(W0.device)), "prepare weights")
    return _solve_affine(W, W0, H, bits, group_size, damp, clip, storage_dtype, 128, True)
