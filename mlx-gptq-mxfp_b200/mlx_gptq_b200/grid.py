"""Quantization grids on the GPU, with the reference's Python API.

Mirrors mlx_gptq/grid.py of the reference (names, arguments, dtypes, errors):
the MLX affine grid (MSE range-shrink clip search, storage-rounded scale/bias)
and the native MXFP4 / MXFP8 grids (E2M1 / E4M3 codes, E8M0 scale per 32).
Every function runs the CUDA kernels of libgptq_b200.so; inputs must be CUDA
tensors.
"""

from __future__ import annotations

import torch

from . import _lib as L

SUPPORTED_BITS = (2, 4, 8)  # grid.py:19
SUPPORTED_MODES = ("affine", "mxfp4", "mxfp8")  # grid.py:20
MX_GROUP_SIZE = 32  # grid.py:21

_E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def mode_defaults(mode: str) -> tuple[int, int]:
    """grid.py:43-50: (group_size, bits) of a mode."""
    if mode == "mxfp4":
        return MX_GROUP_SIZE, 4
    if mode == "mxfp8":
        return MX_GROUP_SIZE, 8
    if mode == "affine":
        return 64, 4
    raise ValueError(f"unsupported quantization mode: {mode}")


def _mxfp_max(mode: str) -> float:
    """grid.py:53-58."""
    if mode == "mxfp4":
        return 6.0
    if mode == "mxfp8":
        return 448.0
    raise ValueError(f"not a microscaling mode: {mode}")


def _dtype_code(dtype: torch.dtype) -> int:
    try:
        return L.DTYPE_CODE[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


@torch.no_grad()
def rtn_quantize(W: torch.Tensor, bits: int, group_size: int, method: str = "mse",
                 storage_dtype: torch.dtype = torch.bfloat16):
    """grid.py:224-246: RTN on the MLX grid (no Hessian). W [..., rows, cols].

    Returns (q uint8 [..., rows, cols], scales, biases [..., rows, cols/G] in
    storage_dtype, W_dq float32)."""
    *lead, R, C = W.shape
    assert C % group_size == 0, f"cols {C} not divisible by group size {group_size}"
    dev = L.require_cuda(W)
    if method not in L.CLIP_CODE:
        raise ValueError(f"unsupported clip method {method}")
    Wc = L.aligned(W)
    rows = Wc.numel() // C if C else 0
    q = torch.empty(*lead, R, C, dtype=torch.uint8, device=dev)
    s = torch.empty(*lead, R, C // group_size, dtype=storage_dtype, device=dev)
    b = torch.empty_like(s)
    dq = torch.empty(*lead, R, C, dtype=torch.float32, device=dev)
    L.check(L.lib().gq_rtn_affine(L.ptr(Wc), _dtype_code(Wc.dtype), rows, C, bits, group_size,
                                  L.CLIP_CODE[method], _dtype_code(storage_dtype), L.ptr(q), L.ptr(s),
                                  L.ptr(b), L.ptr(dq), L.GQ_F32, L.stream_ptr(dev)), "rtn_quantize")
    return q, s, b, dq


@torch.no_grad()
def choose_qparams(w: torch.Tensor, bits: int, method: str = "mse",
                   storage_dtype: torch.dtype = torch.bfloat16, grid_steps: int = 20,
                   max_shrink: float = 0.2):
    """grid.py:167-212 for groups on the last axis (group size 32/64/128/256).

    Returns (scales_stored, biases_stored, scales_f32, biases_f32)."""
    if grid_steps != 20 or max_shrink != 0.2:
        raise ValueError("the GPU clip search implements grid_steps=20, max_shrink=0.2")
    G = w.shape[-1]
    _, s, b, _ = rtn_quantize(w.reshape(-1, G), bits, G, method, storage_dtype)
    shape = w.shape[:-1]
    s, b = s.reshape(shape), b.reshape(shape)
    return s, b, s.float(), b.float()


@torch.no_grad()
def rtn_quantize_mxfp(W: torch.Tensor, mode: str):
    """grid.py:142-151: native MXFP RTN. Returns (q, scale bytes, None, W_dq)."""
    *lead, R, C = W.shape
    if C % MX_GROUP_SIZE:
        raise ValueError(f"columns {C} not divisible by {MX_GROUP_SIZE}")
    if mode not in ("mxfp4", "mxfp8"):
        raise ValueError(f"not a microscaling mode: {mode}")
    dev = L.require_cuda(W)
    Wc = L.aligned(W)
    rows = Wc.numel() // C if C else 0
    q = torch.empty(*lead, R, C, dtype=torch.uint8, device=dev)
    s = torch.empty(*lead, R, C // MX_GROUP_SIZE, dtype=torch.uint8, device=dev)
    dq = torch.empty(*lead, R, C, dtype=torch.float32, device=dev)
    L.check(L.lib().gq_rtn_mxfp(L.ptr(Wc), _dtype_code(Wc.dtype), rows, C, L.MODE_CODE[mode], L.ptr(q), None,
                                L.ptr(s), L.ptr(dq), L.GQ_F32, L.stream_ptr(dev)), "rtn_quantize_mxfp")
    return q, s, None, dq


@torch.no_grad()
def choose_mxfp_scale(w: torch.Tensor, mode: str):
    """grid.py:61-79: E8M0 scales for 32-value groups (last axis of size 32)."""
    if w.shape[-1] != MX_GROUP_SIZE:
        raise ValueError(f"choose_mxfp_scale expects groups of {MX_GROUP_SIZE} on the last axis")
    _mxfp_max(mode)
    _, s, _, _ = rtn_quantize_mxfp(w.reshape(-1, MX_GROUP_SIZE), mode)
    s = s.reshape(w.shape[:-1])
    return s, e8m0_to_float(s)


def e8m0_to_float(scale_bytes: torch.Tensor) -> torch.Tensor:
    """Exact float32 2**(byte - 127) from E8M0 bytes (byte 0 is the subnormal 2**-127)."""
    bits = scale_bytes.to(torch.int32) << 23
    bits = torch.where(scale_bytes == 0, torch.full_like(bits, 0x00400000), bits)
    return bits.view(torch.float32)


@torch.no_grad()
def dequantize_artifact(q: torch.Tensor, scales: torch.Tensor, biases, mode: str, group_size: int):
    """grid.py:154-164: dequantize one Stage-A artifact (float32 out)."""
    if mode not in L.MODE_CODE:
        raise ValueError(f"unsupported quantization mode: {mode}")
    if mode != "affine" and group_size != MX_GROUP_SIZE:
        raise ValueError(f"{mode} requires group size {MX_GROUP_SIZE}")
    dev = L.require_cuda(q, scales, biases)
    qc, sc = L.aligned(q), L.aligned(scales)
    bc = None if biases is None else L.aligned(biases)
    C = q.shape[-1]
    rows = qc.numel() // C if C else 0
    out = torch.empty(q.shape, dtype=torch.float32, device=dev)
    sdt = _dtype_code(sc.dtype) if mode == "affine" else L.GQ_F32
    L.check(L.lib().gq_dequantize(L.ptr(qc), L.ptr(sc), L.ptr(bc), sdt, rows, C, L.MODE_CODE[mode],
                                  group_size, L.ptr(out), L.stream_ptr(dev)), "dequantize_artifact")
    return out


def dequantize_mxfp(q: torch.Tensor, scale_bytes: torch.Tensor, mode: str):
    """grid.py:127-139: returns [..., C/32, 32] float32."""
    out = dequantize_artifact(q, scale_bytes, None, mode, MX_GROUP_SIZE)
    return out.reshape(*q.shape[:-1], -1, MX_GROUP_SIZE)
