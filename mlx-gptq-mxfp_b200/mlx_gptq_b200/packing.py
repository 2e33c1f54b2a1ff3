"""Code packing on the GPU, with the reference's API (mlx_gptq/packing.py).

``pack_q`` / ``unpack_q`` / ``pack_mxfp4`` accept numpy arrays (as the reference
does; the data makes a round trip through the current CUDA device) or CUDA
tensors (returned as CUDA tensors).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib as L

PACKABLE_BITS = (2, 4, 8)  # packing.py:13


def _to_cuda(x):
    if isinstance(x, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(x)).cuda(), True
    L.require_cuda(x)
    return L.aligned(x), False


def pack_q(q, bits: int):
    """packing.py:15-26: uint8 codes [..., C] -> uint32 words [..., C*bits/32], LSB first."""
    if bits not in PACKABLE_BITS:
        raise ValueError(f"cannot pack {bits}-bit for MLX (supported: {PACKABLE_BITS})")
    per = 32 // bits
    *lead, C = q.shape
    assert C % per == 0, f"last dim {C} not divisible by {per}"
    t, was_np = _to_cuda(q)
    t = t.to(torch.uint8)
    words = torch.empty(*lead, C // per, dtype=torch.int32, device=t.device)
    rows = t.numel() // C if C else 0
    L.check(L.lib().gq_pack_q(L.ptr(t), rows, C, bits, L.ptr(words), L.stream_ptr(t.device)), "pack_q")
    if was_np:
        return words.cpu().numpy().view(np.uint32)
    return words.view(torch.uint32) if hasattr(torch, "uint32") else words


def pack_mxfp4(q):
    """packing.py:29-30."""
    return pack_q(q, 4)


def unpack_q(words, bits: int, out_cols: int):
    """packing.py:33-39."""
    if bits not in PACKABLE_BITS:
        raise ValueError(f"cannot unpack {bits}-bit")
    if isinstance(words, np.ndarray):
        t, was_np = torch.from_numpy(np.ascontiguousarray(words).view(np.int32)).cuda(), True
    else:
        L.require_cuda(words)
        t, was_np = L.aligned(words.view(torch.int32) if words.dtype != torch.int32 else words), False
    *lead, nw = t.shape
    q = torch.empty(*lead, out_cols, dtype=torch.uint8, device=t.device)
    rows = t.numel() // nw if nw else 0
    L.check(L.lib().gq_unpack_q(L.ptr(t), rows, nw, bits, out_cols, L.ptr(q), L.stream_ptr(t.device)),
            "unpack_q")
    return q.cpu().numpy() if was_np else q
