"""numpy restatement of the reference's code packing -- TEST INFRASTRUCTURE.

mlx_gptq/packing.py:15-39 (MLX uint32 words, LSB first) and
mlx_gptq/artifacts.py:30-39 (two 4-bit codes per byte, low nibble first).
"""

from __future__ import annotations

import numpy as np

PACKABLE_BITS = (2, 4, 8)


def pack_q(q, bits):
    """packing.py:15-26."""
    if bits not in PACKABLE_BITS:
        raise ValueError(f"cannot pack {bits}-bit for MLX (supported: {PACKABLE_BITS})")
    per = 32 // bits
    q = np.asarray(q, np.uint8)
    *lead, C = q.shape
    assert C % per == 0
    qr = q.reshape(*lead, C // per, per).astype(np.uint32)
    words = np.zeros((*lead, C // per), np.uint32)
    for i in range(per):
        words |= qr[..., i] << np.uint32(bits * i)
    return words


def unpack_q(words, bits, out_cols):
    """packing.py:33-39."""
    per = 32 // bits
    mask = np.uint32((1 << bits) - 1)
    words = np.asarray(words, np.uint32)
    parts = [(words >> np.uint32(bits * i)) & mask for i in range(per)]
    q = np.stack(parts, axis=-1).reshape(*words.shape[:-1], words.shape[-1] * per)
    return q[..., :out_cols].astype(np.uint8)


def pack_nibbles(q):
    """artifacts.py:30-32."""
    q = np.asarray(q, np.uint8)
    assert q.shape[-1] % 2 == 0
    return (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(p):
    """artifacts.py:35-39."""
    p = np.asarray(p, np.uint8)
    return np.stack([p & 0xF, p >> 4], axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)
