"""numpy restatement of the reference's Hessian accumulation -- TEST INFRASTRUCTURE.

mlx_gptq/capture.py:68-76 (Stash.hessian): H = sum over chunks of x^T x with x
the bf16 rows upcast to float32, accumulated in float32, chunks of 65536 rows.
No 1/n factor. The grouped form (one H per expert over its routed token rows)
is what mlx_gptq/sequential.py:546-555 builds by calling Stash.hessian once per
expert stash.
"""

from __future__ import annotations

import numpy as np


def bf16_bits_to_f32(x_bits: np.ndarray) -> np.ndarray:
    """uint16 bfloat16 bit patterns -> float32 (exact)."""
    return (np.asarray(x_bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def hessian(X: np.ndarray, chunk_rows: int = 65536) -> np.ndarray:
    """capture.py:68-76. X: float32 values that are exactly bf16 [N, C]."""
    X = np.asarray(X, np.float32)
    N, C = X.shape
    H = np.zeros((C, C), np.float32)
    for i in range(0, N, chunk_rows):
        x = X[i:i + chunk_rows]
        H += x.T @ x
    return H


def hessian_grouped(X: np.ndarray, token_idx: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    """One H per expert e over rows X[token_idx[offsets[e]:offsets[e+1]]]."""
    X = np.asarray(X, np.float32)
    E = len(offsets) - 1
    C = X.shape[1]
    H = np.zeros((E, C, C), np.float32)
    for e in range(E):
        rows = token_idx[offsets[e]:offsets[e + 1]]
        if len(rows):
            H[e] = hessian(X[rows])
    return H
