"""numpy restatement of the reference's quantization grids -- TEST INFRASTRUCTURE.

Follows mlx_gptq/grid.py of the reference. All arithmetic is float32 with the
same operation order as the torch code (one rounding per torch op), so results
are bit-exact except where the reference sums a vector (the MSE clip search's
``sum(dim=-1)``), whose summation order torch does not document; there only
near-ties between candidate errors can differ.
"""

from __future__ import annotations

import numpy as np

from .log2_table import E_MAX, E_MIN, THRESHOLDS

F32 = np.float32
MX_GROUP_SIZE = 32  # grid.py:21
SUPPORTED_BITS = (2, 4, 8)  # grid.py:19

# grid.py:23-40 -- E2M1 code -> value, code bit 3 is the sign
E2M1_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)
_THRESH = np.array(THRESHOLDS, dtype=np.uint64)


def mode_defaults(mode: str) -> tuple[int, int]:
    """grid.py:43-50."""
    if mode == "mxfp4":
        return MX_GROUP_SIZE, 4
    if mode == "mxfp8":
        return MX_GROUP_SIZE, 8
    if mode == "affine":
        return 64, 4
    raise ValueError(f"unsupported quantization mode: {mode}")


def mxfp_max(mode: str) -> float:
    """grid.py:53-58."""
    if mode == "mxfp4":
        return 6.0
    if mode == "mxfp8":
        return 448.0
    raise ValueError(f"not a microscaling mode: {mode}")


# ---------------------------------------------------------------------------
# storage-dtype rounding
# ---------------------------------------------------------------------------


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 (round to nearest even) -> float32, as torch's
    ``.to(torch.bfloat16).float()``; NaN maps to the canonical quiet NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    r = np.where(np.isnan(x), np.uint64(0x7FC00000), r)
    return r.astype(np.uint32).view(np.float32).reshape(x.shape)


def to_storage(x: np.ndarray, storage: str) -> np.ndarray:
    """``.to(storage_dtype).float()`` for bfloat16 / float16 / float32."""
    if storage == "bfloat16":
        return round_to_bf16(x)
    if storage == "float16":
        return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
    if storage == "float32":
        return np.asarray(x, np.float32)
    raise ValueError(f"unsupported storage dtype {storage}")


# ---------------------------------------------------------------------------
# MLX affine grid
# ---------------------------------------------------------------------------


def choose_qparams(w, bits, method="mse", storage="bfloat16", grid_steps=20, max_shrink=0.2):
    """grid.py:167-212. Groups are the last axis of ``w`` (float32).

    The Python-double factors ``p / maxq`` and ``p`` are cast to float32 before
    the tensor multiply, as torch does for a float32 tensor times a scalar.
    Returns (scales, biases) already rounded through the storage dtype (float32
    copies); the stored tensors are these values in the storage dtype.
    """
    w = np.asarray(w, np.float32)
    maxq = float(2**bits - 1)
    wmin = w.min(axis=-1)
    wmax = w.max(axis=-1)
    if method == "minmax":
        shrinks = [1.0]
    elif method == "mse":
        shrinks = [1.0 - max_shrink * i / grid_steps for i in range(grid_steps + 1)]
    else:
        raise ValueError(f"unsupported clip method {method}")
    rng = (wmax - wmin).astype(np.float32)
    best_err = best_s = best_b = None
    for p in shrinks:
        s = to_storage(rng * F32(p / maxq), storage)
        b = to_storage(wmin * F32(p), storage)
        s_safe = np.where(np.abs(s) < F32(1e-12), F32(1.0), s)
        q = np.clip(np.rint((w - b[..., None]) / s_safe[..., None]), F32(0.0), F32(maxq))
        dq = q * s[..., None] + b[..., None]
        d = dq - w
        err = (d * d).sum(axis=-1, dtype=np.float32)
        if best_err is None:
            best_err, best_s, best_b = err, s, b
        else:
            better = err < best_err
            best_err = np.where(better, err, best_err)
            best_s = np.where(better, s, best_s)
            best_b = np.where(better, b, best_b)
    return best_s.astype(np.float32), best_b.astype(np.float32)


def quantize_with_params(w, s32, b32, bits):
    """grid.py:215-221. Returns (q float32, dq float32)."""
    maxq = float(2**bits - 1)
    s_safe = np.where(np.abs(s32) < F32(1e-12), F32(1.0), s32).astype(np.float32)
    q = np.clip(np.rint((w - b32[..., None]) / s_safe[..., None]), F32(0.0), F32(maxq))
    dq = q * s32[..., None] + b32[..., None]
    return q.astype(np.float32), dq.astype(np.float32)


def rtn_quantize(W, bits, group_size, method="mse", storage="bfloat16"):
    """grid.py:224-246. W [..., R, C] -> (q uint8, scales, biases, W_dq)."""
    W = np.asarray(W, np.float32)
    *lead, R, C = W.shape
    assert C % group_size == 0
    wg = W.reshape(*lead, R, C // group_size, group_size)
    s, b = choose_qparams(wg, bits, method, storage)
    q, dq = quantize_with_params(wg, s, b, bits)
    return q.astype(np.uint8).reshape(*lead, R, C), s, b, dq.reshape(*lead, R, C)


# ---------------------------------------------------------------------------
# native MXFP grids (E2M1 / E4M3 values, E8M0 shared scale per 32)
# ---------------------------------------------------------------------------


def mx_scale_exponent(max_abs: np.ndarray, mode: str) -> np.ndarray:
    """grid.py:68-73: exponent = clamp(round(log2(max_abs / fmax)), -127, 127),
    0 when max_abs == 0.

    With y = max_abs / fmax = m * 2**E, the rounded log2 is E + (bits(y) >= T[E])
    where T is the threshold table measured from the reference's torch
    arithmetic (oracle/make_log2_table.py). Non-finite y (an inf/NaN weight)
    gives -127, which is what torch's float->int32 cast plus clamp yields on x86.
    """
    fmax = F32(mxfp_max(mode))
    max_abs = np.asarray(max_abs, np.float32)
    safe = np.where(max_abs == 0, fmax, max_abs).astype(np.float32)
    y = (safe / fmax).astype(np.float32)
    bits = y.view(np.uint32).astype(np.int64)
    efield = (bits >> 23) & 0xFF
    # E = floor(log2(y)). Among subnormals only the binade [2**-127, 2**-126)
    # (bit patterns >= 0x00400000) can still round up; anything lower ends at -127.
    E = np.where(efield == 0, np.where(bits >= 0x00400000, -127, -128), efield - 127)
    idx = np.clip(E - E_MIN, 0, E_MAX - E_MIN)
    up = (bits.astype(np.uint64) >= _THRESH[idx]).astype(np.int64)
    ex = E + up
    ex = np.where(E < E_MIN, -127, ex)
    ex = np.clip(ex, -127, 127)
    ex = np.where(~np.isfinite(y), -127, ex)
    ex = np.where(max_abs == 0, 0, ex)
    return ex.astype(np.int32)


def exp2_scale(exponent: np.ndarray) -> np.ndarray:
    """torch.pow(2.0, exponent) for integer exponents in [-127, 127] (exact)."""
    return np.ldexp(np.float32(1.0), np.asarray(exponent, np.int32)).astype(np.float32)


def choose_mxfp_scale(w, mode):
    """grid.py:61-79: w [..., 32] -> (scale bytes uint8, scales float32)."""
    w = np.asarray(w, np.float32)
    max_abs = np.abs(w).max(axis=-1)
    ex = mx_scale_exponent(max_abs, mode)
    return (ex + 127).astype(np.uint8), exp2_scale(ex)


def e2m1_codes(x):
    """grid.py:82-105. Nested thresholds restated as a count of passed edges."""
    x = np.asarray(x, np.float32)
    ax = np.abs(x)
    mag = ((ax > 0.25).astype(np.uint8) + (ax >= 0.75) + (ax > 1.25) + (ax >= 1.75)
           + (ax > 2.5) + (ax >= 3.5) + (ax > 5.0)).astype(np.uint8)
    return mag | ((x < 0).astype(np.uint8) << 3)


def e4m3_encode(x):
    """float32 -> float8_e4m3fn bits, round to nearest even; |x| >= 480 and NaN
    give the NaN code 0x7F (sign kept). Same mapping as torch's e4m3fn cast,
    which the reference applies after clamping to +-448 (grid.py:115-121)."""
    x = np.asarray(x, np.float32)
    u = x.view(np.uint32).astype(np.int64)
    sign = ((u >> 31) & 1).astype(np.uint8) << 7
    a = u & 0x7FFFFFFF
    ax = a.astype(np.uint32).view(np.float32)
    # subnormal range |x| < 2**-6: value k * 2**-9, k = rne(|x| * 512) in [0, 8]
    k = np.rint(ax * F32(512.0)).astype(np.int64)
    sub = k
    # normal range: keep 3 mantissa bits with round-to-nearest-even
    e = (a >> 23) - 127
    m = a & 0x7FFFFF
    q = m >> 20
    rem = m & 0xFFFFF
    up = (rem > 0x80000) | ((rem == 0x80000) & ((q & 1) == 1))
    q = q + up
    e = e + (q >> 3)
    q = q & 7
    norm = ((e + 7) << 3) | q
    code = np.where(a < 0x3C800000, sub, norm)  # 0x3C800000 == 2**-6
    code = np.where(a >= 0x43F00000, 0x7F, code)  # 0x43F00000 == 480.0, also inf/NaN
    return (code.astype(np.uint8) | sign).astype(np.uint8)


def e4m3_decode(code):
    """float8_e4m3fn bits -> float32 (torch's ``.float()`` of an e4m3fn tensor)."""
    c = np.asarray(code, np.uint8).astype(np.int64)
    s = np.where(c & 0x80, F32(-1.0), F32(1.0))
    ef = (c >> 3) & 0xF
    mt = c & 7
    val = np.where(ef == 0, mt.astype(np.float32) * F32(2.0**-9),
                   np.ldexp((8 + mt).astype(np.float32) / F32(8.0), (ef - 7).astype(np.int32)))
    val = (s * val).astype(np.float32)
    return np.where((c & 0x7F) == 0x7F, np.float32(np.nan), val).astype(np.float32)


def quantize_mxfp_with_scale(w, scales, mode):
    """grid.py:108-124: fixed per-group scales -> (codes uint8, dq float32)."""
    w = np.asarray(w, np.float32)
    sc = np.asarray(scales, np.float32)[..., None]
    normalized = (w / sc).astype(np.float32)
    if mode == "mxfp4":
        q = e2m1_codes(normalized)
        dq = E2M1_VALUES[q] * sc
    elif mode == "mxfp8":
        bounded = np.clip(normalized, F32(-448.0), F32(448.0))
        q = e4m3_encode(bounded)
        dq = e4m3_decode(q) * sc
    else:
        raise ValueError(f"not a microscaling mode: {mode}")
    return q, dq.astype(np.float32)


def dequantize_mxfp(q, scale_bytes, mode):
    """grid.py:127-139."""
    q = np.asarray(q, np.uint8)
    scales = exp2_scale(np.asarray(scale_bytes).astype(np.int32) - 127)
    if mode == "mxfp4":
        values = E2M1_VALUES[q]
    elif mode == "mxfp8":
        values = e4m3_decode(q)
    else:
        raise ValueError(f"not a microscaling mode: {mode}")
    return values.reshape(*q.shape[:-1], -1, MX_GROUP_SIZE) * scales[..., None]


def rtn_quantize_mxfp(W, mode):
    """grid.py:142-151. W [..., R, C] -> (q uint8, scale bytes, None, W_dq)."""
    W = np.asarray(W, np.float32)
    *lead, R, C = W.shape
    if C % MX_GROUP_SIZE:
        raise ValueError(f"columns {C} not divisible by {MX_GROUP_SIZE}")
    g = W.reshape(*lead, R, C // MX_GROUP_SIZE, MX_GROUP_SIZE)
    sb, sc = choose_mxfp_scale(g, mode)
    q, dq = quantize_mxfp_with_scale(g, sc, mode)
    return q.reshape(*lead, R, C), sb, None, dq.reshape(*lead, R, C)


def dequantize_artifact(q, scales, biases, mode, group_size):
    """grid.py:154-164."""
    q = np.asarray(q)
    if mode == "affine":
        s = np.asarray(scales, np.float32)
        b = np.asarray(biases, np.float32)
        out = q.astype(np.float32).reshape(*q.shape[:-1], -1, group_size) * s[..., None] + b[..., None]
        return out.reshape(q.shape).astype(np.float32)
    if group_size != MX_GROUP_SIZE:
        raise ValueError(f"{mode} requires group size {MX_GROUP_SIZE}")
    return dequantize_mxfp(q, scales, mode).reshape(q.shape)
