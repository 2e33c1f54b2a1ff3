"""numpy restatement of the reference's batched GPTQ solver -- TEST INFRASTRUCTURE.

Follows mlx_gptq/gptq.py of the reference (W [B, R, C], H [B, C, C], float32).
The linear algebra uses numpy/scipy LAPACK in float32 where the reference uses
torch's (cholesky_ex / cholesky_inverse / cholesky); those differ from torch's
only in rounding, which is why solver parity is stated as code agreement and
proxy loss, not bit equality.
"""

from __future__ import annotations

import logging

import numpy as np

from . import grid

log = logging.getLogger(__name__)
F32 = np.float32


class NotPositiveDefinite(RuntimeError):
    pass


def _cholesky_lower(A: np.ndarray):
    """Batched float32 Cholesky with a per-item success flag (cholesky_ex)."""
    B = A.shape[0]
    L = np.zeros_like(A)
    ok = np.ones(B, dtype=bool)
    try:
        L[:] = np.linalg.cholesky(A)
        ok &= np.isfinite(L).all(axis=(1, 2))
        return L, ok
    except np.linalg.LinAlgError:
        pass
    for b in range(B):
        try:
            L[b] = np.linalg.cholesky(A[b])
            ok[b] = bool(np.isfinite(L[b]).all())
        except np.linalg.LinAlgError:
            ok[b] = False
    return L, ok


def prepare_hinv(H: np.ndarray, damp: float, max_attempts: int = 6):
    """gptq.py:27-66: upper Cholesky factor of (H + damp*mean(diag H)*I)^-1,
    escalating damping x10 for items whose factorization fails (<= 6 tries).

    Returns (U, damp_used)."""
    H = np.asarray(H, np.float32)
    B, C, _ = H.shape
    idx = np.arange(C)
    diag_mean = np.maximum(H[:, idx, idx].mean(axis=-1, dtype=np.float32), F32(1e-8)).astype(np.float32)
    cur = np.full(B, damp, dtype=np.float32)
    Hd = H.copy()
    Hd[:, idx, idx] += (diag_mean * cur)[:, None]
    for _ in range(max_attempts):
        L, ok = _cholesky_lower(Hd)
        failed = ~ok
        if not failed.any():
            break
        cur[failed] *= F32(10.0)
        Hd[failed] = H[failed]
        fi = np.nonzero(failed)[0]
        Hd[fi[:, None], idx, idx] += (diag_mean[failed] * cur[failed])[:, None]
        log.warning("cholesky failed for %d/%d matrices, damp -> %.3g",
                    int(failed.sum()), B, float(cur[failed].max()))
    else:
        bad = H[failed]
        diag = bad[:, idx, idx]
        raise NotPositiveDefinite(
            "Hessian not positive definite after damping escalation; "
            f"batch={B} failed={int(failed.sum())} "
            f"nonfinite={int((~np.isfinite(bad)).sum())} "
            f"diag_min={float(diag.min())} diag_max={float(diag.max())} "
            f"value_min={float(bad.min())} value_max={float(bad.max())}"
        )
    # cholesky_inverse(L) = (L L^T)^-1 = L^-T L^-1, then its upper Cholesky factor
    Linv = np.linalg.inv(L).astype(np.float32)
    Linv = np.tril(Linv)
    Hinv = np.matmul(np.swapaxes(Linv, 1, 2), Linv).astype(np.float32)
    Lh, ok = _cholesky_lower(Hinv)
    if not ok.all():
        raise NotPositiveDefinite("inverse Hessian factorization failed")
    return np.swapaxes(Lh, 1, 2).copy(), cur


def _mxfp_groupwise(W, H, mode, damp, algorithm):
    """gptq.py:69-180: per-32-column GPTQ inside each native scale group."""
    B, R, Ccols = W.shape
    G = grid.MX_GROUP_SIZE
    groups = Ccols // G
    q_out = np.empty((B, R, Ccols), np.uint8)
    scales = np.empty((B, R, groups), np.uint8)
    if algorithm not in ("groupwise", "safe-scale-search"):
        raise ValueError(f"unsupported MXFP GPTQ algorithm: {algorithm}")
    offsets = (0, -1, -2, -3, -4, 1, 2) if mode == "mxfp4" else (0, -1, 1)

    def objective(e, Hg):  # einsum("bri,bij,brj->br"), contracted left to right
        return (np.matmul(e, Hg) * e).sum(axis=-1, dtype=np.float32)

    for g in range(groups):
        s0, s1 = g * G, (g + 1) * G
        original = W[:, :, s0:s1].copy()
        Wg = original.copy()
        Hg = H[:, s0:s1, s0:s1]
        U, _ = prepare_hinv(Hg, damp)
        if algorithm == "groupwise":
            sbytes, svals = grid.choose_mxfp_scale(original, mode)
            base_q, base_dq = grid.quantize_mxfp_with_scale(original, svals, mode)
        else:
            bb, _ = grid.choose_mxfp_scale(original, mode)
            bexp = bb.astype(np.int32) - 127
            best = None
            for off in offsets:
                ex = np.clip(bexp + off, -127, 127)
                cb = (ex + 127).astype(np.uint8)
                cs = grid.exp2_scale(ex)
                cq, cdq = grid.quantize_mxfp_with_scale(original, cs, mode)
                obj = objective(cdq - original, Hg)
                if best is None:
                    best, base_q, base_dq, sbytes, svals = obj, cq, cdq, cb, cs
                else:
                    better = obj < best
                    best = np.where(better, obj, best)
                    base_q = np.where(better[..., None], cq, base_q)
                    base_dq = np.where(better[..., None], cdq, base_dq)
                    sbytes = np.where(better, cb, sbytes)
                    svals = np.where(better, cs, svals)
        scales[:, :, g] = sbytes
        gq = np.empty_like(original, dtype=np.uint8)
        gdq = np.empty_like(original)
        for c in range(G):
            col = Wg[:, :, c]
            q, dq = grid.quantize_mxfp_with_scale(col[..., None], svals, mode)
            q, dq = q[..., 0], dq[..., 0]
            d = U[:, c, c][:, None]
            err = ((col - dq) / d).astype(np.float32)
            if c + 1 < G:
                Wg[:, :, c + 1:] -= err[..., None] * U[:, c, c + 1:][:, None, :]
            gq[:, :, c] = q
            gdq[:, :, c] = dq
        if algorithm == "groupwise":
            sel_q, sel_dq = gq, gdq
        else:
            gobj = objective(gdq - original, Hg)
            use = gobj <= best
            sel_q = np.where(use[..., None], gq, base_q)
            sel_dq = np.where(use[..., None], gdq, base_dq)
        smax = np.abs(original).max(axis=-1, keepdims=True)
        limit = np.maximum(smax * F32(32.0), F32(2.0**-126))
        valid = (np.abs(sel_dq) <= limit).all(axis=-1, keepdims=True)
        sel_q = np.where(valid, sel_q, base_q)
        sel_dq = np.where(valid, sel_dq, base_dq)
        q_out[:, :, s0:s1] = sel_q
        W[:, :, s0:s1] = sel_dq
    return q_out, scales, None, W


def gptq_quantize(W, H, bits, group_size, damp=0.01, clip="mse", storage="bfloat16",
                  block_size=128, mode="affine", mxfp_algorithm="auto"):
    """gptq.py:183-272. W [B,R,C] float32 is modified in place (returns W_dq);
    H [B,C,C] float32 has dead-column diagonals set to 1 in place."""
    assert W.ndim == 3 and H.ndim == 3
    B, R, C = W.shape
    assert H.shape == (B, C, C)
    assert C % group_size == 0
    if mode in ("mxfp4", "mxfp8") and group_size != grid.MX_GROUP_SIZE:
        raise ValueError(f"{mode} requires group size {grid.MX_GROUP_SIZE}")
    idx = np.arange(C)
    dead = H[:, idx, idx] <= 0  # gptq.py:216-222
    if dead.any():
        W[np.broadcast_to(dead[:, None, :], W.shape)] = 0.0
        for b in range(B):
            H[b, idx[dead[b]], idx[dead[b]]] = 1.0
    if mode in ("mxfp4", "mxfp8"):
        if mxfp_algorithm == "auto":
            mxfp_algorithm = "safe-scale-search" if mode == "mxfp4" else "groupwise"
        return _mxfp_groupwise(W, H, mode, damp, mxfp_algorithm)
    if mode != "affine":
        raise ValueError(f"unsupported quantization mode: {mode}")
    U, _ = prepare_hinv(H, damp)
    bs = max(block_size, group_size)
    bs -= bs % group_size
    ng = C // group_size
    q_out = np.empty((B, R, C), np.uint8)
    scales = np.empty((B, R, ng), np.float32)
    biases = np.empty((B, R, ng), np.float32)
    s32 = b32 = None
    for i1 in range(0, C, bs):
        i2 = min(i1 + bs, C)
        n = i2 - i1
        W1 = W[:, :, i1:i2].copy()
        Err = np.zeros((B, R, n), np.float32)
        U1 = U[:, i1:i2, i1:i2]
        for j in range(n):
            col = i1 + j
            if col % group_size == 0:
                g = col // group_size
                s32, b32 = grid.choose_qparams(W1[:, :, j:j + group_size], bits, clip, storage)
                scales[:, :, g] = s32
                biases[:, :, g] = b32
            w = W1[:, :, j]
            q, dq = grid.quantize_with_params(w[..., None], s32, b32, bits)
            q, dq = q[..., 0], dq[..., 0]
            d = U1[:, j, j][:, None]
            e = ((w - dq) / d).astype(np.float32)
            if j + 1 < n:
                W1[:, :, j + 1:] -= e[..., None] * U1[:, j, j + 1:][:, None, :]
            Err[:, :, j] = e
            q_out[:, :, col] = q.astype(np.uint8)
            W[:, :, col] = dq
        if i2 < C:
            W[:, :, i2:] -= np.matmul(Err, U[:, i1:i2, i2:]).astype(np.float32)
    return q_out, scales, biases, W


def solve_gptq(W_orig, H, bits, group_size, damp=0.01, clip="mse", storage="bfloat16",
               mode="affine", mxfp_algorithm="auto"):
    """gptq.py:275-302: clones W, solves, returns (q, s, b, W_dq, rel_err[B])."""
    W0 = np.asarray(W_orig, np.float32)
    W = W0.copy()
    q, s, b, Wdq = gptq_quantize(W, H, bits, group_size, damp=damp, clip=clip, storage=storage,
                                 mode=mode, mxfp_algorithm=mxfp_algorithm)
    num = np.sqrt(((Wdq - W0) ** 2).sum(axis=(1, 2), dtype=np.float64))
    den = np.maximum(np.sqrt((W0.astype(np.float64) ** 2).sum(axis=(1, 2))), 1e-12)
    return q, s, b, Wdq, (num / den).astype(np.float32)


def proxy_loss(W, Wq, H):
    """tr((W - Q) H (W - Q)^T) per batch item, float64 (the solver's objective)."""
    D = np.asarray(Wq, np.float64) - np.asarray(W, np.float64)
    return np.einsum("bri,bij,brj->b", D, np.asarray(H, np.float64), D)
