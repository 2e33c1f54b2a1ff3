"""Generate golden vectors from the REAL reference (mlx_gptq, torch CPU).

Run in the development container, where the reference checkout is importable:

    python tests/golden/make_golden.py [--ref PATH_TO_REFERENCE_CHECKOUT]

Writes small .npz fixtures next to this file. The fixtures are committed; the
tests read only them (the reference itself is not available on the GPU box).
Every input is generated from a fixed seed and stored alongside the reference
outputs, so a fixture is self-contained.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
STORAGE = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _f32(t):
    return t.detach().to(torch.float32).cpu().numpy()


def _u8(t):
    return t.detach().cpu().numpy().astype(np.uint8)


def rtn_affine_cases(grid):
    out = {}
    g = torch.Generator().manual_seed(101)
    W = torch.randn(8, 256, generator=g) * torch.linspace(0.02, 4.0, 8).unsqueeze(1)
    W[0, 3] = 12.0
    W[1, 64:128] = 0.0  # constant (zero-range) group -> s == 0 path
    W[2, 128:192] = 0.37  # constant non-zero group
    W[3, :64] = torch.linspace(-1, 1, 64)
    out["W"] = _f32(W)
    for bits in (2, 4, 8):
        for gs in (32, 64, 128):
            for method in ("mse", "minmax"):
                for st in ("bfloat16", "float16", "float32"):
                    q, s, b, dq = grid.rtn_quantize(W.clone(), bits, gs, method=method,
                                                    storage_dtype=STORAGE[st])
                    k = f"{bits}_{gs}_{method}_{st}"
                    out[f"q_{k}"] = _u8(q)
                    out[f"s_{k}"] = _f32(s)
                    out[f"b_{k}"] = _f32(b)
                    out[f"dq_{k}"] = _f32(dq)
    return out


def _boundary_maxes(fmax):
    """float32 group maxima that put max/fmax on both sides of every rounding
    threshold of round(log2(.)), plus exact powers of two and subnormals."""
    sys.path.insert(0, os.path.join(HERE, "..", ".."))
    from oracle.log2_table import THRESHOLDS  # the table under test

    vals = []
    for t in THRESHOLDS:
        y = np.array([t], np.uint32).view(np.float32)[0]
        if not np.isfinite(y):
            continue
        x = np.float32(np.float64(y) * fmax)
        if not np.isfinite(x) or x == 0:
            continue
        xb = int(np.array([x], np.float32).view(np.uint32)[0])
        for d in range(-3, 4):
            if 0 < xb + d < 0x7F800000:
                vals.append(np.array([xb + d], np.uint32).view(np.float32)[0])
    for e in range(-149, 128):
        vals.append(np.float32(np.ldexp(1.0, e)))
        vals.append(np.float32(np.ldexp(1.0, e) * fmax))
    vals = np.array([v for v in vals if np.isfinite(v) and v > 0], np.float32)
    return vals


def rtn_mxfp_cases(grid):
    out = {}
    g = torch.Generator().manual_seed(23)
    for mode, fmax in (("mxfp4", 6.0), ("mxfp8", 448.0)):
        W = torch.randn(17, 96, generator=g) * torch.linspace(0.01, 8.0, 17).unsqueeze(1)
        W[0, :32] = 0.0
        W[1, :32] = torch.tensor([6.0, -6.0, 5.0, -5.0, 4.99, 3.5, 3.49, 2.5, 2.51, 1.75,
                                  1.74, 1.25, 1.26, 0.75, 0.74, 0.25, 0.26, -0.25, -0.26,
                                  0.0, -0.0, 448.0, -448.0, 447.0, 449.0, 1e-30, -1e-30,
                                  1e-40, 2.0, 3.0, -3.0, 1.0])
        W[2, 32:64] = torch.linspace(-448.0, 448.0, 32)
        W[3, 64:96] = torch.full((32,), 1e-39)
        q, s, b, dq = grid.rtn_quantize_mxfp(W.clone(), mode)
        out[f"W_{mode}"] = _f32(W)
        out[f"q_{mode}"] = _u8(q)
        out[f"s_{mode}"] = _u8(s)
        out[f"dq_{mode}"] = _f32(dq)
        # exponent boundaries: each group = [max, small random values]
        maxes = _boundary_maxes(fmax)
        n = len(maxes)
        Wb = torch.rand(n, 32, generator=g) * 0.5
        Wb = Wb * torch.from_numpy(maxes).unsqueeze(1)
        Wb[:, 7] = torch.from_numpy(maxes)
        Wb[::2, 7] *= -1.0
        q, s, b, dq = grid.rtn_quantize_mxfp(Wb.clone(), mode)
        out[f"Wb_{mode}"] = _f32(Wb)
        out[f"qb_{mode}"] = _u8(q)
        out[f"sb_{mode}"] = _u8(s)
        out[f"dqb_{mode}"] = _f32(dq)
    return out


def e4m3_cases():
    """torch's e4m3fn cast on a strided sweep of every float32 in [-480, 480]."""
    step = 4099
    pos = np.arange(0, 0x43F00000 + step, step, dtype=np.uint64)
    pos = pos[pos <= 0x43F00000].astype(np.uint32)
    bits = np.concatenate([pos, pos | np.uint32(0x80000000)])
    x = torch.from_numpy(bits.view(np.float32).copy())
    codes = x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    back = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    return {"bits": bits, "codes": codes, "decode_all": back}


def e4m3_exhaustive_check():
    """Full sweep (not stored): oracle encoder == torch on every float32 in range."""
    from oracle.grid import e4m3_encode

    total = 0
    for lo in range(0, 0x43F00001, 1 << 25):
        hi = min(lo + (1 << 25), 0x43F00001)
        bits = np.arange(lo, hi, dtype=np.uint32)
        for sgn in (0, 0x80000000):
            b = bits | np.uint32(sgn)
            x = b.view(np.float32)
            ref = torch.from_numpy(x.copy()).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
            mine = e4m3_encode(x)
            bad = np.nonzero(ref != mine)[0]
            if len(bad):
                raise SystemExit(f"e4m3 mismatch at bits 0x{int(b[bad[0]]):08X}: "
                                 f"torch {ref[bad[0]]:#x} oracle {mine[bad[0]]:#x}")
            total += len(b)
    print(f"e4m3: oracle encoder == torch on all {total} float32 in [-480, 480]")


def pack_cases(packing, artifacts):
    rng = np.random.default_rng(5)
    out = {}
    for bits in (2, 4, 8):
        q = rng.integers(0, 2**bits, (3, 8, 64)).astype(np.uint8)
        out[f"q{bits}"] = q
        out[f"w{bits}"] = packing.pack_q(q, bits)
    q = rng.integers(0, 16, (5, 64)).astype(np.uint8)
    out["qn"] = q
    out["nib"] = artifacts.pack_nibbles(torch.from_numpy(q)).numpy()
    return out


def _correlated_H(B, C, N, seed, scale_items=True):
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(N, C, generator=g)
    X = base + 0.5 * torch.roll(base, 1, dims=1)
    X[:, 5] *= 20.0
    H = (X.T @ X).unsqueeze(0).repeat(B, 1, 1).contiguous()
    if scale_items and B > 1:
        H[1] *= 3.0
    return H


def solve_cases(gptq):
    out = {}
    cases = [
        ("affine4_g64", dict(bits=4, group_size=64, mode="affine"), 2, 48, 256, 0),
        ("affine2_g32", dict(bits=2, group_size=32, mode="affine"), 1, 32, 128, 1),
        ("affine8_g128", dict(bits=8, group_size=128, mode="affine"), 1, 32, 256, 2),
        ("affine4_g64_minmax_f16", dict(bits=4, group_size=64, mode="affine", clip="minmax",
                                        storage_dtype=torch.float16), 1, 32, 128, 3),
        ("mxfp4_safe", dict(bits=4, group_size=32, mode="mxfp4"), 2, 48, 128, 4),
        ("mxfp4_groupwise", dict(bits=4, group_size=32, mode="mxfp4",
                                 mxfp_algorithm="groupwise"), 2, 48, 128, 5),
        ("mxfp8_groupwise", dict(bits=8, group_size=32, mode="mxfp8"), 2, 48, 128, 6),
        ("mxfp8_safe", dict(bits=8, group_size=32, mode="mxfp8",
                            mxfp_algorithm="safe-scale-search"), 1, 48, 128, 7),
    ]
    for name, kw, B, R, C, seed in cases:
        g = torch.Generator().manual_seed(1000 + seed)
        W = torch.randn(B, R, C, generator=g) * 0.05
        H = _correlated_H(B, C, 2 * C, seed)
        if name == "affine4_g64":
            H[0, 7, :] = 0.0  # dead column 7 in item 0
            H[0, :, 7] = 0.0
        Hin = H.clone()
        q, s, b, Wdq, rel = gptq.solve_gptq(W.clone(), H, **kw)
        out[f"{name}/W"] = _f32(W)
        out[f"{name}/H"] = _f32(Hin)
        out[f"{name}/H_after"] = _f32(H)
        out[f"{name}/q"] = _u8(q)
        out[f"{name}/s"] = _f32(s) if s.dtype != torch.uint8 else _u8(s)
        if b is not None:
            out[f"{name}/b"] = _f32(b)
        out[f"{name}/Wdq"] = _f32(Wdq)
        out[f"{name}/rel"] = _f32(rel)
    # zero Hessian (unrouted expert) and a bad, indefinite diagonal (range guard)
    g = torch.Generator().manual_seed(19)
    W = torch.randn(1, 32, 128, generator=g) * 0.02
    H = torch.zeros(1, 128, 128)
    H[0, torch.arange(128), torch.arange(128)] = torch.linspace(-1.0, 1.0, 128)
    Hin = H.clone()
    q, s, b, Wdq, rel = gptq.solve_gptq(W.clone(), H, bits=4, group_size=32, mode="mxfp4",
                                        mxfp_algorithm="safe-scale-search")
    out["mxfp4_bad/W"], out["mxfp4_bad/H"], out["mxfp4_bad/H_after"] = _f32(W), _f32(Hin), _f32(H)
    out["mxfp4_bad/q"], out["mxfp4_bad/s"], out["mxfp4_bad/Wdq"] = _u8(q), _u8(s), _f32(Wdq)
    out["mxfp4_bad/rel"] = _f32(rel)
    W = torch.randn(1, 8, 64, generator=g)
    H = torch.zeros(1, 64, 64)
    q, s, b, Wdq, rel = gptq.solve_gptq(W.clone(), H.clone(), bits=4, group_size=32)
    out["affine_zeroH/W"], out["affine_zeroH/H"] = _f32(W), _f32(H)
    out["affine_zeroH/q"], out["affine_zeroH/s"], out["affine_zeroH/b"] = _u8(q), _f32(s), _f32(b)
    out["affine_zeroH/Wdq"], out["affine_zeroH/rel"] = _f32(Wdq), _f32(rel)
    return out


def hinv_cases(gptq):
    out = {}
    H = _correlated_H(3, 64, 256, 9)
    H[2] = -H[2] * 0.0 + torch.diag(torch.linspace(-0.02, 1.0, 64))  # escalation case
    U = gptq._prepare_hinv(H.clone(), 0.01)
    out["H"], out["U"] = _f32(H), _f32(U)
    Hg = _correlated_H(4, 32, 128, 10)
    out["Hg"], out["Ug"] = _f32(Hg), _f32(gptq._prepare_hinv(Hg.clone(), 0.01))
    return out


def hessian_cases(capture):
    out = {}
    g = torch.Generator().manual_seed(1)
    X = torch.randn(3000, 96, generator=g).to(torch.bfloat16)
    X[:, 3] *= 20
    st = capture.Stash("x", 96)
    st.add(X[:1000])
    st.add(X[1000:])
    H = st.hessian("cpu", chunk_rows=512)
    out["X_bits"] = X.view(torch.int16).numpy().view(np.uint16)
    out["H"] = _f32(H)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GQ_REFERENCE"),
                    help="reference checkout (or set GQ_REFERENCE)")
    ap.add_argument("--skip-exhaustive", action="store_true")
    args = ap.parse_args()
    if not args.ref:
        ap.error("--ref (or GQ_REFERENCE) must point at the reference checkout")
    sys.path.insert(0, os.path.join(HERE, "..", ".."))
    sys.path.insert(0, args.ref)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from mlx_gptq import artifacts, capture, gptq, grid, packing

    np.savez_compressed(os.path.join(HERE, "rtn_affine.npz"), **rtn_affine_cases(grid))
    np.savez_compressed(os.path.join(HERE, "rtn_mxfp.npz"), **rtn_mxfp_cases(grid))
    np.savez_compressed(os.path.join(HERE, "e4m3.npz"), **e4m3_cases())
    np.savez_compressed(os.path.join(HERE, "pack.npz"), **pack_cases(packing, artifacts))
    np.savez_compressed(os.path.join(HERE, "solve.npz"), **solve_cases(gptq))
    np.savez_compressed(os.path.join(HERE, "hinv.npz"), **hinv_cases(gptq))
    np.savez_compressed(os.path.join(HERE, "hessian.npz"), **hessian_cases(capture))
    if not args.skip_exhaustive:
        e4m3_exhaustive_check()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
