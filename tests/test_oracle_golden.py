"""Pin the numpy oracle to golden vectors produced by the real reference.

CPU only. These tests are what make the oracle trustworthy as the checker for
the CUDA path: RTN grids, E8M0 exponents, E4M3 codes and packing must be
bit-exact; the GPTQ solver (LAPACK rounding differs from torch's) must agree
on >= 99.9% of codes and on the proxy loss within 0.5%.
"""

import numpy as np
import pytest

from oracle import gptq, grid, hessian, packing

CODE_AGREEMENT = 0.999  # fraction of identical codes required (GPTQ solves)
PROXY_RTOL = 0.005  # relative tolerance on tr((W-Q) H (W-Q)^T)


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("method", ["mse", "minmax"])
@pytest.mark.parametrize("st", ["bfloat16", "float16", "float32"])
def test_rtn_affine_bit_exact(golden, bits, gs, method, st):
    g = golden("rtn_affine")
    k = f"{bits}_{gs}_{method}_{st}"
    q, s, b, dq = grid.rtn_quantize(g["W"], bits, gs, method, st)
    np.testing.assert_array_equal(q, g[f"q_{k}"])
    np.testing.assert_array_equal(s, g[f"s_{k}"])
    np.testing.assert_array_equal(b, g[f"b_{k}"])
    np.testing.assert_array_equal(dq, g[f"dq_{k}"])


@pytest.mark.parametrize("mode", ["mxfp4", "mxfp8"])
@pytest.mark.parametrize("which", ["", "b"])
def test_rtn_mxfp_bit_exact(golden, mode, which):
    g = golden("rtn_mxfp")
    W = g[f"W{which}_{mode}"]
    q, s, b, dq = grid.rtn_quantize_mxfp(W, mode)
    assert b is None
    np.testing.assert_array_equal(s, g[f"s{which}_{mode}"])
    np.testing.assert_array_equal(q, g[f"q{which}_{mode}"])
    np.testing.assert_array_equal(dq.view(np.uint32), g[f"dq{which}_{mode}"].view(np.uint32))


def test_e4m3_encode_decode(golden):
    g = golden("e4m3")
    x = g["bits"].view(np.float32)
    codes = grid.e4m3_encode(np.clip(x, -448.0, 448.0))
    np.testing.assert_array_equal(codes, g["codes"])
    dec = grid.e4m3_decode(np.arange(256, dtype=np.uint8))
    ref = g["decode_all"]
    assert np.array_equal(np.isnan(dec), np.isnan(ref))
    ok = ~np.isnan(ref)
    np.testing.assert_array_equal(dec[ok].view(np.uint32), ref[ok].view(np.uint32))


def test_exponent_table_is_a_clean_step():
    from oracle.log2_table import THRESHOLDS

    T = np.array(THRESHOLDS, np.int64)
    E = np.arange(-127, 128)
    lo = np.where(E >= -126, (E + 127) << 23, 1 << (E + 149).clip(0))
    assert np.all(T > lo) and np.all(T < lo * 2 + (E >= -126) * (1 << 23))


def test_pack_bit_exact(golden):
    g = golden("pack")
    for bits in (2, 4, 8):
        w = packing.pack_q(g[f"q{bits}"], bits)
        np.testing.assert_array_equal(w, g[f"w{bits}"])
        np.testing.assert_array_equal(packing.unpack_q(w, bits, 64), g[f"q{bits}"])
    n = packing.pack_nibbles(g["qn"])
    np.testing.assert_array_equal(n, g["nib"])
    np.testing.assert_array_equal(packing.unpack_nibbles(n), g["qn"])
    # 4-bit nibble bytes read as little-endian uint32 are the MLX words
    np.testing.assert_array_equal(
        packing.pack_nibbles(g["q4"]).view("<u4"), packing.pack_q(g["q4"], 4))


def test_pack_rejects_bad_bits():
    with pytest.raises(ValueError):
        packing.pack_q(np.zeros((2, 32), np.uint8), 3)


def test_hessian_matches_reference(golden):
    g = golden("hessian")
    X = hessian.bf16_bits_to_f32(g["X_bits"])
    H = hessian.hessian(X, chunk_rows=512)
    ref = g["H"]
    rel = np.linalg.norm(H - ref) / np.linalg.norm(ref)
    assert rel < 1e-5, rel


def test_prepare_hinv_matches_reference(golden):
    g = golden("hinv")
    for hk, uk in (("H", "U"), ("Hg", "Ug")):
        U, damp = gptq.prepare_hinv(g[hk].copy(), 0.01)
        ref = g[uk]
        rel = np.linalg.norm(U - ref, axis=(1, 2)) / np.linalg.norm(ref, axis=(1, 2))
        assert (rel < 1e-4).all(), rel
    _, damp = gptq.prepare_hinv(g["H"].copy(), 0.01)
    assert damp[2] > 0.01  # the indefinite item escalated


SOLVE_CASES = {
    "affine4_g64": dict(bits=4, group_size=64, mode="affine"),
    "affine2_g32": dict(bits=2, group_size=32, mode="affine"),
    "affine8_g128": dict(bits=8, group_size=128, mode="affine"),
    "affine4_g64_minmax_f16": dict(bits=4, group_size=64, mode="affine", clip="minmax",
                                   storage="float16"),
    "mxfp4_safe": dict(bits=4, group_size=32, mode="mxfp4"),
    "mxfp4_groupwise": dict(bits=4, group_size=32, mode="mxfp4", mxfp_algorithm="groupwise"),
    "mxfp8_groupwise": dict(bits=8, group_size=32, mode="mxfp8"),
    "mxfp8_safe": dict(bits=8, group_size=32, mode="mxfp8", mxfp_algorithm="safe-scale-search"),
    "mxfp4_bad": dict(bits=4, group_size=32, mode="mxfp4", mxfp_algorithm="safe-scale-search"),
}


@pytest.mark.parametrize("name", sorted(SOLVE_CASES))
def test_solve_gptq_matches_reference(golden, name):
    g = golden("solve")
    W = g[f"{name}/W"]
    H = g[f"{name}/H"].copy()
    q, s, b, Wdq, rel = gptq.solve_gptq(W, H, **SOLVE_CASES[name])
    np.testing.assert_array_equal(H, g[f"{name}/H_after"])  # dead-column mutation
    agree = (q == g[f"{name}/q"]).mean()
    assert agree >= CODE_AGREEMENT, agree
    H0 = g[f"{name}/H_after"]
    ours = gptq.proxy_loss(W, Wdq, H0)
    ref = gptq.proxy_loss(W, g[f"{name}/Wdq"], H0)
    np.testing.assert_allclose(ours, ref, rtol=PROXY_RTOL)
    np.testing.assert_allclose(rel, g[f"{name}/rel"], rtol=1e-3)


def test_zero_hessian_affine(golden):
    g = golden("solve")
    q, s, b, Wdq, rel = gptq.solve_gptq(g["affine_zeroH/W"], g["affine_zeroH/H"].copy(),
                                        bits=4, group_size=32)
    assert np.isfinite(Wdq).all()
    np.testing.assert_array_equal(q, g["affine_zeroH/q"])
    np.testing.assert_array_equal(Wdq, g["affine_zeroH/Wdq"])


def test_mxfp_range_guard(golden):
    g = golden("solve")
    W = g["mxfp4_bad/W"]
    _, s, _, Wdq, _ = gptq.solve_gptq(W, g["mxfp4_bad/H"].copy(), bits=4, group_size=32,
                                      mode="mxfp4", mxfp_algorithm="safe-scale-search")
    assert np.isfinite(Wdq).all()
    assert np.abs(Wdq).max() <= np.abs(W).max() * 32.0
    assert int(s.max()) < 250


def test_block_diagonal_padding_keeps_the_factor():
    """The identity behind padding the affine factor to 64-column blocks: H embedded
    block-diagonally with mean(diag H) on the extra diagonal has the same damping and
    an inverse factor whose leading C x C block is U (gptq.py:27-66 restated)."""
    from oracle.gptq import prepare_hinv

    rng = np.random.default_rng(5)
    C, Cp = 96, 128
    X = rng.standard_normal((512, C)).astype(np.float32)
    H = (X.T @ X)[None].astype(np.float32)
    U, *_ = prepare_hinv(H.copy(), 0.01)
    Hp = np.zeros((1, Cp, Cp), np.float32)
    Hp[0, :C, :C] = H[0]
    Hp[0, np.arange(C, Cp), np.arange(C, Cp)] = np.diagonal(H[0]).mean()
    Up, *_ = prepare_hinv(Hp, 0.01)
    np.testing.assert_allclose(Up[0, :C, :C], U[0], rtol=2e-4, atol=1e-6)
    assert np.abs(Up[0, :C, C:]).max() == 0.0
