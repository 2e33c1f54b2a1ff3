"""The affine solver's float32 GEMM (trailing update W[:, i2:] -= Err U[i1:i2, i2:],
reference mlx_gptq/gptq.py:269-270, and the factor's products, gptq.py:27-66) through
the C ABI, on both engines: the TMA-fed tcgen05 kernel and the mma.sync kernels.

Both are 3xTF32 (x = hi + lo, hi*hi + hi*lo + lo*hi), so against a float64 product
the error stays at float32 level: max |C - C64| <= 2e-6 * (|alpha| sum_t |a||b| + |beta C|),
the bound written below per element.
"""

import ctypes

import pytest
import torch

from mlx_gptq_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL = 2e-6


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _op(X, trans):
    return X.transpose(-1, -2) if trans else X


def _run(engine, A, B, C, M, N, K, ta, tb, n_inner, n_outer, alpha, beta, skip=None):
    """A: [outer, inner, rows, lda] style tensors, contiguous; returns status."""
    lda, ldb, ldc = A.shape[-1], B.shape[-1], C.shape[-1]
    sa_i, sb_i, sc_i = A[0, 0].numel(), B[0, 0].numel(), C[0, 0].numel()
    sa_o, sb_o, sc_o = sa_i * n_inner, sb_i * n_inner, sc_i * n_inner
    st = _lib.lib().gq_gemm_f32(_ptr(A), _ptr(B), _ptr(C), M, N, K, lda, ldb, ldc, int(ta), int(tb),
                                n_inner * n_outer, n_inner, sa_o, sa_i, sb_o, sb_i, sc_o, sc_i, alpha, beta,
                                _ptr(skip), engine, None, None)
    torch.cuda.synchronize()
    return st


def _case(M, N, K, ta, tb, n_inner=1, n_outer=1, alpha=-1.0, beta=1.0, pad=4, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    # leading dimensions padded past the logical sizes: the kernels must respect them
    a_rows, a_cols = (K, M) if ta else (M, K)
    b_rows, b_cols = (N, K) if tb else (K, N)
    ld = lambda cols: (cols + 3) // 4 * 4 + pad  # multiples of 4 floats: 16-byte rows for the tensor maps
    A = torch.randn(n_outer, n_inner, a_rows, ld(a_cols), device="cuda", generator=g)
    B = torch.randn(n_outer, n_inner, b_rows, ld(b_cols), device="cuda", generator=g)
    C0 = torch.randn(n_outer, n_inner, M, ld(N), device="cuda", generator=g)
    Al = A[..., :a_cols].double()
    Bl = B[..., :b_cols].double()
    prod = _op(Al, ta) @ _op(Bl, tb)
    ref = C0.double().clone()
    ref[..., :N] = beta * ref[..., :N] + alpha * prod
    bound = RTOL * (abs(alpha) * (_op(Al.abs(), ta) @ _op(Bl.abs(), tb)) + abs(beta) * C0[..., :N].double().abs())
    return A, B, C0, ref, bound


@pytest.mark.parametrize("engine", [1, 0], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, True), (False, True), (True, False)])
@pytest.mark.parametrize("M,N,K", [(200, 300, 100), (256, 384, 128), (129, 131, 37)])
def test_gemm_matches_float64(engine, ta, tb, M, N, K):
    A, B, C, ref, bound = _case(M, N, K, ta, tb)
    assert _run(engine, A, B, C, M, N, K, ta, tb, 1, 1, -1.0, 1.0) == _lib.GQ_OK, _lib.lib().gq_last_error()
    err = (C.double()[..., :N] - ref[..., :N]).abs()
    assert bool((err <= bound[..., :N] + 1e-30).all()), float((err / (bound[..., :N] + 1e-30)).max())
    assert torch.equal(C[..., N:], ref[..., N:].float())  # padding columns untouched


@pytest.mark.parametrize("engine", [1, 0], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("beta", [0.0, 0.5, 1.0])  # TMA store, read-modify-write, TMA reduce-add
def test_gemm_batches_skip_and_beta(engine, beta):
    M, N, K, ni, no = 160, 144, 96, 3, 2
    A, B, C, ref, bound = _case(M, N, K, True, True, ni, no, alpha=0.5, beta=beta, seed=1)
    skip = torch.tensor([0, 1], dtype=torch.int32, device="cuda")  # outer item 1 is left alone
    C_before = C.clone()
    assert _run(engine, A, B, C, M, N, K, True, True, ni, no, 0.5, beta, skip) == _lib.GQ_OK
    err = (C[0].double()[..., :N] - ref[0, ..., :N]).abs()
    assert bool((err <= bound[0, ..., :N] + 1e-30).all())
    assert torch.equal(C[1], C_before[1])


def test_gemm_trailing_update_shape_engines_agree():
    """The affine trailing update's own shape (K = block size 128, N = C - i2), both
    engines within the float32 bound of each other's float64 reference."""
    M, N, K = 1024, 1920, 128
    A, B, C, ref, bound = _case(M, N, K, False, False, pad=0, seed=2)
    C1 = C.clone()
    assert _run(1, A, B, C1, M, N, K, False, False, 1, 1, -1.0, 1.0) == _lib.GQ_OK
    C0 = C.clone()
    assert _run(0, A, B, C0, M, N, K, False, False, 1, 1, -1.0, 1.0) == _lib.GQ_OK
    for out in (C0, C1):
        assert bool(((out.double() - ref).abs() <= bound + 1e-30).all())


def test_gemm_rejects_unaligned_tensor_core_operands():
    A = torch.randn(1, 1, 64, 65, device="cuda")
    B = torch.randn(1, 1, 65, 64, device="cuda")
    C = torch.zeros(1, 1, 64, 64, device="cuda")
    st = _run(1, A, B, C, 64, 64, 65, False, False, 1, 1, 1.0, 0.0)  # lda = 65 is not a multiple of 4
    assert st == _lib.GQ_ERR_ARG
