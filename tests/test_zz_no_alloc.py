"""gq_gptq_mxfp_noalloc: the MXFP GPTQ entry point that allocates nothing.

Some callers cannot allocate device memory themselves: a host that owns every
byte through its own pool, a loop that must not allocate while it runs, or a
foreign-language binding that is handed only the tensors to read and write.
For them the library offers a variant of gq_gptq_mxfp whose rel_err scratch is
a fixed array inside the library instead of a caller workspace. These tests
call it through the C ABI:

* twice in a row on different inputs, comparing every output, rel_err included,
  with the workspace-taking entry point on the same inputs: they must be
  bit-identical (same kernels, same reduction order), and the second call must
  not see the first call's scratch;
* on a problem larger than the fixed scratch: refused with an argument error when
  rel_err is asked for, accepted (and equal to the workspace entry point) when it
  is not, since the column loop then needs no scratch.

Every pointer handed to the library is a real device buffer of the size the
call describes, so even a regression in the size check could not make a kernel
read or write outside memory this test owns.

The file is named so that pytest collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(seed, B=2, R=300, C=512, N=2048):
    rng = np.random.default_rng(seed)
    base = rng.standard_normal((N, C)).astype(np.float32)
    X = base + 0.5 * np.roll(base, 1, axis=1)
    X[:, 7] *= 25.0
    H = np.repeat((X.T @ X)[None], B, axis=0).astype(np.float32)
    H[1:] *= 1.5
    W = (rng.standard_normal((B, R, C)) * 0.02).astype(np.float32)
    return torch.from_numpy(W).cuda(), torch.from_numpy(H).cuda()


def _solve(lib, L, W, f, noalloc):
    B, R, C = W.shape
    q = torch.empty(B, R, C, dtype=torch.uint8, device="cuda")
    qp = torch.empty(B, R, C // 2, dtype=torch.uint8, device="cuda")
    s = torch.empty(B, R, C // 32, dtype=torch.uint8, device="cuda")
    wdq = torch.empty(B, R, C, dtype=torch.float32, device="cuda")
    rel = torch.empty(B, dtype=torch.float32, device="cuda")
    args = [W.data_ptr(), L.GQ_F32, f.H.data_ptr(), f.U.data_ptr(), f.dead.data_ptr(), f.info.data_ptr(),
            B, R, C, L.GQ_MXFP4, L.GQ_MX_SAFE_SCALE_SEARCH, q.data_ptr(), qp.data_ptr(), s.data_ptr(),
            wdq.data_ptr(), L.GQ_F32, rel.data_ptr()]
    if noalloc:
        st = lib.gq_gptq_mxfp_noalloc(*args, L.stream_ptr())
    else:
        ws = torch.empty(lib.gq_gptq_mxfp_workspace_size(B, R, C), dtype=torch.uint8, device="cuda")
        st = lib.gq_gptq_mxfp(*args, ws.data_ptr(), ws.numel(), L.stream_ptr())
    L.check(st, "noalloc test solve")
    torch.cuda.synchronize()
    return q, qp, s, wdq, rel


def test_noalloc_matches_workspace_entry_point_two_calls():
    from mlx_gptq_b200 import _lib as L
    from mlx_gptq_b200.layer import mxfp_factors

    lib = L.lib()
    for seed in (1, 2):  # two calls in a row: the second must not see the first's scratch
        W, H = _problem(seed, R=300 if seed == 1 else 200)
        f = mxfp_factors(H)
        ref = _solve(lib, L, W, f, noalloc=False)
        got = _solve(lib, L, W, f, noalloc=True)
        for a, b in zip(ref, got):
            assert torch.equal(a, b)
        assert torch.isfinite(got[4]).all() and (got[4] > 0).all()


def _oversize():
    """A problem one row tile past the scratch limit, as real device buffers: B = 512,
    R = 131,200 (1,025 row tiles of 128), C = 32 gives 524,800 (tile, group) pairs
    against 524,288. W is bf16 (4.3 GB); H and U are per-item 32 x 32 blocks."""
    B, R, C = 512, 131200, 32
    g = torch.Generator(device="cuda").manual_seed(5)
    W = (torch.randn(B, R, C, generator=g, device="cuda", dtype=torch.float32) * 0.02).to(torch.bfloat16)
    A = torch.randn(B, C, 2 * C, generator=g, device="cuda")
    H = A @ A.transpose(1, 2)
    return W, H


def _run_oversize(lib, L, W, f, noalloc, with_rel):
    B, R, C = W.shape
    qp = torch.empty(B, R, C // 2, dtype=torch.uint8, device="cuda")
    s = torch.empty(B, R, C // 32, dtype=torch.uint8, device="cuda")
    rel = torch.empty(B, dtype=torch.float32, device="cuda") if with_rel else None
    args = [W.data_ptr(), L.GQ_BF16, f.H.data_ptr(), f.U.data_ptr(), f.dead.data_ptr(), f.info.data_ptr(),
            B, R, C, L.GQ_MXFP4, L.GQ_MX_SAFE_SCALE_SEARCH, None, qp.data_ptr(), s.data_ptr(), None, L.GQ_F32,
            None if rel is None else rel.data_ptr()]
    if noalloc:
        st = lib.gq_gptq_mxfp_noalloc(*args, L.stream_ptr())
    else:
        st = lib.gq_gptq_mxfp(*args, None, 0, L.stream_ptr())
    torch.cuda.synchronize()
    return st, qp, s


def test_noalloc_size_limit_applies_only_to_rel_err():
    from mlx_gptq_b200 import _lib as L
    from mlx_gptq_b200.layer import mxfp_factors

    lib = L.lib()
    W, H = _oversize()
    f = mxfp_factors(H)
    assert int(lib.gq_gptq_mxfp_workspace_size(*W.shape)) // 8 > 524288
    st, _, _ = _run_oversize(lib, L, W, f, noalloc=True, with_rel=True)
    assert st == L.GQ_ERR_ARG
    assert b"fixed scratch" in lib.gq_last_error()
    st, qp, s = _run_oversize(lib, L, W, f, noalloc=True, with_rel=False)
    L.check(st, "noalloc without rel_err")
    st, qp_ref, s_ref = _run_oversize(lib, L, W, f, noalloc=False, with_rel=False)
    L.check(st, "workspace entry point without rel_err")
    assert torch.equal(qp, qp_ref) and torch.equal(s, s_ref)
