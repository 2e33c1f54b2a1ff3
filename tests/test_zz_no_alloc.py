"""gq_gptq_mxfp_noalloc: the MXFP GPTQ entry point that allocates nothing.

Some callers cannot allocate device memory themselves: a host that owns every
byte through its own pool, a loop that must not allocate while it runs, or a
foreign-language binding that is handed only the tensors to read and write.
For them the library offers a variant of gq_gptq_mxfp whose rel_err scratch is
a fixed array inside the library instead of a caller workspace. This test calls
it through the C ABI, twice in a row on different inputs, and compares every
output with the workspace-taking entry point on the same inputs (it must be
bit-identical: same kernels, same reduction order). It also checks that a
problem larger than the fixed scratch is refused with an argument error.

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
        for a, b in zip(ref[:4], got[:4]):
            assert torch.equal(a, b)
        torch.testing.assert_close(got[4], ref[4], rtol=1e-6, atol=0.0)
        assert torch.isfinite(got[4]).all() and (got[4] > 0).all()


def test_noalloc_rejects_problems_beyond_its_scratch():
    from mlx_gptq_b200 import _lib as L

    lib = L.lib()
    p = ctypes.c_void_p(256)
    # 128 * ceil(4096/128) * (8192/32) = 1,048,576 (tile, group) pairs > 524,288
    st = lib.gq_gptq_mxfp_noalloc(p, L.GQ_F32, p, p, None, None, 128, 4096, 8192, L.GQ_MXFP4,
                                  L.GQ_MX_SAFE_SCALE_SEARCH, None, None, p, None, L.GQ_F32, p, None)
    assert st == L.GQ_ERR_ARG
    assert b"fixed scratch" in lib.gq_last_error()
