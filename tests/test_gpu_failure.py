"""Failure detection on the GPU without a fault: a bounded wait that runs out.

The tcgen05 pipelines never spin forever: every mbarrier wait gives up after a
limit, raises the CTA's abort flag and records GQ_ERR_TIMEOUT in a device status
word the host reads. Here a self-test kernel waits, through the same routine, on a
barrier phase that nothing completes, with a 50 ms limit; the host must see the
timeout status and the context must stay usable afterwards.
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    from mlx_gptq_b200 import _lib as L
    from mlx_gptq_b200 import hessian_from_rows

    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    gave_up = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    L.check(L.lib().gq_selftest_wait_timeout(50_000_000, status.data_ptr(), gave_up.data_ptr(), L.stream_ptr()),
            "selftest")
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert int(gave_up.item()) == 1
    assert int(status.item()) == L.GQ_ERR_TIMEOUT
    assert 0.04 < elapsed < 5.0
    # the context is still usable: a normal kernel right after
    X = torch.randn(512, 64, device="cuda").to(torch.bfloat16)
    H = hessian_from_rows(X)
    assert torch.allclose(H.double(), X.double().T @ X.double(), rtol=1e-4, atol=1e-2)


def test_selftest_rejects_unbounded_limit():
    from mlx_gptq_b200 import _lib as L

    p = 16
    assert L.lib().gq_selftest_wait_timeout(10_000_000_000, p, p, None) == L.GQ_ERR_ARG


def test_hessian_path_raises_on_a_timed_out_status_word():
    """The Hessian wrappers pass the device's status word to every launch and the
    solver entry points read it: a word holding GQ_ERR_TIMEOUT (set here by the host,
    as a wait that gave up would) makes Stash.hessian and solve_gptq raise."""
    from mlx_gptq_b200 import _lib as L
    from mlx_gptq_b200 import Stash, solve_gptq

    st = Stash("probe", 64)
    st.add(torch.randn(256, 64, device="cuda").to(torch.bfloat16))
    word = L.status_word(torch.device("cuda", torch.cuda.current_device()))
    word.fill_(L.GQ_ERR_TIMEOUT)
    with pytest.raises(L.GQError):
        st.hessian("cuda")
    assert int(word.item()) == 0
    H = st.hessian("cuda")  # clear word: normal result
    word.fill_(L.GQ_ERR_TIMEOUT)
    with pytest.raises(L.GQError):
        solve_gptq(torch.randn(1, 8, 64, device="cuda") * 0.02, H.unsqueeze(0).clone(), 4, 32, mode="mxfp4")
    assert int(word.item()) == 0
