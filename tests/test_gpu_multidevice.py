"""Several devices in one process (needs 2 GPUs; skipped otherwise).

The reference calls solve_gptq concurrently from one Python thread per device
(sequential.py:625-626), so the C ABI must be re-entrant: per-call stream and device,
per-device state behind a mutex, no shared mutable globals. Two threads solve on two
devices at once, repeatedly, and every result must be bit-identical to the same solve
run alone; then the in-process expert spread (pipeline.solve_experts_on_devices) must
equal a one-device batch."""

import threading

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two CUDA devices")]


def _problem(seed, dev, mode):
    g = torch.Generator(device=dev).manual_seed(seed)
    X = (torch.randn(8192, 1024, generator=g, device=dev) * (1 + 9 * (torch.rand(1024, generator=g, device=dev) > 0.98)))
    from mlx_gptq_b200 import hessian_from_rows

    H = hessian_from_rows(X.to(torch.bfloat16)).unsqueeze(0).repeat(2, 1, 1)
    W = torch.randn(2, 384, 1024, generator=g, device=dev) * 0.02
    return W, H


@pytest.mark.parametrize("mode", ["mxfp4", "affine"])
def test_solve_gptq_concurrently_on_two_devices(mode):
    from mlx_gptq_b200 import solve_gptq

    bits, gs = (4, 32) if mode == "mxfp4" else (4, 64)
    devs = [torch.device("cuda", 0), torch.device("cuda", 1)]
    probs = {}
    for i, d in enumerate(devs):
        with torch.cuda.device(d):
            probs[i] = _problem(i + 3, d, mode)
    alone = {}
    for i, d in enumerate(devs):
        with torch.cuda.device(d):
            W, H = probs[i]
            alone[i] = solve_gptq(W, H.clone(), bits, gs, mode=mode)
            torch.cuda.synchronize(d)
    got, errors = {}, []

    def worker(i):
        try:
            with torch.cuda.device(devs[i]):
                W, H = probs[i]
                for r in range(4):
                    got[(i, r)] = solve_gptq(W, H.clone(), bits, gs, mode=mode)
                torch.cuda.synchronize(devs[i])
        except Exception as exc:  # reported below, on the main thread
            errors.append(exc)

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    for (i, r), out in got.items():
        for a, b in zip(out, alone[i]):
            if a is None:
                assert b is None
            else:
                assert a.device == devs[i] and torch.equal(a, b), (mode, i, r)


def test_expert_spread_over_two_devices_matches_one_device():
    """A fused task's experts split over cuda:0 and cuda:1 by worker threads equal the
    batch solved on cuda:0 alone (same Hessians, same kernels)."""
    from mlx_gptq_b200 import capture, pipeline

    dev0 = torch.device("cuda", 0)
    E, R, C = 6, 96, 256
    g = torch.Generator(device=dev0).manual_seed(11)
    param = torch.nn.Parameter((torch.randn(E, R, C, generator=g, device=dev0) * 0.02).to(torch.bfloat16))
    rows = [torch.randn(n, C, generator=g, device=dev0).to(torch.bfloat16) for n in (900, 40, 300, 0, 1200, 7)]

    class Mgr:
        def tokens(self, key):
            return rows[int(key)].shape[0]

        def expert_hessians(self, task, device, experts, timer=None):
            H = torch.zeros(len(experts), C, C, device=device)
            for j, e in enumerate(experts):
                if rows[e].shape[0]:
                    capture.hessian_accumulate(rows[e].to(device), H[j], 1.0, 0.0)
            return H

    task = capture.FusedExpertTask("mlp.experts", "down_proj", param, E, [str(e) for e in range(E)])
    args = pipeline.LayerSolveArgs(bits=4, group_size=32, mode="mxfp4", mxfp_algorithm="safe-scale-search")
    experts = list(range(E))
    one = pipeline.solve_experts_on_devices(Mgr(), task, experts, [dev0], 4, args)
    two = pipeline.solve_experts_on_devices(Mgr(), task, experts, [dev0, torch.device("cuda", 1)], 4, args)
    for a, b in zip(one, two):
        if a is None:
            assert b is None
        else:
            assert a.device == dev0 and b.device == dev0 and torch.equal(a, b)
