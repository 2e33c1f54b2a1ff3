"""The expert exchange between GPU ranks (one process per GPU, NCCL), both forms: the
copy-engine pushes into symmetric buffers and the all_gather fallback. Every rank must
end with every expert's slab, three rounds in a row on the same buffers, and the two
forms must agree. Needs two CUDA devices; skipped otherwise. The ranks are child
processes; a rank that fails raises on the host and the process-group timeout (60 s)
ends the others' collectives."""

import os

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two CUDA devices")]


def _rank(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    from mlx_gptq_b200.expert_batch import Exchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        E = 11
        shares = [[e for e in range(E) if e % world == r] for r in range(world)]
        got = {}
        for push in (True, False):
            ex = Exchange(shares, rank, dist.group.WORLD, dev, push=push)
            out = ex.buffer((257, 33), torch.uint8)
            for it in range(3):
                mine = torch.stack([torch.full((257, 33), (e * 7 + it) % 251, dtype=torch.uint8, device=dev)
                                    for e in shares[rank]])
                ex.start(mine, out)
                ex.wait()
                full = ex.expert_order(out)
                want = torch.stack([torch.full((257, 33), (e * 7 + it) % 251, dtype=torch.uint8, device=dev)
                                    for e in range(E)])
                assert torch.equal(full, want), (push, it)
            got[push] = full.cpu()
        assert torch.equal(got[True], got[False])
        results[rank] = "ok"
    finally:
        dist.destroy_process_group()


def test_exchange_push_and_all_gather_on_two_ranks():
    import torch.multiprocessing as mp

    port = 29700 + os.getpid() % 200
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_rank, args=(2, port, results), nprocs=2, join=True)
        assert dict(results) == {0: "ok", 1: "ok"}
