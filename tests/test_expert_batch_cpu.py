"""Host-side logic of the sharded expert batch (mlx_gptq_b200.expert_batch), on CPU:
the LPT expert split, the piece layout of a skewed routing, and the exchange's
all-gather into expert order across two gloo ranks."""

import os

import pytest
import torch


def test_plan_experts_balances_a_skewed_batch():
    from mlx_gptq_b200.expert_batch import SOLVE_UNITS_PER_ELEM, plan_experts

    counts = [500_000] * 8 + [100] * 112 + [0] * 8
    shares = plan_experts(counts, 8, (2048, 768), 4_718_592)
    assert sorted(e for s in shares for e in s) == list(range(128))
    per_tok = 2048 ** 2 + 768 ** 2
    loads = [sum(counts[e] * per_tok + SOLVE_UNITS_PER_ELEM * 4_718_592 for e in s) for s in shares]
    assert max(loads) <= 1.05 * (sum(loads) / 8)
    assert all(sum(1 for e in s if counts[e] == 500_000) == 1 for s in shares)  # one heavy expert each


def test_plan_experts_charges_experts_without_tokens():
    """An expert without tokens costs its RTN fallback, so the rank that takes it gets
    fewer routed tokens than a rank without one."""
    from mlx_gptq_b200.expert_batch import RTN_FALLBACK_UNITS, SOLVE_UNITS_PER_ELEM, plan_experts

    counts = [30_000] * 8 + [0]
    shares = plan_experts(counts, 3, (2048, 768), 4_718_592)
    per_token = 2048 ** 2 + 768 ** 2
    cost = lambda sh: sum(counts[e] * per_token + SOLVE_UNITS_PER_ELEM * 4_718_592 +
                          (RTN_FALLBACK_UNITS if counts[e] == 0 else 0) for e in sh)
    holder = next(sh for sh in shares if 8 in sh)
    assert sorted(e for sh in shares for e in sh) == list(range(9))
    assert max(map(cost, shares)) - min(map(cost, shares)) <= cost([0])  # LPT: within one item
    assert sum(counts[e] for e in holder) <= min(sum(counts[e] for e in sh) for sh in shares if 8 not in sh)


def test_piece_layout_cuts_heavy_experts_and_keeps_rows():
    from mlx_gptq_b200.expert_batch import piece_layout

    counts = [4000, 64, 0, 900]
    offsets = torch.zeros(5, dtype=torch.int64)
    offsets[1:] = torch.cumsum(torch.tensor(counts), 0)
    tok = torch.randperm(sum(counts)).to(torch.int32)
    lay = piece_layout(tok, offsets, [0, 1, 2, 3], 2048, "cpu", waves=1.0, tiles_per_wave=74)
    n = lay.offsets.numel() - 1
    assert lay.n == 4 and n == 4 + len(lay.extra)
    assert int(lay.offsets[-1]) == sum(counts)
    # every expert's rows appear exactly once across its pieces
    pieces = {i: [lay.token_idx[int(lay.offsets[i]):int(lay.offsets[i + 1])]] for i in range(4)}
    for j, (i, _) in enumerate(lay.extra):
        pieces[i].append(lay.token_idx[int(lay.offsets[4 + j]):int(lay.offsets[5 + j])])
    for i, c in enumerate(counts):
        got = torch.cat(pieces[i]).sort().values
        want = tok[int(offsets[i]):int(offsets[i + 1])].sort().values
        assert torch.equal(got, want)
    assert any(i == 0 for i, _ in lay.extra)  # the heavy expert is cut
    assert torch.equal(tok.index_select(0, lay.perm), lay.token_idx)


def _exchange_rank(rank, world, port, out):
    import torch.distributed as dist

    from mlx_gptq_b200.expert_batch import Exchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shares = [[0, 3, 4], [1, 2]]
    ex = Exchange(shares, rank, dist.group.WORLD, "cpu")
    assert not ex.push  # host tensors: the all_gather form
    mine = torch.tensor([[e * 10, e * 10 + 1] for e in shares[rank]], dtype=torch.int32)
    full = ex.buffer((2,), torch.int32)
    assert full.shape == (6, 2)  # rank-major, 3 slots per rank
    ex.start(mine, full)
    ex.wait()
    assert [ex.slot_of[e] for e in range(5)] == [0, 3, 4, 1, 2]
    out[rank] = ex.expert_order(full).tolist()
    dist.destroy_process_group()


def test_exchange_gathers_every_expert_to_every_rank():
    import torch.multiprocessing as mp

    port = 29500 + os.getpid() % 1000
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_exchange_rank, args=(2, port, out), nprocs=2, join=True)
        want = [[e * 10, e * 10 + 1] for e in range(5)]
        assert out[0] == want and out[1] == want


def test_span_layout_covers_each_expert_once():
    from mlx_gptq_b200.expert_batch import piece_layout

    counts = [5000, 10, 0, 700, 64]
    offsets = torch.zeros(6, dtype=torch.int64)
    offsets[1:] = torch.cumsum(torch.tensor(counts), 0)
    lay = piece_layout(None, offsets, [0, 1, 2, 3, 4], 768, "cpu", waves=1.0, tiles_per_wave=74)
    assert lay.token_idx is None and lay.spans is not None and len(lay.spans) == 5 + len(lay.extra)
    rows = {i: [lay.spans[i]] for i in range(5)}
    for j, (i, _) in enumerate(lay.extra):
        rows[i].append(lay.spans[5 + j])
    for i, c in enumerate(counts):
        covered = sorted(r for a, k in rows[i] for r in range(a, a + k))
        assert covered == list(range(int(offsets[i]), int(offsets[i]) + c))


def test_merge_plan_groups_pieces_by_expert_in_order():
    """The merge plan handed to gq_hessian_merge_pieces: one target per expert with extra
    pieces, its pieces in piece order, CSR pointers consistent; None without pieces."""
    from mlx_gptq_b200.expert_batch import PieceLayout

    lay = PieceLayout(n=4, extra=[(0, 1), (2, 1), (0, 2), (0, 3), (2, 2)], offsets=torch.zeros(10, dtype=torch.int64))
    t, ptr, pieces = lay.merge_plan("cpu")
    assert t.tolist() == [0, 2]
    assert ptr.tolist() == [0, 3, 5]
    assert pieces.tolist() == [4, 6, 7, 5, 8]  # expert 0: pieces 4, 6, 7; expert 2: pieces 5, 8
    assert lay.merge_plan("cpu") is lay.merge  # built once
    assert PieceLayout(n=2, extra=[], offsets=torch.zeros(3, dtype=torch.int64)).merge_plan("cpu") is None
