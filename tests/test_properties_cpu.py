"""Property tests (hypothesis) of the host-side scheduling and routing logic."""

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from mlx_gptq_b200.experts import _token_ranks, route
from mlx_gptq_b200.pipeline import _wave_parts, lpt_partition


@st.composite
def routings(draw):
    T = draw(st.integers(1, 40))
    E = draw(st.integers(1, 9))
    k = draw(st.integers(1, min(E, 4)))
    rows = []
    for _ in range(T):
        experts = draw(st.permutations(list(range(E))))[:k]
        # occasionally a dropped slot (index E), as capacity-limited routers emit
        rows.append([E if draw(st.integers(0, 9)) == 0 else e for e in experts])
    return torch.tensor(rows, dtype=torch.long), E


@settings(max_examples=200, deadline=None)
@given(routings())
def test_route_orders_slots_like_the_eager_loop(r):
    idx, E = r
    tok, pos, counts, counts_dev = route(idx, E)
    assert counts == counts_dev.tolist() == [int((idx == e).sum()) for e in range(E)]
    off = 0
    for e in range(E):  # eager: torch.where over the [top_k, tokens] mask of expert e
        j_ref, t_ref = torch.where((idx == e).T)
        assert torch.equal(tok[off:off + counts[e]], t_ref) and torch.equal(pos[off:off + counts[e]], j_ref)
        off += counts[e]
    assert off == tok.numel()
    # each token's slots ranked by ascending expert
    ranks = _token_ranks(tok, idx.shape[0])
    expert_of = torch.repeat_interleave(torch.arange(E), torch.tensor(counts))
    for t in range(idx.shape[0]):
        sel = (tok == t).nonzero().flatten()
        order = torch.argsort(expert_of[sel])
        assert torch.equal(ranks[sel][order], torch.arange(sel.numel()))


@settings(max_examples=200, deadline=None)
@given(st.lists(st.one_of(st.floats(0, 1e6, allow_nan=False), st.integers(0, 3).map(float)), max_size=60),
       st.integers(1, 9))
def test_lpt_partition_is_a_partition_within_the_lpt_bound(costs, parts):
    bins = lpt_partition(costs, parts)
    assert len(bins) == parts
    assert sorted(i for b in bins for i in b) == list(range(len(costs)))
    if costs:
        loads = [sum(costs[i] for i in b) for b in bins]
        # any list schedule (LPT included) ends by mean load + (1 - 1/m) * largest item
        bound = sum(costs) / parts + (1.0 - 1.0 / parts) * max(costs)
        assert max(loads) <= bound * (1 + 1e-9) + 1e-9
    assert lpt_partition(costs, parts) == bins  # deterministic


@settings(max_examples=300, deadline=None)
@given(st.integers(1, 5000), st.integers(1, 200), st.integers(1, 16))
def test_wave_parts_cover_the_tiles_in_at_most_one_wave_each(tiles, per_wave, world):
    parts = _wave_parts(tiles, per_wave, world)
    assert parts[0][0] == 0 and parts[-1][1] == tiles
    assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
    assert all(e > b for b, e in parts) and len(parts) <= world
    if world > 1 and -(-tiles // per_wave) <= world:
        assert all(e - b <= per_wave for b, e in parts)
    if world == 1:
        assert parts == [(0, tiles)]


@settings(max_examples=100, deadline=None)
@given(st.lists(st.tuples(st.integers(1, 12), st.integers(1, 3)), min_size=1, max_size=6),
       st.one_of(st.none(), st.integers(1, 30)), st.integers(1, 4))
def test_segment_store_equals_concatenation(batches, reserve, E):
    """Any sequence of batches, with or without a (possibly too small) reservation, leaves
    the store equal to the concatenation of what it was given."""
    from mlx_gptq_b200.capture import SegmentStore

    g = torch.Generator().manual_seed(len(batches) * 31 + E)
    st_ = SegmentStore(E, reserve)
    ins, acts, toks, counts_all = [], [], [], []
    base = 0
    for T, k in batches:
        hidden = torch.randn(T, 4, generator=g)
        e = torch.randint(0, E, (T * k,), generator=g)
        counts = torch.bincount(e, minlength=E).tolist()
        tok = torch.randint(0, T, (T * k,), generator=g)
        out = st_.acts_out(T * k, T, 3, torch.float32, "cpu")
        a = torch.randn(T * k, 3, generator=g)
        out.copy_(a)
        st_.add(hidden, tok, counts, out)
        ins.append(hidden)
        acts.append(a)
        toks.append(tok + base)
        counts_all.append(counts)
        base += T
    assert torch.equal(st_.inputs[:st_.n_tok], torch.cat(ins))
    assert torch.equal(st_.acts[:st_.n_slot], torch.cat(acts))
    assert torch.equal(st_.tok[:st_.n_slot].long(), torch.cat(toks))
    assert st_.counts == [sum(c[e] for c in counts_all) for e in range(E)]


@settings(max_examples=100, deadline=None)
@given(st.sampled_from([2, 4, 8]), st.integers(1, 5), st.integers(1, 6), st.integers(0, 2**31 - 1))
def test_oracle_packing_round_trip(bits, rows, words, seed):
    import numpy as np

    from oracle.packing import pack_q, unpack_q

    per = 32 // bits
    q = np.random.default_rng(seed).integers(0, 1 << bits, (rows, words * per)).astype(np.uint8)
    w = pack_q(q, bits)
    assert w.dtype == np.uint32 and w.shape == (rows, words)
    assert np.array_equal(unpack_q(w, bits, words * per), q)
    # LSB first: the first code sits in the lowest bits of the first word
    assert np.array_equal(w[:, 0] & ((1 << bits) - 1), q[:, 0].astype(np.uint32))


class _FakeMgr:
    """The parts of a CaptureManager that plan_layer reads."""

    def __init__(self, expert_tokens, linear_specs):
        import types

        self.stashes, self.fused_tasks, self.linear_tasks = {}, [], []
        for ti, (E, R, C, toks) in enumerate(expert_tokens):
            keys = []
            for e in range(E):
                k = f"m{ti}.p::e{e}"
                self.stashes[k] = types.SimpleNamespace(tokens=toks[e], in_features=C)
                keys.append(k)
            self.fused_tasks.append(types.SimpleNamespace(param=torch.empty(E, R, C, device="meta"),
                                                          stash_keys=keys, num_experts=E))
        for si, (C, toks, outs) in enumerate(linear_specs):
            key = f"lin{si}"
            self.stashes[key] = types.SimpleNamespace(tokens=toks, in_features=C)
            for j, R in enumerate(outs):
                self.linear_tasks.append(types.SimpleNamespace(
                    name=f"lin{si}_{j}", stash_key=key, module=types.SimpleNamespace(out_features=R)))

    def tokens(self, key):
        return self.stashes[key].tokens


@st.composite
def layers(draw):
    fused = []
    for _ in range(draw(st.integers(0, 2))):
        E = draw(st.integers(1, 12))
        fused.append((E, 64, draw(st.sampled_from([64, 128, 2048])),
                      draw(st.lists(st.integers(0, 5000), min_size=E, max_size=E))))
    linears = [(draw(st.sampled_from([256, 2048, 4096])), draw(st.integers(0, 10**6)),
                draw(st.lists(st.integers(32, 4096), min_size=1, max_size=3)))
               for _ in range(draw(st.integers(0, 3)))]
    return fused, linears


@settings(max_examples=150, deadline=None)
@given(layers(), st.integers(1, 8), st.integers(1, 148), st.booleans())
def test_plan_layer_assigns_every_item_once(layer, world, per_wave, dp):
    from mlx_gptq_b200 import pipeline

    fused, linears = layer
    mgr = _FakeMgr(fused, linears)
    orig = pipeline.hessian_tile_count
    pipeline.hessian_tile_count = lambda c: (-(-c // 256)) * (-(-c // 256) + 1) // 2
    try:
        plans, by_stash, ranges = pipeline.plan_layer(mgr, world, per_wave=per_wave, dp=dp)
    finally:
        pipeline.hessian_tile_count = orig
    assert len(plans) == world
    for ti, (E, _, _, _) in enumerate(fused):
        assert sorted(e for p in plans for e in p["experts"][ti]) == list(range(E))
    assert sorted(n for p in plans for n in p["linears"]) == sorted(t.name for t in mgr.linear_tasks)
    if dp:
        assert all(not p["hessian_parts"] for p in plans) and ranges == {}
    else:
        for key, rs in ranges.items():
            held = sorted((b, e) for p in plans for k, b, e in p["hessian_parts"] if k == key)
            assert held == rs and rs[0][0] == 0
