"""tcgen05 Hessian kernel vs the reference (golden) and a float64 torch reference.

Tolerance (north star): relative Frobenius error <= 1e-5.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HESSIAN_RTOL = 1e-5


@pytest.fixture(autouse=True, params=["1sm", "2sm"])
def hessian_kernel(request, monkeypatch):
    """Every test runs with both tcgen05 kernels: 128x256 tiles on one SM, 256x256 on a CTA pair."""
    monkeypatch.setenv("GQ_HESSIAN_KERNEL", request.param)
    return request.param


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


def test_hessian_matches_reference_golden(golden):
    from mlx_gptq_b200 import Stash

    g = golden("hessian")
    X = torch.from_numpy(g["X_bits"].view(np.int16).copy()).view(torch.bfloat16)
    st = Stash("x", 96)
    st.add(X[:1000])
    st.add(X[1000:])
    H = st.hessian("cuda", chunk_rows=512)
    assert _rel(H.cpu(), torch.from_numpy(g["H"])) < HESSIAN_RTOL
    assert torch.equal(H, H.T)


@pytest.mark.parametrize("n,c", [(1000, 96), (4096, 256), (20000, 768), (65536, 1024), (3, 64), (777, 200)])
def test_hessian_vs_float64(n, c):
    from mlx_gptq_b200 import hessian_from_rows

    torch.manual_seed(n + c)
    X = torch.randn(n, c, device="cuda")
    X[:, : max(1, c // 64)] *= 20.0  # outlier channels
    X = X.to(torch.bfloat16)
    H = hessian_from_rows(X)
    ref = X.double().T @ X.double()
    assert _rel(H, ref) < HESSIAN_RTOL
    assert torch.equal(H, H.T)


def test_hessian_accumulate_alpha_beta():
    from mlx_gptq_b200 import hessian_accumulate

    torch.manual_seed(3)
    X1 = torch.randn(3000, 256, device="cuda").to(torch.bfloat16)
    X2 = torch.randn(5000, 256, device="cuda").to(torch.bfloat16)
    H = torch.full((256, 256), 7.0, device="cuda")
    hessian_accumulate(X1, H, 1.0, 0.0)
    hessian_accumulate(X2, H, 0.5, 1.0)
    ref = X1.double().T @ X1.double() + 0.5 * (X2.double().T @ X2.double())
    assert _rel(H, ref) < HESSIAN_RTOL


def test_hessian_strided_rows_and_zero_tokens():
    from mlx_gptq_b200 import hessian_accumulate

    torch.manual_seed(4)
    big = torch.randn(2048, 384, device="cuda").to(torch.bfloat16)
    X = big[:, :256]  # row stride 384
    H = torch.empty(256, 256, device="cuda")
    hessian_accumulate(X, H, 1.0, 0.0)
    assert _rel(H, X.double().T @ X.double()) < HESSIAN_RTOL
    H2 = H.clone()
    hessian_accumulate(X[:0], H2, 1.0, 1.0)  # no tokens: unchanged
    assert torch.equal(H2, H)
    hessian_accumulate(X[:0], H2, 1.0, 0.0)  # no tokens, overwrite: zeros
    assert int(torch.count_nonzero(H2)) == 0


def test_hessian_full_size_property():
    """At the bench's size (K = 4096), H is symmetric, PSD-diagonal and close to fp64."""
    from mlx_gptq_b200 import hessian_from_rows

    torch.manual_seed(5)
    X = (torch.randn(131072, 4096, device="cuda")).to(torch.bfloat16)
    H = hessian_from_rows(X)
    ref = X[:, :512].double().T @ X.double()
    assert _rel(H[:512], ref) < HESSIAN_RTOL
    assert torch.equal(H, H.T)


def _routing(T, E, k, seed, empty=(3,)):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, E, generator=g) + torch.linspace(2.0, -2.0, E)  # skewed load
    for e in empty:
        logits[:, e] = -1e9
    top = logits.topk(k, dim=1).indices  # [T, k]
    slots = top.reshape(-1)
    tok = torch.arange(T).repeat_interleave(k)
    order = torch.sort(slots, stable=True).indices
    token_idx = tok[order].to(torch.int32)
    counts = torch.bincount(slots, minlength=E)
    offsets = torch.zeros(E + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, 0)
    return token_idx, offsets


@pytest.mark.parametrize("T,E,k,c", [(3000, 8, 2, 256), (20000, 16, 4, 512), (1000, 5, 1, 96)])
def test_hessian_grouped_matches_per_expert_dense(T, E, k, c):
    """One grouped launch == the dense kernel on each expert's gathered rows (bit-exact),
    and == float64 within the tolerance; experts without tokens get zeros."""
    from mlx_gptq_b200 import hessian_from_rows, hessian_grouped

    torch.manual_seed(T)
    X = torch.randn(T, c, device="cuda")
    X[:, 1] *= 20.0
    X = X.to(torch.bfloat16)
    token_idx, offsets = _routing(T, E, k, seed=T)
    H = hessian_grouped(X, token_idx, offsets, E)
    for e in range(E):
        rows = token_idx[offsets[e]:offsets[e + 1]].long().cuda()
        if len(rows) == 0:
            assert int(torch.count_nonzero(H[e])) == 0
            continue
        Xe = X[rows]
        assert torch.equal(H[e], hessian_from_rows(Xe))
        assert _rel(H[e], Xe.double().T @ Xe.double()) < HESSIAN_RTOL


def test_hessian_grouped_vs_oracle_and_beta():
    from mlx_gptq_b200 import hessian_grouped
    from oracle import hessian as ohess

    torch.manual_seed(9)
    T, E, c = 2048, 6, 128
    X = torch.randn(T, c, device="cuda").to(torch.bfloat16)
    token_idx, offsets = _routing(T, E, 2, seed=9, empty=(0,))
    ref = ohess.hessian_grouped(X.float().cpu().numpy(), token_idx.numpy(), offsets.numpy())
    H = torch.full((E, c, c), 2.0, device="cuda")
    hessian_grouped(X, token_idx, offsets, E, H=H, alpha=1.0, beta=1.0)
    got = H.cpu().numpy() - 2.0
    for e in range(E):
        den = max(float(np.linalg.norm(ref[e])), 1e-30)
        assert float(np.linalg.norm(got[e] - ref[e])) / den < 1e-5 or den < 1e-20


@pytest.mark.parametrize("parts", [3, 8])
@pytest.mark.parametrize("c", [1088, 2048])
def test_hessian_tile_ranges_compose_bit_exact(parts, c):
    """Disjoint tile ranges write disjoint blocks whose union is the full H, bit for bit
    (how ranks holding every row of X split one Hessian)."""
    from mlx_gptq_b200.capture import hessian_accumulate, hessian_from_rows, hessian_tile_count

    g = torch.Generator(device="cuda").manual_seed(c + parts)
    X = torch.randn(3000, c, generator=g, device="cuda").to(torch.bfloat16)
    full = hessian_from_rows(X)
    T = hessian_tile_count(c)
    assert T > parts
    total = torch.zeros(c, c, device="cuda")
    written = torch.zeros(c, c, dtype=torch.int32, device="cuda")
    for r in range(parts):
        Hr = torch.full((c, c), float("nan"), device="cuda")
        hessian_accumulate(X, Hr, 1.0, 0.0, tiles=(r * T // parts, (r + 1) * T // parts))
        mine = ~torch.isnan(Hr)
        written += mine.int()
        total += torch.where(mine, Hr, torch.zeros_like(Hr))
    assert bool((written == 1).all())  # every element written by exactly one range
    assert torch.equal(total, full)
    with pytest.raises(ValueError):
        hessian_accumulate(X, full, 1.0, 0.0, tiles=(0, T + 1))


@pytest.mark.parametrize("c", [96, 768, 2048])
def test_hessian_spans_match_per_expert_dense(c):
    """Span form (rows read in place, partial last steps from the tail buffer) == the
    dense kernel on each span's rows, bit for bit: odd lengths, an empty span, a span
    of exactly 64 rows, overlapping and unordered spans; beta accumulates."""
    from mlx_gptq_b200 import hessian_from_rows
    from mlx_gptq_b200.capture import hessian_spans

    g = torch.Generator(device="cuda").manual_seed(c)
    X = (torch.randn(5000, c, generator=g, device="cuda") * 3.0).to(torch.bfloat16)
    spans = [(0, 1000), (1000, 37), (1037, 0), (1100, 64), (40, 3900), (4999, 1), (2000, 2999)]
    H = hessian_spans(X, spans)
    for e, (a, k) in enumerate(spans):
        if k == 0:
            assert int(torch.count_nonzero(H[e])) == 0
            continue
        assert torch.equal(H[e], hessian_from_rows(X[a:a + k])), (c, e)
    H2 = hessian_spans(X, spans, H=H.clone(), alpha=1.0, beta=1.0)
    torch.testing.assert_close(H2, 2.0 * H, rtol=0, atol=0)
    with pytest.raises(ValueError):
        hessian_spans(X, [(4990, 20)])  # past the last row


@pytest.mark.parametrize("form", ["gather", "spans"])
def test_expert_pieces_merged_in_order(form):
    """Heavy experts cut into pieces (one grouped launch over the pieces) and summed by
    the one-launch merge: bit for bit the pieces' Hessians added one by one in piece
    order, and within float32 rounding of each expert's dense Hessian."""
    from mlx_gptq_b200 import hessian_from_rows
    from mlx_gptq_b200.capture import hessian_grouped, hessian_spans
    from mlx_gptq_b200.expert_batch import expert_hessians, piece_layout

    c = 256
    g = torch.Generator(device="cuda").manual_seed(7)
    counts = [3000, 5, 0, 700, 1999]
    off = [0]
    for n in counts:
        off.append(off[-1] + n)
    X = torch.randn(off[-1], c, generator=g, device="cuda").to(torch.bfloat16)
    tok = torch.randperm(off[-1], generator=g, device="cuda").to(torch.int32)
    lay = piece_layout(tok if form == "gather" else None, torch.tensor(off), list(range(len(counts))), c, "cuda",
                       waves=1.0, tiles_per_wave=4)
    assert lay.extra  # the heavy experts were cut
    V = lay.offsets.numel() - 1
    raw = (hessian_grouped(X, lay.token_idx, lay.offsets, V) if form == "gather" else hessian_spans(X, lay.spans))
    for j, (i, _) in enumerate(lay.extra):
        raw[i].add_(raw[lay.n + j])
    H = expert_hessians(X, lay)
    assert torch.equal(H, raw[: lay.n])
    for e, n in enumerate(counts):
        rows = X[tok[off[e]:off[e + 1]].long()] if form == "gather" else X[off[e]:off[e + 1]]
        if n == 0:
            assert int(torch.count_nonzero(H[e])) == 0
            continue
        ref = hessian_from_rows(rows).double()
        err = float((H[e].double() - ref).norm() / ref.norm())
        assert err < 1e-5, (form, e, err)


@pytest.mark.parametrize("c", [5, 64])  # odd c: the element-wise path; c % 4 == 0 after squaring: float4
def test_merge_pieces_entry_point_order_and_bits(c):
    """gq_hessian_merge_pieces through the C ABI: each target gets its pieces added one
    after another in list order (bit-identical to sequential adds), other slabs untouched."""
    import ctypes

    from mlx_gptq_b200 import _lib

    g = torch.Generator(device="cuda").manual_seed(c)
    H = torch.randn(7, c, c, generator=g, device="cuda") * torch.logspace(-3, 3, 7, device="cuda")[:, None, None]
    targets, lists = [0, 2], [[5, 3, 6], [4]]
    want = H.clone()
    for t, ps in zip(targets, lists):
        for p in ps:
            want[t] += want[p]
    dev = lambda v: torch.tensor(v, dtype=torch.int64, device="cuda")
    tg, ptr, pcs = dev(targets), dev([0, 3, 4]), dev([5, 3, 6, 4])
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    st = _lib.lib().gq_hessian_merge_pieces(p(H), c, 2, p(tg), p(ptr), p(pcs), None)
    torch.cuda.synchronize()
    assert st == _lib.GQ_OK
    assert torch.equal(H, want)
