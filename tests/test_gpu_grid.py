"""GPU grids and packing vs the reference's golden vectors: bit-exact."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STORAGE = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("method", ["mse", "minmax"])
@pytest.mark.parametrize("st", ["bfloat16", "float16", "float32"])
def test_rtn_affine_bit_exact(golden, bits, gs, method, st):
    from mlx_gptq_b200 import grid

    g = golden("rtn_affine")
    k = f"{bits}_{gs}_{method}_{st}"
    q, s, b, dq = grid.rtn_quantize(_cuda(g["W"]), bits, gs, method, STORAGE[st])
    assert s.dtype == STORAGE[st] and b.dtype == STORAGE[st]
    np.testing.assert_array_equal(q.cpu().numpy(), g[f"q_{k}"])
    np.testing.assert_array_equal(s.float().cpu().numpy(), g[f"s_{k}"])
    np.testing.assert_array_equal(b.float().cpu().numpy(), g[f"b_{k}"])
    np.testing.assert_array_equal(dq.cpu().numpy(), g[f"dq_{k}"])


@pytest.mark.parametrize("mode", ["mxfp4", "mxfp8"])
@pytest.mark.parametrize("which", ["", "b"])
def test_rtn_mxfp_bit_exact(golden, mode, which):
    from mlx_gptq_b200 import grid

    g = golden("rtn_mxfp")
    q, s, b, dq = grid.rtn_quantize_mxfp(_cuda(g[f"W{which}_{mode}"]), mode)
    assert b is None and s.dtype == torch.uint8
    np.testing.assert_array_equal(s.cpu().numpy(), g[f"s{which}_{mode}"])
    np.testing.assert_array_equal(q.cpu().numpy(), g[f"q{which}_{mode}"])
    np.testing.assert_array_equal(dq.cpu().numpy().view(np.uint32), g[f"dq{which}_{mode}"].view(np.uint32))


def test_e4m3_codes_bit_exact(golden):
    """MXFP8 with a group max of 448 has scale 2^0, so the codes are the E4M3 cast itself."""
    from mlx_gptq_b200 import grid

    g = golden("e4m3")
    x = np.clip(g["bits"].view(np.float32), -448.0, 448.0)
    n = (len(x) // 31) * 31
    groups = x[:n].reshape(-1, 31)
    W = np.concatenate([groups, np.full((groups.shape[0], 1), 448.0, np.float32)], axis=1)
    q, s, _, dq = grid.rtn_quantize_mxfp(_cuda(W), "mxfp8")
    assert (s.cpu().numpy() == 127).all()
    np.testing.assert_array_equal(q.cpu().numpy()[:, :31].reshape(-1), g["codes"][:n])


def test_dequantize_matches_rtn(golden):
    from mlx_gptq_b200 import grid

    g = golden("rtn_mxfp")
    for mode in ("mxfp4", "mxfp8"):
        W = _cuda(g[f"W_{mode}"])
        q, s, _, dq = grid.rtn_quantize_mxfp(W, mode)
        out = grid.dequantize_artifact(q, s, None, mode, 32)
        assert torch.equal(out, dq)
    ga = golden("rtn_affine")
    q, s, b, dq = grid.rtn_quantize(_cuda(ga["W"]), 4, 64, "mse", torch.float32)
    assert torch.equal(grid.dequantize_artifact(q, s, b, "affine", 64), dq)


def test_pack_bit_exact(golden):
    from mlx_gptq_b200 import artifacts, packing

    g = golden("pack")
    for bits in (2, 4, 8):
        w = packing.pack_q(g[f"q{bits}"], bits)
        np.testing.assert_array_equal(w, g[f"w{bits}"])
        np.testing.assert_array_equal(packing.unpack_q(w, bits, 64), g[f"q{bits}"])
        wt = packing.pack_q(_cuda(g[f"q{bits}"]), bits)
        assert wt.is_cuda
    n = artifacts.pack_nibbles(_cuda(g["qn"]))
    np.testing.assert_array_equal(n.cpu().numpy(), g["nib"])
    np.testing.assert_array_equal(artifacts.unpack_nibbles(n).cpu().numpy(), g["qn"])


def test_rtn_mxfp4_packed_output_matches_pack_q(golden):
    """The fused nibble output of the RTN kernel equals pack_nibbles of its codes."""
    from mlx_gptq_b200 import _lib as L
    from mlx_gptq_b200 import artifacts

    g = golden("rtn_mxfp")
    W = _cuda(g["W_mxfp4"])
    R, C = W.shape
    q = torch.empty(R, C, dtype=torch.uint8, device="cuda")
    qp = torch.empty(R, C // 2, dtype=torch.uint8, device="cuda")
    s = torch.empty(R, C // 32, dtype=torch.uint8, device="cuda")
    L.check(L.lib().gq_rtn_mxfp(W.data_ptr(), L.GQ_F32, R, C, L.GQ_MXFP4, q.data_ptr(), qp.data_ptr(),
                                s.data_ptr(), None, 0, L.stream_ptr()), "rtn")
    assert torch.equal(qp, artifacts.pack_nibbles(q))


def test_pack_edge_cases():
    from mlx_gptq_b200 import packing

    with pytest.raises(ValueError):
        packing.pack_q(np.zeros((2, 32), np.uint8), 3)
    empty = packing.pack_q(np.zeros((0, 32), np.uint8), 4)
    assert empty.shape == (0, 4)
    full = np.full((3, 64), 15, np.uint8)
    assert (packing.pack_q(full, 4) == 0xFFFFFFFF).all()


@pytest.mark.parametrize("mode,fmax", [("mxfp4", 6.0), ("mxfp8", 448.0)])
def test_mxfp_element_codes_dense_sweep(mode, fmax):
    """Every element code of the MXFP grids vs the oracle on ~1M values: a group max of
    fmax pins the scale to 2^0, so the other 31 entries are quantized as they are.
    Covers every threshold +-1 ulp, zeros of both signs, subnormals and saturation."""
    from mlx_gptq_b200 import grid
    from oracle import grid as ogrid

    rng = np.random.default_rng(2024)
    edges = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 448.0, 464.0, 2.0**-9, 2.0**-6, 2.0**-10],
                     np.float32)
    near = np.concatenate([np.nextafter(edges, np.float32(0)), edges, np.nextafter(edges, np.float32(1e9))])
    vals = np.concatenate([near, -near, [0.0, -0.0, 1e-40, -1e-40, 7.0, -7.0, 500.0, -500.0]]).astype(np.float32)
    rnd = (rng.standard_normal(1 << 20) * rng.choice([0.01, 0.3, 1.0, 3.0, 100.0], 1 << 20)).astype(np.float32)
    x = np.concatenate([vals, rnd])
    x = np.clip(x, -fmax, fmax) if mode == "mxfp4" else x
    n = (len(x) // 31) * 31
    W = np.concatenate([x[:n].reshape(-1, 31), np.full((n // 31, 1), fmax, np.float32)], axis=1)
    q, s, _, dq = grid.rtn_quantize_mxfp(_cuda(W), mode)
    oq, os_, _, odq = ogrid.rtn_quantize_mxfp(W, mode)
    np.testing.assert_array_equal(s.cpu().numpy(), os_)
    np.testing.assert_array_equal(q.cpu().numpy(), oq)
    np.testing.assert_array_equal(dq.cpu().numpy().view(np.uint32), odq.view(np.uint32))
