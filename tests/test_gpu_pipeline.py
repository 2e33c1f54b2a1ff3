"""Layer pipeline on the GPU: capture -> grouped Hessians -> batched solves -> artifacts.

Each expert's artifact must equal a direct solve_gptq on that expert's captured
rows (same kernels: bit-exact), the layer's weights must be the dequantized
artifacts, and the artifact store must round-trip.
"""

import numpy as np
import pytest
import torch

from test_pipeline_cpu import ToyMoELayer

pytestmark = pytest.mark.gpu


def _captured(mode_seed=0, E=6, H=128, k=2, T=512, group_size=32):
    from mlx_gptq_b200.capture import CaptureManager

    torch.manual_seed(mode_seed)
    layer = ToyMoELayer(H=H, E=E, k=k).cuda()
    layer.experts.gate_up_proj.data.mul_(0.05)
    layer.experts.down_proj.data.mul_(0.05)
    mgr = CaptureManager(layer, exclude_regex=r"(^|\.)gate$", group_size=group_size)
    with mgr, torch.no_grad():
        for _ in range(2):
            mgr.begin_batch()
            layer(torch.randn(T // 2, H, device="cuda"))
    return layer, mgr


@pytest.mark.parametrize("mode,bits,gs", [("mxfp4", 4, 32), ("affine", 4, 64), ("mxfp8", 8, 32)])
def test_solve_layer_matches_direct_solves(mode, bits, gs, tmp_path):
    from mlx_gptq_b200 import hessian_from_rows, solve_gptq
    from mlx_gptq_b200.artifacts import ArtifactReader, ArtifactWriter
    from mlx_gptq_b200.grid import dequantize_artifact
    from mlx_gptq_b200.pipeline import LayerSolveArgs, solve_layer

    layer, mgr = _captured(group_size=gs)
    gu = next(t for t in mgr.fused_tasks if t.param_name == "gate_up_proj")
    W0 = gu.param.detach().clone()
    rows = {e: mgr.stashes[gu.stash_keys[e]].rows("cuda") for e in range(gu.num_experts)}
    args = LayerSolveArgs(bits=bits, group_size=gs, mode=mode)
    res = solve_layer("model.layers.0", mgr, args, "cuda")
    R = W0.shape[1]
    for e in range(gu.num_experts):
        if rows[e].shape[0] == 0:
            continue
        H = hessian_from_rows(rows[e]).unsqueeze(0).contiguous()
        q, s, b, W_dq, rel = solve_gptq(W0[e:e + 1].float(), H, bits, gs, mode=mode)
        qg, sg, bg = res.tensors[f"model.layers.0.experts.{e}.gate_proj.weight"]
        qu, su, bu = res.tensors[f"model.layers.0.experts.{e}.up_proj.weight"]
        assert torch.equal(torch.cat([qg, qu]), q[0].cpu())
        assert torch.equal(torch.cat([sg, su]), s[0].cpu())
        assert torch.equal(gu.param.data[e], W_dq[0].to(gu.param.dtype))
        meta = res.meta[f"model.layers.0.experts.{e}.gate_proj.weight"]
        assert meta["kind"] == "expert" and meta["out_features"] == R // 2 and meta["tokens"] == rows[e].shape[0]
    # linears: q/k share one stash
    assert {m["kind"] for m in res.meta.values()} == {"expert", "linear"}
    # artifact store round trip + dequantization == new layer weights
    writer = ArtifactWriter(str(tmp_path), {"mode": mode, "bits": bits, "group_size": gs,
                                            "storage_dtype": "bfloat16"})
    writer.write_layer(0, res.tensors, res.meta)
    reader = ArtifactReader(str(tmp_path))
    name = "model.layers.0.q_proj.weight"
    q, s, b, info = reader.get(name)
    assert info["q_packed"] == ("nibble" if bits == 4 else "raw")
    assert torch.equal(q, res.tensors[name][0])
    dq = dequantize_artifact(q.cuda(), s.cuda(), None if b is None else b.cuda(), mode, gs)
    assert torch.equal(dq.to(layer.q_proj.weight.dtype), layer.q_proj.weight.data)


def test_expert_hessians_vs_float64():
    layer, mgr = _captured(E=5, H=96)
    dn = next(t for t in mgr.fused_tasks if t.param_name == "down_proj")
    Hs = mgr.expert_hessians(dn, "cuda")
    for e in range(dn.num_experts):
        X = mgr.stashes[dn.stash_keys[e]].rows("cuda").double()
        ref = X.T @ X
        if X.shape[0] == 0:
            assert int(torch.count_nonzero(Hs[e])) == 0
            continue
        assert float((Hs[e].double() - ref).norm() / ref.norm()) < 1e-5
