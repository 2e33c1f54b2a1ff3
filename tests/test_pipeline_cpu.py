"""Capture routing and layer scheduling host logic (CPU, no kernels).

Mirrors the behaviour the reference's tests/test_capture.py pins: router
exclusion, q/k input dedup into one stash, top-k routing invariants, gate_up
and down token counts per expert, unrouted-expert backfill (64 sampled rows).
The sharded layer solve is checked with gloo ranks and a fake solver: every
rank ends with the single-process result.
"""

import os
import re

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from mlx_gptq_b200.capture import CaptureManager
from mlx_gptq_b200.pipeline import LayerSolveArgs, artifact_names_for_fused, lpt_partition


class FusedExperts(nn.Module):
    """transformers >= 5 fused expert layout: F.linear on one expert slice at a time."""

    def __init__(self, E=4, H=32, I=32):
        super().__init__()
        self.gate_up_proj = nn.Parameter(torch.randn(E, 2 * I, H))
        self.down_proj = nn.Parameter(torch.randn(E, H, I))
        self.num_experts = E

    def forward(self, x, top_k_index):
        out = torch.zeros_like(x)
        for e in range(self.num_experts):
            tok = (top_k_index == e).any(dim=-1).nonzero().flatten()
            if tok.numel() == 0:
                continue
            gate, up = F.linear(x[tok], self.gate_up_proj[torch.tensor(e)]).chunk(2, -1)
            out.index_add_(0, tok, F.linear(F.silu(gate) * up, self.down_proj[torch.tensor(e)]))
        return out


class ToyMoELayer(nn.Module):
    def __init__(self, H=32, E=4, k=2):
        super().__init__()
        self.q_proj = nn.Linear(H, H, bias=False)
        self.k_proj = nn.Linear(H, H, bias=False)
        self.gate = nn.Linear(H, E, bias=False)  # router: excluded
        self.experts = FusedExperts(E=E, H=H)
        self.k = k

    def forward(self, x):
        y = self.q_proj(x) + self.k_proj(x)
        return self.experts(y, self.gate(y).topk(self.k, dim=-1).indices)


class OneExpertLayer(nn.Module):
    def __init__(self):
        super().__init__()
        self.experts = FusedExperts()

    def forward(self, x):
        return self.experts(x, torch.zeros((x.shape[0], 1), dtype=torch.long))


def test_capture_discovery_dedup_and_routing():
    torch.manual_seed(0)
    layer = ToyMoELayer()
    mgr = CaptureManager(layer, exclude_regex=r"(^|\.)gate$", group_size=32)
    assert {t.name for t in mgr.linear_tasks} == {"q_proj", "k_proj"}
    assert {t.param_name for t in mgr.fused_tasks} == {"gate_up_proj", "down_proj"}
    T = 64
    with mgr:
        mgr.begin_batch()
        layer(torch.randn(T, 32))
    keys = {t.stash_key for t in mgr.linear_tasks}
    assert len(keys) == 1 and mgr.stashes[keys.pop()].tokens == T  # q/k share one stash
    gu = next(t for t in mgr.fused_tasks if t.param_name == "gate_up_proj")
    dn = next(t for t in mgr.fused_tasks if t.param_name == "down_proj")
    assert sum(mgr.stashes[k].tokens for k in gu.stash_keys) == 2 * T
    for kg, kd in zip(gu.stash_keys, dn.stash_keys):
        assert mgr.stashes[kg].tokens == mgr.stashes[kd].tokens
    mgr.check_capture_happened()
    stats = mgr.expert_token_stats()
    assert set(stats) == {"experts.gate_up_proj", "experts.down_proj"}


def test_group_size_filter_and_capture_check():
    layer = nn.Sequential(nn.Linear(48, 8, bias=False), nn.Linear(64, 8, bias=False))
    mgr = CaptureManager(layer, exclude_regex=None, group_size=32)
    assert [t.name for t in mgr.linear_tasks] == ["1"]  # 48 % 32 != 0: stays unquantized
    mgr = CaptureManager(layer, exclude_regex=None, group_size=16)
    assert {t.name for t in mgr.linear_tasks} == {"0", "1"}
    moe = OneExpertLayer()
    mgr = CaptureManager(moe, exclude_regex=None, group_size=32)
    with pytest.raises(RuntimeError, match="No tokens captured"):
        mgr.check_capture_happened()


def test_unrouted_experts_backfill():
    torch.manual_seed(0)
    layer = OneExpertLayer()
    mgr = CaptureManager(layer, exclude_regex=None, group_size=32)
    with mgr:
        mgr.begin_batch()
        layer(torch.randn(96, 32))
    gu = next(t for t in mgr.fused_tasks if t.param_name == "gate_up_proj")
    dn = next(t for t in mgr.fused_tasks if t.param_name == "down_proj")
    assert mgr.stashes[gu.stash_keys[0]].tokens == 96 and mgr.stashes[gu.stash_keys[1]].tokens == 0
    assert mgr.backfill_unrouted_experts() == {"experts": [1, 2, 3]}
    for e in (1, 2, 3):
        assert mgr.stashes[gu.stash_keys[e]].tokens == 64
        assert mgr.stashes[dn.stash_keys[e]].tokens == 64
        assert mgr.fallback_experts[gu.stash_keys[e]] == "all_expert_inputs"


def test_artifact_names_and_overrides():
    layer = ToyMoELayer()
    mgr = CaptureManager(layer, exclude_regex=r"(^|\.)gate$", group_size=32)
    gu = next(t for t in mgr.fused_tasks if t.param_name == "gate_up_proj")
    dn = next(t for t in mgr.fused_tasks if t.param_name == "down_proj")
    assert artifact_names_for_fused("model.layers.3", gu, 7) == [
        "model.layers.3.experts.7.gate_proj.weight", "model.layers.3.experts.7.up_proj.weight"]
    assert artifact_names_for_fused("model.layers.3", dn, 0) == ["model.layers.3.experts.0.down_proj.weight"]
    args = LayerSolveArgs(bits=4, overrides=[(re.compile(r"down_proj"), 8)])
    assert args.bits_for("x.experts.0.down_proj.weight") == 8 and args.bits_for("x.q_proj.weight") == 4


def test_lpt_partition_balances_and_covers():
    costs = [100, 1, 1, 1, 50, 50, 3, 0, 0, 7]
    bins = lpt_partition(costs, 3)
    assert sorted(i for b in bins for i in b) == list(range(len(costs)))
    loads = [sum(costs[i] for i in b) for b in bins]
    assert max(loads) == 100 and min(loads) >= 50
    assert lpt_partition(costs, 1) == [list(range(len(costs)))]
    assert lpt_partition([], 4) == [[], [], [], []]


def _fake_dequant(q, s, b, mode, group_size):
    return q.float() * 0.01 * s.float().repeat_interleave(group_size, dim=-1)


def _fake_pack(q):
    return q[..., 0::2] | (q[..., 1::2] << 4)


def _fake_unpack(p):
    return torch.stack([p & 15, p >> 4], dim=-1).reshape(*p.shape[:-1], -1)


def _fake_solve(W, H, bits, args):
    """Deterministic stand-in for the GPU solver (CPU tensors); W_dq is the
    dequantization of (q, s), as it is for the real MXFP solver."""
    B, R, C = W.shape
    d = H.diagonal(dim1=-2, dim2=-1).unsqueeze(1)
    q = (W.abs() * 7 + d * 1e-3).round().clamp(0, 15).to(torch.uint8)
    s = torch.full((B, R, C // args.group_size), 3, dtype=torch.uint8)
    W_dq = _fake_dequant(q, s, None, args.mode, args.group_size)
    rel = W_dq.flatten(1).norm(dim=1)
    return q, s, None, W_dq, rel


def install_fakes(pipeline_mod, capture_mod, setattr_=setattr):
    """Replace the CUDA pieces the layer solve calls with CPU stand-ins (pass
    monkeypatch.setattr inside the test process, so they are undone afterwards)."""
    for obj, name, fn in ((pipeline_mod, "_solve_batch", _fake_solve),
                          (pipeline_mod, "dequantize_artifact", _fake_dequant),
                          (pipeline_mod, "pack_nibbles", _fake_pack), (pipeline_mod, "unpack_nibbles", _fake_unpack),
                          (pipeline_mod, "hessian_tile_count", _fake_tile_count),
                          (pipeline_mod, "hessian_tiles_per_wave", _fake_tiles_per_wave),
                          (capture_mod.CaptureManager, "expert_hessians", _fake_expert_hessians),
                          (capture_mod.Stash, "hessian", _fake_stash_hessian)):
        setattr_(obj, name, fn)


def _fake_expert_hessians(self, task, device, experts=None, timer=None):
    experts = list(range(task.num_experts)) if experts is None else list(experts)
    C = task.param.shape[-1]
    return torch.stack([torch.eye(C) * (self.stashes[task.stash_keys[e]].tokens + 1) for e in experts])


def _fake_stash_hessian(self, device, chunk_rows=65536, tiles=None):
    """A stand-in H; with tiles=(b, e) only rows b..e (one "tile" per row), zero elsewhere."""
    H = torch.eye(self.in_features) * (self.tokens + 1) + 0.01 * torch.arange(self.in_features).float()
    if tiles is not None:
        mask = torch.zeros(self.in_features, 1)
        mask[tiles[0]:tiles[1]] = 1
        H = H * mask
    return H


def _fake_tile_count(c):
    return c


def _fake_tiles_per_wave(device=None):
    return 20  # a 32-feature stash (32 "tiles") is formed in two parts


def _run_layer(rank, world, port, out_dir, setattr_=setattr):
    import torch.distributed as dist

    from mlx_gptq_b200 import capture, pipeline

    install_fakes(pipeline, capture, setattr_)
    group = None
    if world > 1:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        group = dist.group.WORLD
    torch.manual_seed(0)
    layer = ToyMoELayer(E=5, k=2)
    mgr = CaptureManager(layer, exclude_regex=r"(^|\.)gate$", group_size=32)
    with mgr:
        mgr.begin_batch()
        layer(torch.randn(40, 32))
    args = LayerSolveArgs(bits=4, group_size=32, mode="mxfp4")
    res = pipeline.solve_layer("model.layers.0", mgr, args, "cpu", group=group)
    torch.save({"tensors": res.tensors, "meta": res.meta,
                "weights": {k: v.detach().clone() for k, v in layer.state_dict().items()}},
               os.path.join(out_dir, f"r{world}_{rank}.pt"))
    if world > 1:
        dist.destroy_process_group()


def test_sharded_layer_solve_matches_single_process(tmp_path, monkeypatch):
    import socket

    import torch.multiprocessing as mp

    _run_layer(0, 1, 0, str(tmp_path), monkeypatch.setattr)
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    mp.start_processes(_run_layer, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    ref = torch.load(tmp_path / "r1_0.pt")
    for r in range(2):
        got = torch.load(tmp_path / f"r2_{r}.pt")
        assert got["meta"] == ref["meta"]
        assert set(got["tensors"]) == set(ref["tensors"])
        for k, (q, s, b) in ref["tensors"].items():
            q2, s2, b2 = got["tensors"][k]
            assert torch.equal(q, q2) and torch.equal(s, s2)
        for k, v in ref["weights"].items():
            assert torch.equal(v, got["weights"][k]), k


def test_plan_layer_covers_every_item_once_and_balances(monkeypatch):
    from mlx_gptq_b200 import pipeline
    from mlx_gptq_b200.pipeline import plan_layer

    monkeypatch.setattr(pipeline, "hessian_tile_count", _fake_tile_count)

    torch.manual_seed(0)
    layer = ToyMoELayer(E=6, k=2)
    mgr = CaptureManager(layer, exclude_regex=r"(^|\.)gate$", group_size=32)
    with mgr:
        mgr.begin_batch()
        layer(torch.randn(64, 32))
    for world in (1, 2, 3, 8):
        plans, by_stash, ranges = plan_layer(mgr, world, per_wave=10)
        assert len(plans) == world
        for key, rs in ranges.items():  # tile ranges tile the stash's H, each part on one rank
            assert [r for p in plans for r in p["hessian_parts"] if r[0] == key] is not None
            got = sorted((b, e) for p in plans for k, b, e in p["hessian_parts"] if k == key)
            assert got == rs and rs[0][0] == 0 and all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            assert len(rs) == (1 if world == 1 else min(world, 4))
        for ti, task in enumerate(mgr.fused_tasks):
            got = sorted(e for p in plans for e in p["experts"][ti])
            assert got == list(range(task.num_experts))
        assert sorted(k for p in plans for k in p["linears"]) == sorted(t.name for t in mgr.linear_tasks)
    # q/k share one stash: one linear item
    assert len(by_stash) == 1 and len(next(iter(by_stash.values()))) == 2


def test_vram_budget_splits_expert_batches(monkeypatch):
    """A budget smaller than one expert's working set solves experts in chunks of one;
    the artifacts equal those of one batched solve (sequential.py:314-318)."""
    from mlx_gptq_b200 import capture, pipeline

    install_fakes(pipeline, capture, monkeypatch.setattr)
    calls = []
    real = pipeline._solve_batch

    def counting(W, H, bits, args):
        calls.append(W.shape[0])
        return real(W, H, bits, args)

    monkeypatch.setattr(pipeline, "_solve_batch", counting)
    assert pipeline.expert_chunk_size(2048, 1536, 16.0) == int(16 * 2**30 // ((3 * 2048**2 + 3 * 1536 * 2048) * 4))
    assert pipeline.expert_chunk_size(64, 64, 1e-9) == 1
    out = {}
    for budget in (None, 1e-9):
        torch.manual_seed(0)
        layer = ToyMoELayer(E=5, k=2)
        mgr = CaptureManager(layer, exclude_regex=r"(^|\.)gate$", group_size=32)
        with mgr:
            mgr.begin_batch()
            layer(torch.randn(40, 32))
        calls.clear()
        res = pipeline.solve_layer("model.layers.0", mgr, LayerSolveArgs(bits=4, group_size=32, mode="mxfp4",
                                                                         vram_gb=budget), "cpu")
        out[budget] = (res, list(calls))
    assert max(out[1e-9][1]) == 1 and max(out[None][1]) == 5
    for k, (q, s, b) in out[None][0].tensors.items():
        q2, s2, _ = out[1e-9][0].tensors[k]
        assert torch.equal(q, q2) and torch.equal(s, s2)
