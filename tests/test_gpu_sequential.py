"""Layer-sequential driver on the GPU: a tiny random-init Qwen3-MoE stack.

Layer 0's artifacts are checked against the oracle (numpy restatement of the
reference solver) on the same captured rows: codes agree on >= 99.9% of
elements, E8M0 scales and per-tensor rel_err within the GPTQ tolerances. The
resume path (dequantized artifacts written back) reproduces the hidden states
of the run that wrote them bit for bit.
"""

import types

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TINY = dict(model_type="qwen3_moe", vocab_size=1024, hidden_size=128, intermediate_size=256,
            moe_intermediate_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
            head_dim=32, num_experts=8, num_experts_per_tok=2, decoder_sparse_step=1, norm_topk_prob=True,
            max_position_embeddings=256)


def _args(mode="mxfp4", experts_forward="grouped"):
    from mlx_gptq_b200 import sequential

    return types.SimpleNamespace(devices=["cuda:0"], dtype="bfloat16", layers_attr="model.layers",
                                 checkpoint_model_prefix=None, artifact_layers_prefix=None,
                                 exclude=sequential.DEFAULT_EXCLUDE, group_size=32, bits=4 if mode == "mxfp4" else 8,
                                 mode=mode, mxfp_algorithm="safe-scale-search" if mode == "mxfp4" else "groupwise",
                                 damp=0.01, clip="mse", overrides=[], batch_size=4,
                                 experts_forward=experts_forward)


def _samples():
    return torch.randint(0, TINY["vocab_size"], (8, 64), generator=torch.Generator().manual_seed(1))


def _rows_f32(rows):
    return rows.float().cpu().numpy()


@pytest.mark.parametrize("mode", ["mxfp4", "mxfp8"])
def test_stack_layer0_matches_oracle(mode, tmp_path):
    from mlx_gptq_b200 import sequential
    from mlx_gptq_b200.artifacts import ArtifactReader, ArtifactWriter
    from mlx_gptq_b200.capture import CaptureManager
    from oracle import gptq as ogptq
    from oracle import hessian as ohess

    args = _args(mode)
    model = sequential.build_model(TINY)
    src = sequential.SyntheticWeights(model, "cuda:0", seed=0)
    pipe = sequential.Pipeline(model, src, args)
    writer = ArtifactWriter(str(tmp_path), {"mode": mode, "bits": args.bits, "group_size": 32,
                                            "storage_dtype": "bfloat16"})
    pipe.run(_samples(), writer, layers=1)
    reader = ArtifactReader(str(tmp_path))

    # the same capture again, on a fresh skeleton with the same synthetic weights
    model2 = sequential.build_model(TINY)
    pipe2 = sequential.Pipeline(model2, sequential.SyntheticWeights(model2, "cuda:0", seed=0), args)
    batches = pipe2.catch_layer0_inputs(_samples(), args.batch_size)
    layer = pipe2.layers[0]
    sequential.materialize_module(layer, "model.layers.0", pipe2.shards, pipe2.dev0, pipe2.dtype)
    W0 = {n: p.detach().float().cpu().numpy() for n, p in layer.named_parameters()}
    mgr = CaptureManager(layer, args.exclude, 32, stash_device="cuda:0")
    with mgr:
        pipe2.forward_layer(layer, batches, 0, capture_mgr=mgr)
    mgr.backfill_unrouted_experts()

    checked = agree = total = 0
    for t in mgr.linear_tasks:
        H = ohess.hessian(_rows_f32(mgr.stashes[t.stash_key].rows("cuda")))
        q, s, _, _, rel = ogptq.solve_gptq(W0[f"{t.name}.weight"][None], H[None], args.bits, 32, mode=mode,
                                           mxfp_algorithm=args.mxfp_algorithm)
        gq, gs, gb, info = reader.get(f"model.layers.0.{t.name}.weight")
        agree += int((gq.numpy() == q[0]).sum())
        total += q[0].size
        assert (gs.numpy() == s[0]).mean() >= 0.999
        assert abs(info["rel_err"] - float(rel[0])) <= 0.005 * float(rel[0]) + 1e-6
        checked += 1
    for task in mgr.fused_tasks:
        Wp = W0[f"{task.module_name}.{task.param_name}"]
        for e in range(task.num_experts):
            rows = _rows_f32(mgr.expert_rows(task, e, "cuda"))
            H = ohess.hessian(rows)
            q, s, _, _, _ = ogptq.solve_gptq(Wp[e][None], H[None], args.bits, 32, mode=mode,
                                             mxfp_algorithm=args.mxfp_algorithm)
            names = [f"model.layers.0.{task.module_name}.{e}.{k}.weight" for k in
                     (("gate_proj", "up_proj") if task.param_name == "gate_up_proj" else (task.param_name,))]
            got = [reader.get(n) for n in names]
            gq = np.concatenate([g[0].numpy() for g in got], 0)
            gs = np.concatenate([g[1].numpy() for g in got], 0)
            agree += int((gq == q[0]).sum())
            total += q[0].size
            assert (gs == s[0]).mean() >= 0.999
            assert got[0][3]["tokens"] == rows.shape[0]
            checked += 1
    assert checked == 4 + 2 * 8
    assert agree / total >= 0.999, agree / total


def test_stack_resume_reproduces_hidden_states(tmp_path):
    from mlx_gptq_b200 import sequential
    from mlx_gptq_b200.artifacts import ArtifactReader, ArtifactWriter

    args = _args("mxfp4")
    header = {"mode": "mxfp4", "bits": 4, "group_size": 32, "storage_dtype": "bfloat16"}
    model = sequential.build_model(TINY)
    pipe = sequential.Pipeline(model, sequential.SyntheticWeights(model, "cuda:0", seed=0), args)
    out = pipe.run(_samples(), ArtifactWriter(str(tmp_path), header))
    assert [s.layer for s in pipe.stats] == [0, 1]
    assert all(0.0 < s.rel_err_max < 0.5 for s in pipe.stats)

    model2 = sequential.build_model(TINY)
    pipe2 = sequential.Pipeline(model2, sequential.SyntheticWeights(model2, "cuda:0", seed=0), args)
    writer = ArtifactWriter(str(tmp_path), header)
    assert writer.layer_done(0) and writer.layer_done(1)
    out2 = pipe2.run(_samples(), writer, reader_for_resume=ArtifactReader(str(tmp_path)))
    assert pipe2.stats == []  # every layer resumed
    for (h1, _), (h2, _) in zip(out, out2):
        assert torch.equal(h1, h2)


def test_grouped_and_eager_expert_forward_give_identical_artifacts(tmp_path):
    """The sort-based expert forward with segment capture is the eager loop with
    F.linear interception, bit for bit: same hidden states, same artifacts."""
    from mlx_gptq_b200 import sequential
    from mlx_gptq_b200.artifacts import ArtifactReader, ArtifactWriter

    header = {"mode": "mxfp4", "bits": 4, "group_size": 32, "storage_dtype": "bfloat16"}
    outs = {}
    for fwd in ("eager", "grouped"):
        model = sequential.build_model(TINY)
        pipe = sequential.Pipeline(model, sequential.SyntheticWeights(model, "cuda:0", seed=0), _args(
            experts_forward=fwd))
        assert pipe.grouped_experts == (2 if fwd == "grouped" else 0)
        outs[fwd] = pipe.run(_samples(), ArtifactWriter(str(tmp_path / fwd), header))
    for (a, _), (b, _) in zip(outs["eager"], outs["grouped"]):
        assert torch.equal(a, b)
    ra, rb = ArtifactReader(str(tmp_path / "eager")), ArtifactReader(str(tmp_path / "grouped"))
    assert set(ra.tensors) == set(rb.tensors)
    for name in ra.tensors:
        qa, sa, _, ia = ra.get(name)
        qb, sb, _, ib = rb.get(name)
        assert torch.equal(qa, qb) and torch.equal(sa, sb) and ia == ib, name


@pytest.mark.parametrize("tokens", [4096, 1000])
def test_grouped_forward_bit_identical_at_qwen3_30b_a3b_shapes(tokens):
    """Hidden 2048, 128 experts of intermediate 768, top-8: the sort-based forward
    (grouped GEMM launches) equals the eager per-expert loop bit for bit."""
    from transformers import AutoConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeExperts

    from mlx_gptq_b200.experts import grouped_experts_forward

    cfg = AutoConfig.for_model("qwen3_moe", hidden_size=2048, moe_intermediate_size=768, num_experts=128,
                               num_experts_per_tok=8)
    cfg._experts_implementation = "eager"
    g = torch.Generator(device="cuda").manual_seed(7)
    m = Qwen3MoeExperts(cfg).to("cuda", torch.bfloat16)
    with torch.no_grad():
        m.gate_up_proj.copy_(torch.randn(m.gate_up_proj.shape, generator=g, device="cuda") * 0.02)
        m.down_proj.copy_(torch.randn(m.down_proj.shape, generator=g, device="cuda") * 0.02)
        x = torch.randn(tokens, 2048, generator=g, device="cuda").to(torch.bfloat16)
        logits = torch.randn(tokens, 128, generator=g, device="cuda")
        logits[:, :4] += 3.0  # skewed routing, some experts see few or no tokens
        w, idx = torch.softmax(logits, -1).topk(8, dim=-1)
        w = (w / w.sum(-1, keepdim=True)).to(torch.bfloat16)
        ref = m(x, idx, w)
        got = grouped_experts_forward(m, x, idx, w)
    assert torch.equal(ref, got)
