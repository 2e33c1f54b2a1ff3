"""Layer-sequential driver host logic (CPU, no kernels).

Mirrors what the reference's tests/test_sequential_context.py pins (checkpoint
buffers materialized, per-layer positional/keyword call contexts preserved with
shared containers) and runs a tiny Qwen3-MoE skeleton end to end with the GPU
solver replaced by a deterministic fake: artifact names and metadata follow the
reference, and a 2-rank gloo run equals the single-process run.
"""

import os
import types

import pytest
import torch

from mlx_gptq_b200 import sequential
from mlx_gptq_b200.sequential import Pipeline, SyntheticWeights, materialize_module

TINY_QWEN3_MOE = dict(model_type="qwen3_moe", vocab_size=512, hidden_size=64, intermediate_size=128,
                      moe_intermediate_size=32, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=16, num_experts=8, num_experts_per_tok=2, decoder_sparse_step=1, norm_topk_prob=True,
                      max_position_embeddings=256)


class ContextLayer(torch.nn.Module):
    def __init__(self, layer_idx, observations):
        super().__init__()
        self.layer_idx = layer_idx
        self.observations = observations

    def forward(self, hidden_states, per_layer_input, shared_state, layer_tag):
        self.observations.append((self.layer_idx, per_layer_input.clone(), layer_tag, dict(shared_state)))
        shared_state[self.layer_idx] = layer_tag
        return hidden_states + per_layer_input


class ContextModel(torch.nn.Module):
    def __init__(self, observations):
        super().__init__()
        self.embed_tokens = torch.nn.Embedding(16, 4)
        self.layers = torch.nn.ModuleList([ContextLayer(0, observations), ContextLayer(1, observations)])

    def get_input_embeddings(self):
        return self.embed_tokens

    def forward(self, input_ids, use_cache=False):
        h = self.embed_tokens(input_ids)
        shared = {}
        for i, layer in enumerate(self.layers):
            h = layer(h, torch.full_like(h, i + 1), shared_state=shared, layer_tag=f"layer-{i}")
        return h


class FakeShards:
    def __init__(self, tensors):
        self.tensors = tensors

    def has(self, name):
        return name in self.tensors

    def get(self, name):
        return self.tensors[name]


def _args(**kw):
    base = dict(devices=["cpu"], dtype="bfloat16", layers_attr="model.layers", checkpoint_model_prefix=None,
                artifact_layers_prefix=None, exclude=sequential.DEFAULT_EXCLUDE, group_size=32, bits=4,
                mode="mxfp4", mxfp_algorithm="safe-scale-search", damp=0.01, clip="mse", overrides=[],
                batch_size=2)
    base.update(kw)
    return types.SimpleNamespace(**base)


def test_materialize_module_loads_non_meta_checkpoint_buffers():
    module = torch.nn.Linear(2, 2, bias=False, device="meta")
    module.register_buffer("layer_scalar", torch.ones(1))
    materialize_module(module, "layer", FakeShards({"layer.weight": torch.eye(2),
                                                   "layer.layer_scalar": torch.tensor([3.0])}),
                       "cpu", torch.bfloat16)
    assert module.weight.device.type == "cpu" and module.weight.dtype == torch.bfloat16
    assert module.layer_scalar.item() == 3.0


def test_materialize_fuses_per_expert_checkpoint_tensors():
    class Experts(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_up_proj = torch.nn.Parameter(torch.empty(3, 4, 2, device="meta"))
            self.down_proj = torch.nn.Parameter(torch.empty(3, 2, 2, device="meta"))

    m = Experts()
    raw = {}
    for e in range(3):
        raw[f"x.{e}.gate_proj.weight"] = torch.full((2, 2), float(e))
        raw[f"x.{e}.up_proj.weight"] = torch.full((2, 2), 10.0 + e)
        raw[f"x.{e}.down_proj.weight"] = torch.full((2, 2), 20.0 + e)
    # parameters live directly on the module: prefix "x" and names "gate_up_proj"/"down_proj"
    wrapper = torch.nn.Module()
    wrapper.experts = m
    raw = {k.replace("x.", "w.experts.", 1): v for k, v in raw.items()}
    materialize_module(wrapper, "w", FakeShards(raw), "cpu", torch.float32)
    for e in range(3):
        assert (m.gate_up_proj[e, :2] == e).all() and (m.gate_up_proj[e, 2:] == 10 + e).all()
        assert (m.down_proj[e] == 20 + e).all()
    with pytest.raises(KeyError):
        materialize_module(torch.nn.Linear(2, 2, device="meta"), "missing", FakeShards({}), "cpu", torch.float32)


def test_capture_preserves_positional_and_per_layer_context(monkeypatch):
    observations = []
    model = ContextModel(observations)
    pipe = Pipeline(model, shards=None, args=_args(layers_attr="layers"))
    monkeypatch.setattr(sequential, "materialize_module", lambda *a, **k: None)
    monkeypatch.setattr(sequential, "free_module", lambda *a, **k: None)
    batches = pipe.catch_layer0_inputs(torch.tensor([[1, 2, 3]]), batch_size=1)
    assert observations == [] and len(batches) == 1
    hidden, contexts = batches[0]
    assert len(contexts) == 2
    assert torch.equal(contexts[0][0][0], torch.ones_like(hidden))
    assert torch.equal(contexts[1][0][0], torch.full_like(hidden, 2))
    assert contexts[0][1]["layer_tag"] == "layer-0" and contexts[1][1]["layer_tag"] == "layer-1"
    assert contexts[0][1]["shared_state"] is contexts[1][1]["shared_state"]
    for i, layer in enumerate(model.layers):
        batches[0] = (pipe.forward_layer(layer, batches, i)[0], contexts)
    assert [o[2] for o in observations] == ["layer-0", "layer-1"]
    assert observations[0][3] == {} and observations[1][3] == {0: "layer-0"}
    assert torch.allclose(batches[0][0].float(), hidden.float() + 3, atol=0.02, rtol=0)


def test_synthetic_weights_are_seeded_per_name():
    model = sequential.build_model(TINY_QWEN3_MOE)
    a, b = SyntheticWeights(model, "cpu", seed=0), SyntheticWeights(model, "cpu", seed=0)
    c = SyntheticWeights(model, "cpu", seed=1)
    name = "model.layers.0.mlp.experts.gate_up_proj"
    assert a.has(name) and a.get(name).shape == (8, 64, 64)
    assert torch.equal(a.get(name), b.get(name)) and not torch.equal(a.get(name), c.get(name))
    assert not torch.equal(a.get(name), a.get("model.layers.1.mlp.experts.gate_up_proj"))
    assert (a.get("model.layers.0.input_layernorm.weight") == 1).all()
    assert abs(float(a.get(name).std()) - 0.02) < 0.002
    assert not a.has("model.rotary_emb.inv_freq")  # real buffer, kept


def _fake_solver(monkeypatch):
    import test_pipeline_cpu as fakes

    from mlx_gptq_b200 import capture, pipeline

    monkeypatch.setattr(pipeline, "_solve_batch", fakes._fake_solve)
    monkeypatch.setattr(pipeline, "dequantize_artifact", fakes._fake_dequant)
    monkeypatch.setattr(pipeline, "pack_nibbles", fakes._fake_pack)
    monkeypatch.setattr(pipeline, "unpack_nibbles", fakes._fake_unpack)
    monkeypatch.setattr(pipeline, "hessian_tile_count", fakes._fake_tile_count)
    monkeypatch.setattr(pipeline, "hessian_tiles_per_wave", fakes._fake_tiles_per_wave)
    monkeypatch.setattr(capture.CaptureManager, "expert_hessians", fakes._fake_expert_hessians)
    monkeypatch.setattr(capture.Stash, "hessian", fakes._fake_stash_hessian)


class _Writer:
    def __init__(self):
        self.layers = {}

    def layer_done(self, i):
        return False

    def write_layer(self, i, tensors, meta):
        self.layers[i] = (tensors, meta)


def test_tiny_qwen3_moe_stack_names_and_stats(monkeypatch):
    _fake_solver(monkeypatch)
    model = sequential.build_model(TINY_QWEN3_MOE)
    pipe = Pipeline(model, SyntheticWeights(model, "cpu", seed=0), _args())
    samples = torch.randint(0, 512, (4, 32), generator=torch.Generator().manual_seed(1))
    w = _Writer()
    pipe.run(samples, w)
    assert sorted(w.layers) == [0, 1]
    tensors, meta = w.layers[0]
    names = set(meta)
    for p in ("q_proj", "k_proj", "v_proj", "o_proj"):
        assert f"model.layers.0.self_attn.{p}.weight" in names
    for e in range(8):
        for p in ("gate_proj", "up_proj", "down_proj"):
            assert f"model.layers.0.mlp.experts.{e}.{p}.weight" in names
    assert not any(".mlp.gate." in n for n in names)  # router excluded
    assert len(names) == 4 + 3 * 8
    assert meta["model.layers.0.mlp.experts.0.gate_proj.weight"]["out_features"] == 32
    assert meta["model.layers.0.mlp.experts.0.down_proj.weight"]["in_features"] == 32
    assert sum(meta[f"model.layers.0.mlp.experts.{e}.gate_proj.weight"]["tokens"] for e in range(8)) >= 4 * 32 * 2
    assert [s.layer for s in pipe.stats] == [0, 1] and pipe.stats[0].experts == 16
    # layers go back to meta after processing
    assert all(p.is_meta for p in model.model.layers[0].parameters())


def _run_stack(rank, world, port, out_dir, setattr_=setattr):
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(__file__))
    from test_pipeline_cpu import install_fakes

    from mlx_gptq_b200 import capture, pipeline

    install_fakes(pipeline, capture, setattr_)
    group = None
    if world > 1:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        group = dist.group.WORLD
    model = sequential.build_model(TINY_QWEN3_MOE)
    pipe = Pipeline(model, SyntheticWeights(model, "cpu", seed=0), _args(), group=group)
    samples = torch.randint(0, 512, (4, 32), generator=torch.Generator().manual_seed(1))
    w = _Writer()
    out = pipe.run(samples, w)
    torch.save({"layers": w.layers, "hidden": [h for h, _ in out]}, os.path.join(out_dir, f"s{world}_{rank}.pt"))
    if world > 1:
        dist.destroy_process_group()


def test_sharded_stack_matches_single_process(tmp_path, monkeypatch):
    import socket

    import torch.multiprocessing as mp

    _run_stack(0, 1, 0, str(tmp_path), monkeypatch.setattr)
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    mp.start_processes(_run_stack, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    ref = torch.load(tmp_path / "s1_0.pt")
    r0 = torch.load(tmp_path / "s2_0.pt")
    r1 = torch.load(tmp_path / "s2_1.pt")
    assert r1["layers"] == {}  # only rank 0 writes
    assert sorted(r0["layers"]) == sorted(ref["layers"])
    for li, (tensors, meta) in ref["layers"].items():
        t2, m2 = r0["layers"][li]
        assert m2 == meta
        for k, (q, s, b) in tensors.items():
            assert torch.equal(q, t2[k][0]) and torch.equal(s, t2[k][1])
    for got in (r0, r1):
        for h, h_ref in zip(got["hidden"], ref["hidden"]):
            assert torch.equal(h, h_ref)


def _tiny_layer(seed=0):
    model = sequential.build_model(TINY_QWEN3_MOE)
    layer = model.model.layers[0]
    materialize_module(layer, "model.layers.0", SyntheticWeights(model, "cpu", seed=seed), "cpu", torch.bfloat16)
    return model, layer


def test_grouped_experts_forward_is_bit_identical_to_eager():
    from mlx_gptq_b200.experts import grouped_experts_forward, install_grouped_experts, route

    _, layer = _tiny_layer()
    experts = layer.mlp.experts
    g = torch.Generator().manual_seed(3)
    x = torch.randn(96, 64, generator=g).to(torch.bfloat16)
    logits = torch.randn(96, 8, generator=g)
    w, idx = torch.softmax(logits, -1).topk(2, dim=-1)
    w = (w / w.sum(-1, keepdim=True)).to(torch.bfloat16)
    idx[:5] = torch.tensor([7, 0])  # ties in expert order across tokens
    with torch.no_grad():
        ref = experts(x, idx, w)
        got = grouped_experts_forward(experts, x, idx, w)
    assert torch.equal(ref, got)
    tok, pos, counts, counts_dev = route(idx, 8)
    assert counts_dev.tolist() == counts
    assert sum(counts) == 96 * 2 and counts == torch.bincount(idx.flatten(), minlength=8).tolist()
    for e in range(8):  # eager row order: torch.where on the [top_k, tokens] mask
        off = sum(counts[:e])
        j_ref, t_ref = torch.where((idx == e).T)
        assert torch.equal(tok[off:off + counts[e]], t_ref) and torch.equal(pos[off:off + counts[e]], j_ref)
    assert install_grouped_experts(layer) == 1


def test_segment_capture_matches_linear_interception():
    from mlx_gptq_b200.capture import CaptureManager
    from mlx_gptq_b200.experts import install_grouped_experts

    def capture(grouped):
        _, layer = _tiny_layer()
        if grouped:
            install_grouped_experts(layer)
        mgr = CaptureManager(layer, sequential.DEFAULT_EXCLUDE, 32)
        g = torch.Generator().manual_seed(5)
        pos = torch.arange(24).unsqueeze(0)
        outs = []
        with mgr, torch.no_grad():
            for _ in range(2):
                mgr.begin_batch()
                h = torch.randn(1, 24, 64, generator=g).to(torch.bfloat16)
                rot = sequential.build_model(TINY_QWEN3_MOE).model.rotary_emb
                cos_sin = rot(h, pos)
                outs.append(layer(h, position_embeddings=cos_sin, attention_mask=None, position_ids=pos))
        return mgr, outs

    m_e, out_e = capture(False)
    m_g, out_g = capture(True)
    for a, b in zip(out_e, out_g):
        a = a[0] if isinstance(a, tuple) else a
        b = b[0] if isinstance(b, tuple) else b
        assert torch.equal(a, b)
    assert m_g._segments and not m_e._segments
    for te, tg in zip(m_e.fused_tasks, m_g.fused_tasks):
        for e in range(te.num_experts):
            assert m_e.stashes[te.stash_keys[e]].tokens == m_g.stashes[tg.stash_keys[e]].tokens
            assert torch.equal(m_e.expert_rows(te, e, "cpu"), m_g.expert_rows(tg, e, "cpu")), (te.param_name, e)
    assert m_e.expert_token_stats() == m_g.expert_token_stats()


def _dp_expert_hessians(self, task, device, experts=None, timer=None):
    """Additive stand-in: H = rows^T rows of the captured rows (float64 -> float32)."""
    experts = list(range(task.num_experts)) if experts is None else list(experts)
    C = task.param.shape[-1]
    out = []
    for e in experts:
        if e is None:
            out.append(torch.zeros(C, C))
            continue
        r = self.expert_rows(task, e, "cpu").double()
        out.append((r.T @ r).float())
    return torch.stack(out)


def _dp_stash_hessian(self, device, chunk_rows=65536, tiles=None):
    r = self.rows("cpu").double()
    return (r.T @ r).float()


def _dp_fake_solve(W, H, bits, args):
    """Codes from W alone; the Hessian reaches the result through rel_err = trace(H),
    which the test compares within the fp32 summation tolerance."""
    B, R, C = W.shape
    q = (W.abs() * 7).round().clamp(0, 15).to(torch.uint8)
    s = torch.full((B, R, C // args.group_size), 3, dtype=torch.uint8)
    import test_pipeline_cpu as fakes

    W_dq = fakes._fake_dequant(q, s, None, args.mode, args.group_size)
    return q, s, None, W_dq, H.diagonal(dim1=-2, dim2=-1).sum(-1)


def _run_dp(rank, world, port, out_dir, setattr_=setattr):
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(__file__))
    from test_pipeline_cpu import install_fakes

    from mlx_gptq_b200 import capture, pipeline

    install_fakes(pipeline, capture, setattr_)
    setattr_(pipeline, "_solve_batch", _dp_fake_solve)
    setattr_(capture.CaptureManager, "expert_hessians", _dp_expert_hessians)
    setattr_(capture.Stash, "hessian", _dp_stash_hessian)
    group = None
    if world > 1:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        group = dist.group.WORLD
    model = sequential.build_model(TINY_QWEN3_MOE)
    pipe = Pipeline(model, SyntheticWeights(model, "cpu", seed=0), _args(), group=group, dp=world > 1)
    samples = torch.randint(0, 512, (8, 32), generator=torch.Generator().manual_seed(1))
    w = _Writer()
    out = pipe.run(samples, w)
    torch.save({"layers": w.layers, "hidden": [h for h, _ in out]}, os.path.join(out_dir, f"dp{world}_{rank}.pt"))
    if world > 1:
        dist.destroy_process_group()


def test_dp_windows_stack_matches_single_process(tmp_path, monkeypatch):
    """Each rank forwards half the windows; summed Hessians and token counts give the
    single-process artifacts and, across the two ranks, the same hidden states."""
    import socket

    import torch.multiprocessing as mp

    _run_dp(0, 1, 0, str(tmp_path), monkeypatch.setattr)
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    mp.start_processes(_run_dp, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    ref = torch.load(tmp_path / "dp1_0.pt")
    r0, r1 = torch.load(tmp_path / "dp2_0.pt"), torch.load(tmp_path / "dp2_1.pt")
    assert r1["layers"] == {}
    for li, (tensors, meta) in ref["layers"].items():
        t2, m2 = r0["layers"][li]
        assert {k: v["tokens"] for k, v in m2.items()} == {k: v["tokens"] for k, v in meta.items()}
        for k, (q, s, b) in tensors.items():
            assert torch.equal(q, t2[k][0]) and torch.equal(s, t2[k][1]), k
            # trace of the summed Hessian == trace of the single-process one (fp32 order)
            assert abs(m2[k]["rel_err"] - meta[k]["rel_err"]) <= 1e-5 * abs(meta[k]["rel_err"]) + 1e-5, k
    hidden = r0["hidden"] + r1["hidden"]
    assert len(hidden) == len(ref["hidden"])
    for a, b in zip(hidden, ref["hidden"]):
        assert torch.equal(a, b)


def test_segment_store_grows_without_a_reservation():
    """Buffers double when no token count is reserved; the rows stay in capture order."""
    from mlx_gptq_b200.capture import SegmentStore

    st = SegmentStore(num_experts=3)
    g = torch.Generator().manual_seed(0)
    ref_in, ref_act, ref_tok = [], [], []
    for T in (5, 9, 17):
        hidden = torch.randn(T, 4, generator=g)
        counts = [T, 0, T]  # 2 slots per token
        tok = torch.cat([torch.arange(T), torch.arange(T)])
        out = st.acts_out(2 * T, T, 6, torch.float32, "cpu")
        acts = torch.randn(2 * T, 6, generator=g)
        out.copy_(acts)
        st.add(hidden, tok, counts, out)
        ref_in.append(hidden)
        ref_act.append(acts)
        ref_tok.append(tok + sum(h.shape[0] for h in ref_in[:-1]))
    assert st.n_tok == 31 and st.n_slot == 62 and st.counts == [31, 0, 31]
    assert torch.equal(st.inputs[:st.n_tok], torch.cat(ref_in))
    assert torch.equal(st.acts[:st.n_slot], torch.cat(ref_act))
    assert torch.equal(st.tok[:st.n_slot].long(), torch.cat(ref_tok))
    assert torch.equal(st.slot_experts("cpu"), torch.cat([torch.tensor([0] * T + [2] * T) for T in (5, 9, 17)]))
    assert st.nbytes() > 0


def test_segment_store_keeps_rows_on_the_stash_device():
    """A store pinned to another device than the forward's declines to lend its buffer
    (the forward keeps its own activations) and receives copies."""
    from mlx_gptq_b200.capture import SegmentStore

    st = SegmentStore(num_experts=2, device="meta")
    assert st.acts_out(4, 2, 3, torch.float32, "cpu") is None
    st2 = SegmentStore(num_experts=2, device="cpu")
    assert st2.acts_out(4, 2, 3, torch.float32, "cpu") is not None


def _ple_checkpoint(tmp_path):
    from safetensors.torch import save_file

    shard_0 = torch.arange(12, dtype=torch.float32).reshape(4, 3)
    shard_1 = shard_0 + 100
    name = "layer.ple.ple_embedding.ngram_embedding.shard_{i}.weight"
    save_file({name.format(i=0): shard_0, name.format(i=1): shard_1}, str(tmp_path / "model.safetensors"))
    wm = {name.format(i=i): "model.safetensors" for i in range(2)}
    (tmp_path / "model.safetensors.index.json").write_text(__import__("json").dumps({"weight_map": wm}))
    return sequential.RawShardIndex(str(tmp_path)), torch.cat([shard_0, shard_1])


def test_lazy_sharded_embedding_reads_selected_rows(tmp_path):
    """tests/test_lazy_ple.py: rows come from the shard that holds them, repeats included."""
    index, table = _ple_checkpoint(tmp_path)
    emb = sequential.LazyShardedEmbedding("layer.ple.ple_embedding.ngram_embedding", index, 2, 4, 3,
                                          torch.device("cpu"), torch.float32)
    ids = torch.tensor([[0, 4, 7], [5, 1, 3], [7, 7, 0]])
    assert torch.equal(emb(ids), table[ids.reshape(-1)].reshape(3, 3, 3))


def test_install_lazy_ple_replaces_the_fused_table(tmp_path):
    index, table = _ple_checkpoint(tmp_path)

    class Ple(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.ple_embedding = torch.nn.Module()
            self.ple_embedding.ngram_embedding = torch.nn.Embedding(8, 3, device="meta")

    layer = torch.nn.Module()
    layer.ple = Ple()
    sequential.install_lazy_ple(layer, "layer", index, "cpu", torch.float32)
    emb = layer.ple.ple_embedding.ngram_embedding
    assert isinstance(emb, sequential.LazyShardedEmbedding) and emb.n_shards == 2 and emb.rows_per_shard == 4
    assert torch.equal(emb(torch.tensor([6, 2])), table[[6, 2]])
    bad = torch.nn.Module()
    bad.ple = Ple()
    bad.ple.ple_embedding.ngram_embedding = torch.nn.Embedding(9, 3, device="meta")
    with pytest.raises(ValueError):
        sequential.install_lazy_ple(bad, "layer", index, "cpu", torch.float32)
