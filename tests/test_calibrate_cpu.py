"""Stage A command line (mlx_gptq_b200.calibrate): flag rules, budgets, data windows,
checkpoint prefixes, and a CPU run over a tiny on-disk Qwen3-MoE checkpoint with the
GPU pieces replaced by deterministic stand-ins (reference tests: test_vram_budgets.py,
test_prefix_mapping.py; calibrate.py:97-293)."""

import json
import os
import types

import numpy as np
import pytest
import torch

from mlx_gptq_b200 import calibrate, sequential

TINY = dict(model_type="qwen3_moe", vocab_size=512, hidden_size=64, intermediate_size=128, moe_intermediate_size=32,
            num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=16, num_experts=8,
            num_experts_per_tok=2, decoder_sparse_step=1, norm_topk_prob=True, max_position_embeddings=256)


def test_single_budget_is_broadcast_to_all_devices():
    assert calibrate.parse_vram_budgets("12", ["cuda:0", "cuda:1"]) == {"cuda:0": 12.0, "cuda:1": 12.0}


def test_per_device_budgets_preserve_heterogeneous_capacity():
    assert calibrate.parse_vram_budgets("4.2,18.6,83.4", ["cuda:0", "cuda:1", "cuda:2"]) == {
        "cuda:0": 4.2, "cuda:1": 18.6, "cuda:2": 83.4}


def test_per_device_budget_count_must_match():
    with pytest.raises(ValueError, match="one comma-separated value per device"):
        calibrate.parse_vram_budgets("4,8", ["cuda:0", "cuda:1", "cuda:2"])
    with pytest.raises(ValueError, match="positive"):
        calibrate.parse_vram_budgets("0", ["cuda:0"])


def _resolve(argv):
    return calibrate.resolve_args(calibrate.build_parser(), argv)


def test_mode_rules():
    base = ["--model", "m", "--output", "o", "--calibration-tokens", "t.npy", "--devices", "cpu"]
    a = _resolve(base + ["--mode", "mxfp4"])
    assert (a.group_size, a.bits, a.mxfp_algorithm) == (32, 4, "safe-scale-search")
    a = _resolve(base + ["--mode", "mxfp8"])
    assert (a.group_size, a.bits, a.mxfp_algorithm) == (32, 8, "groupwise")
    a = _resolve(base + ["--mode", "affine", "--override", ".*down_proj.*=8"])
    assert (a.group_size, a.bits, a.mxfp_algorithm) == (64, 4, "none")
    assert a.overrides[0][0].search("mlp.down_proj.weight") and a.overrides[0][1] == 8
    assert a.vram_gb == {"cpu": 16.0}
    assert _resolve(base + ["--lazy-ple"]).lazy_ple
    for bad in (["--mode", "mxfp4", "--bits", "8"], ["--mode", "mxfp8", "--group-size", "64"],
                ["--mode", "mxfp4", "--override", "x=8"]):
        with pytest.raises(SystemExit):
            _resolve(base + bad)
    with pytest.raises(SystemExit):
        _resolve(["--model", "m", "--output", "o"])  # neither --dataset nor --calibration-tokens


class _Tok:
    """Whitespace tokenizer: word i of a fixed vocabulary -> id i."""
    eos_token_id = 0

    def __call__(self, text, add_special_tokens=False):
        return types.SimpleNamespace(input_ids=[1 + (hash(w) % 400) for w in text.split()])

    def __len__(self):
        return 512


def test_load_calibration_windows(tmp_path):
    txt = tmp_path / "a.txt"
    txt.write_text(" ".join(f"w{i}" for i in range(3000)))
    jl = tmp_path / "b.jsonl"
    jl.write_text("\n".join(json.dumps({"body": " ".join(f"v{i}" for i in range(500))}) for _ in range(3)))
    s = calibrate.load_calibration(_Tok(), f"{txt},{jl}:body", nsamples=8, seqlen=128, seed=3)
    assert s.shape == (8, 128) and s.dtype == torch.int64
    s2 = calibrate.load_calibration(_Tok(), f"{txt},{jl}:body", nsamples=8, seqlen=128, seed=3)
    assert torch.equal(s, s2)
    with pytest.raises(ValueError, match="offline"):
        calibrate.load_calibration(_Tok(), "hf:wikitext", 1, 8)
    with pytest.raises(ValueError, match="tokens < seqlen"):
        calibrate.load_calibration(_Tok(), str(txt), 1, 5000)


def test_multimodal_checkpoint_prefixes_are_independent():
    class Backbone(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = torch.nn.ModuleList([torch.nn.Linear(4, 4, bias=False)])

    class Runtime(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.model = Backbone()

    args = types.SimpleNamespace(devices=["cpu"], dtype="bfloat16", layers_attr="model.layers",
                                 checkpoint_model_prefix="model.language_model",
                                 artifact_layers_prefix="language_model.model.layers")
    p = sequential.Pipeline(Runtime(), shards=None, args=args)
    assert p._checkpoint_name("model.embed_tokens") == "model.language_model.embed_tokens"
    assert p.checkpoint_layers_prefix_fmt.format(7) == "model.language_model.layers.7"
    assert p.artifact_layers_prefix_fmt.format(7) == "language_model.model.layers.7"


def write_tiny_checkpoint(path, cfg=TINY, seed=0):
    from golden.make_stack_golden import write_checkpoint

    return write_checkpoint(path, cfg, seed)


def test_cli_runs_and_resumes_on_cpu(tmp_path, monkeypatch):
    import test_pipeline_cpu as fakes

    from mlx_gptq_b200 import artifacts, grid, pipeline

    from mlx_gptq_b200 import capture

    for mod, name, fn in ((pipeline, "_solve_batch", fakes._fake_solve),
                          (pipeline, "dequantize_artifact", fakes._fake_dequant),
                          (pipeline, "pack_nibbles", fakes._fake_pack), (pipeline, "unpack_nibbles", fakes._fake_unpack),
                          (pipeline, "hessian_tile_count", fakes._fake_tile_count),
                          (artifacts, "pack_nibbles", fakes._fake_pack), (artifacts, "unpack_nibbles", fakes._fake_unpack),
                          (grid, "dequantize_artifact", fakes._fake_dequant),
                          (capture.CaptureManager, "expert_hessians", fakes._fake_expert_hessians),
                          (capture.Stash, "hessian", fakes._fake_stash_hessian)):
        monkeypatch.setattr(mod, name, fn)
    model_dir = write_tiny_checkpoint(str(tmp_path / "model"))
    toks = tmp_path / "t.npy"
    np.save(toks, np.random.default_rng(1).integers(0, 512, (4, 32)).astype(np.int64))
    out = str(tmp_path / "out")
    argv = ["--model", model_dir, "--output", out, "--calibration-tokens", str(toks), "--mode", "mxfp4",
            "--devices", "cpu", "--batch-size", "2"]
    calibrate.main(argv)
    man = json.load(open(os.path.join(out, "manifest.json")))
    assert man["layers_done"] == [0, 1] and man["mode"] == "mxfp4" and man["algorithm"] == "safe-scale-search"
    assert man["nsamples"] == 4 and man["seqlen"] == 32 and len(man["calibration_tokens_sha256"]) == 64
    names = set(man["tensors"])
    assert "model.layers.1.self_attn.o_proj.weight" in names
    assert "model.layers.0.mlp.experts.7.down_proj.weight" in names and len(names) == 2 * (4 + 3 * 8)
    assert os.path.exists(os.path.join(out, "calib_tokens.npy"))
    before = open(os.path.join(out, "manifest.json")).read()
    calibrate.main(argv)  # every layer resumes from its artifacts
    assert open(os.path.join(out, "manifest.json")).read() == before
    bad = tmp_path / "bad.npy"
    np.save(bad, np.full((2, 8), 999, np.int64))
    with pytest.raises(ValueError, match="exceed vocabulary"):
        calibrate.main(["--model", model_dir, "--output", str(tmp_path / "o2"), "--calibration-tokens", str(bad),
                        "--devices", "cpu"])


def _write_tokenizer(model_dir, vocab_size=300):
    """A word-level tokenizer (w2 .. w{n-1}, [UNK] = 0, </s> = 1) saved the Hugging Face way."""
    from tokenizers import Tokenizer, models, pre_tokenizers

    vocab = {"[UNK]": 0, "</s>": 1, **{f"w{i}": i for i in range(2, vocab_size)}}
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.save(os.path.join(model_dir, "tokenizer.json"))
    with open(os.path.join(model_dir, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": "</s>", "unk_token": "[UNK]"}, f)


def test_cli_dataset_path_with_the_model_tokenizer(tmp_path, monkeypatch):
    """--dataset: documents tokenized by the model's own tokenizer, joined with EOS and cut
    into windows (data.py:load_calibration), saved as calib_tokens.npy and hashed into the
    manifest; token ids are checked against the tokenizer's vocabulary."""
    import test_pipeline_cpu as fakes

    from mlx_gptq_b200 import artifacts, capture, grid, pipeline

    fakes.install_fakes(pipeline, capture, monkeypatch.setattr)
    for mod, name, fn in ((artifacts, "pack_nibbles", fakes._fake_pack), (artifacts, "unpack_nibbles", fakes._fake_unpack),
                          (grid, "dequantize_artifact", fakes._fake_dequant)):
        monkeypatch.setattr(mod, name, fn)
    model_dir = write_tiny_checkpoint(str(tmp_path / "model"))
    _write_tokenizer(model_dir)
    text = tmp_path / "corpus.txt"
    rng = np.random.default_rng(0)
    text.write_text(" ".join(f"w{i}" for i in rng.integers(2, 300, 4000)))
    out = str(tmp_path / "out")
    calibrate.main(["--model", model_dir, "--output", out, "--dataset", str(text), "--nsamples", "4",
                    "--seqlen", "32", "--mode", "mxfp4", "--devices", "cpu", "--batch-size", "2", "--seed", "3"])
    toks = np.load(os.path.join(out, "calib_tokens.npy"))
    assert toks.shape == (4, 32) and toks.min() >= 1 and toks.max() < 300
    man = json.load(open(os.path.join(out, "manifest.json")))
    assert man["dataset"] == str(text) and man["nsamples"] == 4 and man["layers_done"] == [0, 1]
    import hashlib

    assert man["calibration_tokens_sha256"] == hashlib.sha256(open(os.path.join(out, "calib_tokens.npy"),
                                                                   "rb").read()).hexdigest()


def test_validate_artifacts_report(tmp_path, monkeypatch):
    """validate_artifacts.py:21-76: a clean run verifies; a corrupted scale (range blow-up),
    a tensor missing from the checkpoint and a shape mismatch are reported as failures."""
    import safetensors.torch as st

    import test_pipeline_cpu as fakes

    from mlx_gptq_b200 import artifacts, capture, grid, pipeline, validate

    fakes.install_fakes(pipeline, capture, monkeypatch.setattr)
    for mod, name, fn in ((artifacts, "pack_nibbles", fakes._fake_pack), (artifacts, "unpack_nibbles", fakes._fake_unpack),
                          (grid, "dequantize_artifact", fakes._fake_dequant),
                          (validate, "dequantize_artifact", fakes._fake_dequant)):
        monkeypatch.setattr(mod, name, fn)
    model_dir = write_tiny_checkpoint(str(tmp_path / "model"))
    toks = tmp_path / "t.npy"
    np.save(toks, np.random.default_rng(1).integers(0, 512, (4, 32)).astype(np.int64))
    out = str(tmp_path / "out")
    calibrate.main(["--model", model_dir, "--output", out, "--calibration-tokens", str(toks), "--mode", "mxfp4",
                    "--devices", "cpu", "--batch-size", "2"])
    # the fake dequantization is 0.03 * code: scale the source so that is within range
    src = st.load_file(f"{model_dir}/model.safetensors")
    src = {k: (v.float() * 100).to(torch.bfloat16) for k, v in src.items()}
    st.save_file(src, f"{model_dir}/model.safetensors")
    r = validate.validate(model_dir, out, device="cpu")
    assert r["status"] == "verified" and r["tensors"] == 2 * (4 + 3 * 8) and not r["failures"]
    assert len(r["worst"]) == 20 and r["worst"][0]["ratio"] >= r["worst"][-1]["ratio"]

    name = "model.layers.0.self_attn.q_proj.weight"  # artifact far outside its source's range
    src[name] = (src[name].float() * 1e-4).to(torch.bfloat16)
    del src["model.layers.1.self_attn.k_proj.weight"]
    src["model.layers.1.self_attn.v_proj.weight"] = src["model.layers.1.self_attn.v_proj.weight"][:, :32].contiguous()
    st.save_file(src, f"{model_dir}/model.safetensors")
    r = validate.validate(model_dir, out, device="cpu")
    errors = {f["name"]: f["error"] for f in r["failures"]}
    assert r["status"] == "failed"
    assert errors[name].startswith("group range ratio")
    assert errors["model.layers.1.self_attn.k_proj.weight"] == "missing source tensor"
    assert errors["model.layers.1.self_attn.v_proj.weight"].startswith("shape")
    assert validate.main(["--model", model_dir, "--calib", out, "--device", "cpu",
                          "--output", str(tmp_path / "report.json")]) == 1


def _cli_rank(rank, world, port, out_dir, model_dir, toks, dp):
    import os
    import sys

    sys.path.insert(0, os.path.dirname(__file__))
    import test_pipeline_cpu as fakes

    from mlx_gptq_b200 import artifacts, capture, grid, pipeline

    fakes.install_fakes(pipeline, capture)
    artifacts.pack_nibbles, artifacts.unpack_nibbles = fakes._fake_pack, fakes._fake_unpack
    grid.dequantize_artifact = fakes._fake_dequant
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    argv = ["--model", model_dir, "--output", out_dir, "--calibration-tokens", toks, "--mode", "mxfp4",
            "--devices", "cpu", "--batch-size", "2"] + (["--dp-windows"] if dp else [])
    calibrate.main(argv)


@pytest.mark.parametrize("dp", [False, True])
def test_cli_two_processes(tmp_path, dp):
    """The command line under two gloo processes writes one artifact set: identical to one
    process by default; with --dp-windows the same names and layer-0 token counts summed
    over the processes."""
    import socket

    import torch.multiprocessing as mp

    model_dir = write_tiny_checkpoint(str(tmp_path / "model"))
    toks = str(tmp_path / "t.npy")
    np.save(toks, np.random.default_rng(1).integers(0, 512, (4, 32)).astype(np.int64))
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    out2 = str(tmp_path / "out2")
    mp.start_processes(_cli_rank, args=(2, port, out2, model_dir, toks, dp), nprocs=2, start_method="spawn")
    # one process, same fakes, in a fresh child (the fakes stay out of this test process)
    out1 = str(tmp_path / "out1")
    mp.start_processes(_cli_rank, args=(1, port + 1, out1, model_dir, toks, False), nprocs=1,
                       start_method="spawn")
    m1 = json.load(open(os.path.join(out1, "manifest.json")))
    m2 = json.load(open(os.path.join(out2, "manifest.json")))
    assert m1["layers_done"] == m2["layers_done"] == [0, 1]
    assert sorted(m1["tensors"]) == sorted(m2["tensors"])
    # with --dp-windows layer 0's counts are sums over the processes; later layers see
    # weights solved from these stand-in Hessians, which are not sums over processes
    layers = ("model.layers.0.",) if dp else ("model.layers.",)
    assert ({k: v["tokens"] for k, v in m1["tensors"].items() if k.startswith(layers)}
            == {k: v["tokens"] for k, v in m2["tensors"].items() if k.startswith(layers)})
    if not dp:
        import safetensors.torch as st

        for li in (0, 1):
            a = st.load_file(os.path.join(out1, f"layer_{li:04d}.safetensors"))
            b = st.load_file(os.path.join(out2, f"layer_{li:04d}.safetensors"))
            assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)


def test_cli_spreads_experts_over_every_listed_device(tmp_path, monkeypatch):
    """--devices with several entries in one process (the reference's multi-device mode,
    sequential.py:471-474, 610-626): every fused task's experts go to a worker thread per
    device and the artifacts equal a one-device run's. Two host "devices" stand in for
    GPUs, with the fake solver."""
    import safetensors.torch as st
    import test_pipeline_cpu as fakes

    from mlx_gptq_b200 import artifacts, capture, grid, pipeline

    fakes.install_fakes(pipeline, capture, monkeypatch.setattr)
    for mod, name, fn in ((artifacts, "pack_nibbles", fakes._fake_pack), (artifacts, "unpack_nibbles", fakes._fake_unpack),
                          (grid, "dequantize_artifact", fakes._fake_dequant)):
        monkeypatch.setattr(mod, name, fn)
    calls = []
    real = pipeline.solve_experts_on_devices

    def spy(mgr, task, experts, devices, *a, **k):
        calls.append((task.param_name, len(experts), [str(d) for d in devices]))
        return real(mgr, task, experts, devices, *a, **k)

    monkeypatch.setattr(pipeline, "solve_experts_on_devices", spy)
    model_dir = write_tiny_checkpoint(str(tmp_path / "model"))
    toks = tmp_path / "t.npy"
    np.save(toks, np.random.default_rng(1).integers(0, 512, (4, 32)).astype(np.int64))
    outs = {}
    for devs in ("cpu", "cpu,cpu"):
        out = str(tmp_path / devs.replace(",", "_"))
        calibrate.main(["--model", model_dir, "--output", out, "--calibration-tokens", str(toks), "--mode", "mxfp4",
                        "--devices", devs, "--batch-size", "2"])
        outs[devs] = out
    assert calls and all(d == ["cpu", "cpu"] and n == 8 for _, n, d in calls)
    for li in (0, 1):
        a = st.load_file(os.path.join(outs["cpu"], f"layer_{li:04d}.safetensors"))
        b = st.load_file(os.path.join(outs["cpu,cpu"], f"layer_{li:04d}.safetensors"))
        assert sorted(a) == sorted(b) and all(torch.equal(a[k], b[k]) for k in a)
