"""The Stage A command line on the GPU over a tiny on-disk Qwen3-MoE checkpoint
(per-expert safetensors as Hugging Face ships them): artifacts for every linear and
expert, in the reference's format, valid codes, a sane rel_err, and a resumed run
that leaves the manifest unchanged."""

import json
import os

import numpy as np
import pytest
import torch

from test_calibrate_cpu import TINY, write_tiny_checkpoint

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["mxfp4", "affine"])
def test_cli_end_to_end(mode, tmp_path):
    from mlx_gptq_b200 import calibrate
    from mlx_gptq_b200.artifacts import ArtifactReader
    from mlx_gptq_b200.grid import dequantize_artifact

    cfg = dict(TINY, hidden_size=128, moe_intermediate_size=64, head_dim=32)
    model_dir = write_tiny_checkpoint(str(tmp_path / "model"), cfg)
    toks = tmp_path / "t.npy"
    np.save(toks, np.random.default_rng(1).integers(0, cfg["vocab_size"], (8, 64)).astype(np.int64))
    out = str(tmp_path / "out")
    argv = ["--model", model_dir, "--output", out, "--calibration-tokens", str(toks), "--mode", mode,
            "--devices", "cuda:0", "--batch-size", "4"]
    if mode == "affine":
        argv += ["--group-size", "64", "--override", r".*down_proj.*=8"]
    calibrate.main(argv)
    man = json.load(open(os.path.join(out, "manifest.json")))
    assert man["layers_done"] == [0, 1]
    assert len(man["tensors"]) == 2 * (4 + 3 * 8)
    reader = ArtifactReader(out)
    for name, info in man["tensors"].items():
        q, s, b, info = reader.get(name)
        bits = info["bits"]
        if mode == "affine" and ".down_proj." in name:
            assert bits == 8
        assert int(q.max()) < (1 << bits) and (b is None) == (mode != "affine")
        assert 0.0 < info["rel_err"] < 0.5, (name, info["rel_err"])
        dq = dequantize_artifact(q.cuda(), s.cuda(), None if b is None else b.cuda(), mode, info["group_size"])
        assert torch.isfinite(dq).all()
    before = open(os.path.join(out, "manifest.json")).read()
    calibrate.main(argv)
    assert open(os.path.join(out, "manifest.json")).read() == before
