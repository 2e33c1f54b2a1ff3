"""Golden artifacts of the REAL reference's layer-sequential Stage A on CPU.

Runs mlx_gptq.sequential.Pipeline (the reference's own capture, Hessians,
solve_gptq, artifact writer) over a tiny seeded Qwen3-MoE checkpoint and stores
its per-tensor codes, scales, rel_err and token counts in stack_mxfp4.npz; then runs
the reference's Stage B streaming packer (mlx_gptq/stream_pack.py) on those
artifacts, as they are and without one stacked projection's artifacts (RTN fallback), and
stores a summary of each MLX output (dtype, shape and sha256 of every tensor, the
index's weight map, the config's quantization entry):

    python tests/golden/make_stack_golden.py [--ref PATH_TO_REFERENCE_CHECKOUT]

The checkpoint is not stored: write_checkpoint() regenerates it bit for bit from
its seed (CPU generators), in this container and on a GPU box, so the tests run
their own pipeline on the same weights and windows and compare with the fixture.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import tempfile
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "mlx-gptq-mxfp_b200"))

STACK_CONFIG = dict(model_type="qwen3_moe", vocab_size=512, hidden_size=128, intermediate_size=256,
                    moe_intermediate_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                    head_dim=32, num_experts=8, num_experts_per_tok=2, decoder_sparse_step=1, norm_topk_prob=True,
                    max_position_embeddings=256)
WINDOWS_SEED, N_WINDOWS, SEQLEN, BATCH = 1, 8, 64, 4


def write_checkpoint(path: str, cfg: dict = STACK_CONFIG, seed: int = 0) -> str:
    """config.json + model.safetensors (per-expert tensors, as Hugging Face ships them),
    weights from mlx_gptq_b200.sequential.SyntheticWeights on the CPU, stored in bf16."""
    from safetensors.torch import save_file

    from mlx_gptq_b200 import sequential

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    model = sequential.build_model(dict(cfg))
    src = sequential.SyntheticWeights(model, "cpu", seed=seed)
    tensors = {}
    for name in src.shapes:
        t = src.get(name).to(torch.bfloat16)
        if name.endswith(("experts.gate_up_proj", "experts.down_proj")):
            base, kind = name.rsplit(".", 1)
            for e in range(t.shape[0]):
                if kind == "gate_up_proj":
                    half = t.shape[1] // 2
                    tensors[f"{base}.{e}.gate_proj.weight"] = t[e, :half].contiguous()
                    tensors[f"{base}.{e}.up_proj.weight"] = t[e, half:].contiguous()
                else:
                    tensors[f"{base}.{e}.down_proj.weight"] = t[e].contiguous()
        else:
            tensors[name] = t.contiguous()
    save_file(tensors, os.path.join(path, "model.safetensors"))
    return path


def windows() -> np.ndarray:
    return np.random.default_rng(WINDOWS_SEED).integers(0, STACK_CONFIG["vocab_size"],
                                                        (N_WINDOWS, SEQLEN)).astype(np.int64)


def _json_bytes(obj) -> np.ndarray:
    return np.frombuffer(json.dumps(obj, sort_keys=True).encode(), dtype=np.uint8)


def packed_summary(mlx_dir: str) -> dict:
    """Every tensor of an MLX output directory as [dtype, shape, sha256 of its bytes], plus
    its index's weight map (file per key) and the quantization entry of its config."""
    import hashlib

    from safetensors import safe_open

    tensors = {}
    index = json.load(open(os.path.join(mlx_dir, "model.safetensors.index.json")))
    for fname in sorted(set(index["weight_map"].values())):
        with safe_open(os.path.join(mlx_dir, fname), framework="pt") as f:
            for k in f.keys():
                t = f.get_tensor(k).contiguous()
                raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
                tensors[k] = [str(t.dtype), list(t.shape), hashlib.sha256(raw).hexdigest()]
    cfg = json.load(open(os.path.join(mlx_dir, "config.json")))
    return {"tensors": tensors, "weight_map": index["weight_map"], "quantization": cfg["quantization"]}


def run_reference_packer(model_dir: str, calib: str, mlx_dir: str) -> dict:
    from mlx_gptq.stream_pack import StreamingPacker

    StreamingPacker(model_dir, calib, mlx_dir, "mxfp4", 4, 32,
                    r"(^|\.)(gate|router)$|shared_expert_gate|e_score|(^|\.)ple($|\.)").run()
    return packed_summary(mlx_dir)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GQ_REFERENCE"),
                    help="reference checkout (or set GQ_REFERENCE)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref (or GQ_REFERENCE) must point at the reference checkout")
    sys.path.insert(0, a.ref)
    from mlx_gptq.artifacts import ArtifactReader, ArtifactWriter
    from mlx_gptq.sequential import DEFAULT_EXCLUDE, Pipeline, RawShardIndex

    from mlx_gptq_b200 import sequential

    torch.manual_seed(0)
    scratch = os.path.join(ROOT, "_build")  # git-ignored build scratch
    os.makedirs(scratch, exist_ok=True)
    with tempfile.TemporaryDirectory(dir=scratch) as tmp:
        model_dir = write_checkpoint(os.path.join(tmp, "model"))
        out = os.path.join(tmp, "out")
        args = types.SimpleNamespace(devices=["cpu"], dtype="bfloat16", layers_attr="model.layers",
                                     checkpoint_model_prefix=None, artifact_layers_prefix=None, batch_size=BATCH,
                                     exclude=DEFAULT_EXCLUDE, group_size=32, bits=4, mode="mxfp4",
                                     mxfp_algorithm="safe-scale-search", damp=0.01, clip="mse", overrides=[],
                                     vram_gb={"cpu": 16.0}, lazy_ple=False)
        model = sequential.build_model(dict(STACK_CONFIG))  # meta skeleton, eager experts
        writer = ArtifactWriter(out, {"mode": "mxfp4", "bits": 4, "group_size": 32, "storage_dtype": "bfloat16"})
        with torch.no_grad():
            Pipeline(model, RawShardIndex(model_dir), args).run(torch.from_numpy(windows()), writer)
        reader = ArtifactReader(out)
        fx, meta = {}, {}
        fx["packed"] = _json_bytes(run_reference_packer(model_dir, out, os.path.join(tmp, "mlx")))
        # the same without layer 1's down_proj artifacts: that stacked switch_mlp tensor
        # falls back to RTN (the packer requires every remaining artifact to be used)
        drop = [n for n in reader.tensors if n.startswith("model.layers.1.mlp.experts.") and
                n.endswith(".down_proj.weight")]
        out_rtn = os.path.join(tmp, "out_rtn")
        shutil.copytree(out, out_rtn)
        man = json.load(open(os.path.join(out_rtn, "manifest.json")))
        for n in drop:
            del man["tensors"][n]
        json.dump(man, open(os.path.join(out_rtn, "manifest.json"), "w"))
        fx["packed_rtn"] = _json_bytes(run_reference_packer(model_dir, out_rtn, os.path.join(tmp, "mlx_rtn")))
        fx["packed_rtn_dropped"] = _json_bytes(sorted(drop))
        for name, info in sorted(reader.tensors.items()):
            q, s, b, info = reader.get(name)
            fx[f"q:{name}"] = q.numpy().astype(np.uint8)
            fx[f"s:{name}"] = s.numpy().astype(np.uint8)
            meta[name] = {"rel_err": info["rel_err"], "tokens": info["tokens"], "kind": info["kind"]}
        fx["meta"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
        np.savez_compressed(os.path.join(HERE, "stack_mxfp4.npz"), **fx)
        print(f"stack_mxfp4.npz: {len(meta)} tensors")


if __name__ == "__main__":
    main()
