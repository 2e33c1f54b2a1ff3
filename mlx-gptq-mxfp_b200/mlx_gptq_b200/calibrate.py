"""Stage A command line on B200 (mlx_gptq/calibrate.py, same flags).

    python -m mlx_gptq_b200.calibrate --model DIR --output OUT \\
        --calibration-tokens windows.npy --mode mxfp4

Several GPUs, two ways:

    python -m mlx_gptq_b200.calibrate --devices cuda:0,cuda:1,... --model DIR ...
    torchrun --nproc-per-node 8 -m mlx_gptq_b200.calibrate --model DIR ...

The first is the reference's own mode: one process, the layer forward on the first
device, each fused expert parameter's experts spread over every listed device (one
worker thread per device), the plain linears on the first device. The second runs
one process per GPU (the process's GPU is LOCAL_RANK): experts and linears split
over the ranks, one all-gather of the quantized outputs per task. Hugging Face
dataset sources (hf:, hfchat:) need a network and are refused; Flint models are not
supported.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import logging
import os
import re
import shutil

import numpy as np
import torch

log = logging.getLogger("mlx_gptq_b200")


def parse_overrides(specs):
    """calibrate.py:63-68: 'REGEX=BITS' -> [(compiled regex, bits)]."""
    out = []
    for spec in specs or []:
        pattern, _, bits = spec.rpartition("=")
        out.append((re.compile(pattern), int(bits)))
    return out


def parse_vram_budgets(spec: str, devices: list[str]) -> dict[str, float]:
    """calibrate.py:71-82: one budget for every device or one per device (GiB)."""
    values = [float(v.strip()) for v in spec.split(",")]
    if len(values) == 1:
        values *= len(devices)
    if len(values) != len(devices):
        raise ValueError("--vram-gb must be one value or one comma-separated value per device")
    if any(v <= 0 for v in values):
        raise ValueError("--vram-gb values must be positive")
    return dict(zip(devices, values))


def build_parser() -> argparse.ArgumentParser:
    from .grid import SUPPORTED_BITS, SUPPORTED_MODES
    from .sequential import DEFAULT_EXCLUDE

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", required=True, help="local model dir (config.json + safetensors)")
    ap.add_argument("--output", required=True, help="artifact output dir")
    ap.add_argument("--dataset", default=None, help="comma-separated: file.txt | file.jsonl[:field]")
    ap.add_argument("--calibration-tokens", default=None,
                    help="pre-tokenized int64 .npy windows; copied into the artifact receipt")
    ap.add_argument("--nsamples", type=int, default=256)
    ap.add_argument("--seqlen", type=int, default=2048)
    ap.add_argument("--batch-size", type=int, default=4, help="sequences per forward")
    ap.add_argument("--mode", default="affine", choices=SUPPORTED_MODES)
    ap.add_argument("--mxfp-algorithm", default="auto", choices=("auto", "groupwise", "safe-scale-search"))
    ap.add_argument("--bits", type=int, default=None, choices=SUPPORTED_BITS)
    ap.add_argument("--group-size", type=int, default=None, choices=(32, 64, 128))
    ap.add_argument("--clip", default="mse", choices=("mse", "minmax"))
    ap.add_argument("--damp", type=float, default=0.01)
    ap.add_argument("--dtype", default="bfloat16", choices=("bfloat16", "float16"))
    ap.add_argument("--devices", default=None,
                    help="comma-separated; the forward runs on the first, experts are spread over all")
    ap.add_argument("--vram-gb", default="16", help="expert-solve budget in GiB (one value or one per device)")
    ap.add_argument("--layers-attr", default="model.layers")
    ap.add_argument("--checkpoint-model-prefix", default=None)
    ap.add_argument("--artifact-layers-prefix", default=None)
    ap.add_argument("--exclude", default=DEFAULT_EXCLUDE, help="regex of layer-relative names to leave unquantized")
    ap.add_argument("--lazy-ple", action="store_true",
                    help="read per-layer embedding rows from the source shards instead of materializing them")
    ap.add_argument("--override", action="append", metavar="REGEX=BITS", help="per-tensor bit override")
    ap.add_argument("--trust-remote-code", action="store_true")
    ap.add_argument("--seed", type=int, default=17)
    ap.add_argument("--experts-forward", default="grouped", choices=("grouped", "eager"),
                    help="sort-based expert forward (bit-identical to the eager loop) or the eager loop")
    ap.add_argument("--dp-windows", action="store_true",
                    help="with several processes: each forwards its share of the windows and Hessians are "
                         "summed over processes (the forward scales; results match one process within the "
                         "Hessian tolerance instead of bit for bit)")
    return ap


def resolve_args(ap: argparse.ArgumentParser, argv=None):
    """Parse and apply the reference's mode rules (calibrate.py:167-190)."""
    from .grid import mode_defaults

    args = ap.parse_args(argv)
    default_group, default_bits = mode_defaults(args.mode)
    args.group_size = args.group_size or default_group
    args.bits = args.bits or default_bits
    if args.mode in ("mxfp4", "mxfp8"):
        if (args.group_size, args.bits) != (default_group, default_bits):
            ap.error(f"{args.mode} requires --group-size {default_group} and --bits {default_bits}")
        if args.override:
            ap.error("bit overrides are not supported for native MXFP modes")
        if args.mxfp_algorithm == "auto":
            args.mxfp_algorithm = "safe-scale-search" if args.mode == "mxfp4" else "groupwise"
    else:
        args.mxfp_algorithm = "none"
    if args.dataset is None and args.calibration_tokens is None:
        ap.error("one of --dataset or --calibration-tokens is required")
    local = int(os.environ.get("LOCAL_RANK", "-1"))
    if args.devices:
        args.devices = [d.strip() for d in args.devices.split(",")]
    elif torch.cuda.is_available():
        args.devices = [f"cuda:{i}" for i in range(torch.cuda.device_count())]
    else:
        args.devices = ["cpu"]
    try:
        args.vram_gb = parse_vram_budgets(args.vram_gb, args.devices)
    except ValueError as exc:
        ap.error(str(exc))
    if local >= 0 and args.devices[0].startswith("cuda"):  # one process per GPU under torchrun
        dev = f"cuda:{local}"
        args.vram_gb = {dev: args.vram_gb.get(dev, next(iter(args.vram_gb.values())))}
        args.devices = [dev]
    args.overrides = parse_overrides(args.override)
    return args


def _read_source(spec: str) -> list[str]:
    """data.py:_read_source for local files (hf: sources need a network)."""
    if spec.startswith(("hf:", "hfchat:")):
        raise ValueError(f"{spec}: Hugging Face dataset sources are not available offline")
    if ".jsonl" in spec:
        path, _, fld = spec.partition(".jsonl")
        path += ".jsonl"
        fld = fld.lstrip(":") or "text"
        with open(path) as f:
            return [json.loads(line)[fld] for line in f if line.strip()]
    with open(spec) as f:
        return [f.read()]


def load_calibration(tokenizer, sources: str, nsamples: int, seqlen: int, seed: int = 17) -> torch.Tensor:
    """data.py:load_calibration: documents tokenized and joined with EOS, then
    nsamples windows of seqlen tokens (disjoint when the stream allows)."""
    docs = []
    for spec in sources.split(","):
        if spec.strip():
            docs.extend(_read_source(spec.strip()))
    if not docs:
        raise ValueError("no calibration documents loaded")
    eos = tokenizer.eos_token_id
    stream: list[int] = []
    for d in docs:
        stream.extend(tokenizer(d, add_special_tokens=False).input_ids)
        if eos is not None:
            stream.append(eos)
    ids = np.asarray(stream, dtype=np.int64)
    if len(ids) < seqlen + 1:
        raise ValueError(f"corpus has {len(ids)} tokens < seqlen {seqlen}")
    rng = np.random.default_rng(seed)
    max_start = len(ids) - seqlen
    n_disjoint = max_start // seqlen
    if n_disjoint >= nsamples:
        starts = rng.permutation(n_disjoint)[:nsamples] * seqlen
    else:
        log.warning("corpus supports %d disjoint windows of %d tokens; sampling %d overlapping windows",
                    n_disjoint, seqlen, nsamples)
        starts = rng.integers(0, max_start + 1, size=nsamples)
    return torch.from_numpy(np.stack([ids[s:s + seqlen] for s in sorted(starts)]))


_TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json", "tokenizer.model", "vocab.json")


def _vocab_size(model_dir: str, trust_remote_code: bool, config) -> tuple[object, int]:
    if not any(os.path.exists(os.path.join(model_dir, f)) for f in _TOKENIZER_FILES):
        log.warning("no tokenizer files in %s; checking token ids against config.vocab_size", model_dir)
        return None, int(config.vocab_size)
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(model_dir, trust_remote_code=trust_remote_code)
        return tok, len(tok)
    except Exception as exc:  # no tokenizer files: pre-tokenized windows are checked against the config
        log.warning("no tokenizer in %s (%s); checking token ids against config.vocab_size", model_dir, exc)
        return None, int(config.vocab_size)


def main(argv=None):
    from .artifacts import ArtifactReader, ArtifactWriter
    from .sequential import Pipeline, RawShardIndex, build_model

    ap = build_parser()
    args = resolve_args(ap, argv)
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s", datefmt="%H:%M:%S")
    if not os.path.isdir(args.model):
        ap.error("--model must be a local directory (no network)")
    with open(os.path.join(args.model, "config.json")) as f:
        if json.load(f).get("model_type") == "flint":
            ap.error("Flint models are not supported by this build")

    group, rank = None, 0
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import datetime

        import torch.distributed as dist

        dev = torch.device(args.devices[0])
        if dev.type == "cuda":
            torch.cuda.set_device(dev)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=1800), device_id=dev)
        else:  # host-only runs (tests): gloo
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        group, rank = dist.group.WORLD, dist.get_rank()
    log.info("device %s (rank %d), expert-solve VRAM budget %s GiB", args.devices[0], rank, args.vram_gb)

    model = build_model(args.model, torch.bfloat16 if args.dtype == "bfloat16" else torch.float16)
    tokenizer, vocab = _vocab_size(args.model, args.trust_remote_code, model.config)

    tokens_path = os.path.join(args.output, "calib_tokens.npy")
    if os.path.exists(tokens_path):
        samples = torch.from_numpy(np.load(tokens_path))
    elif args.calibration_tokens is not None:
        arr = np.load(os.path.abspath(args.calibration_tokens))
        if arr.ndim != 2:
            raise ValueError(f"calibration tokens must be rank 2, got shape {arr.shape}")
        if rank == 0:
            os.makedirs(args.output, exist_ok=True)
            shutil.copyfile(os.path.abspath(args.calibration_tokens), tokens_path)
        samples = torch.from_numpy(arr)
    else:
        if tokenizer is None:
            raise ValueError("--dataset needs the model's tokenizer")
        samples = load_calibration(tokenizer, args.dataset, args.nsamples, args.seqlen, args.seed)
        if rank == 0:
            os.makedirs(args.output, exist_ok=True)
            np.save(tokens_path, samples.numpy())
    if group is not None:
        import torch.distributed as dist

        dist.barrier(group=group)
    if samples.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"calibration tokens must be integer IDs, got {samples.dtype}")
    if int(samples.min()) < 0 or int(samples.max()) >= vocab:
        raise ValueError(f"token IDs [{int(samples.min())}, {int(samples.max())}] exceed vocabulary {vocab}")
    with open(tokens_path, "rb") as f:
        tokens_sha256 = hashlib.file_digest(f, "sha256").hexdigest()

    header = {"model": args.model, "algorithm": args.mxfp_algorithm if args.mode != "affine" else "gptq",
              "mode": args.mode, "bits": args.bits, "group_size": args.group_size, "storage_dtype": args.dtype,
              "clip": args.clip, "damp": args.damp, "nsamples": int(samples.shape[0]),
              "seqlen": int(samples.shape[1]), "dataset": args.dataset,
              "calibration_tokens": args.calibration_tokens, "calibration_tokens_sha256": tokens_sha256,
              "layers_attr": args.layers_attr, "checkpoint_model_prefix": args.checkpoint_model_prefix,
              "artifact_layers_prefix": args.artifact_layers_prefix}
    # rank 0 writes; layer L's file goes to disk while layer L+1 is calibrated
    writer = ArtifactWriter(args.output, header, overlap=True) if rank == 0 else _ReadOnlyWriter(args.output)
    reader = ArtifactReader(args.output) if writer.manifest["layers_done"] else None
    pipe = Pipeline(model, RawShardIndex(args.model), args, group=group, dp=args.dp_windows)
    try:
        with torch.no_grad():
            pipe.run(samples, writer, reader_for_resume=reader)
    finally:
        writer.close()  # the last layer's file and manifest entry are on disk
    if group is not None:
        import torch.distributed as dist

        dist.barrier(group=group)
        dist.destroy_process_group()
    log.info("artifacts written to %s", args.output)


class _ReadOnlyWriter:
    """Ranks other than 0 see which layers the manifest has (resume) and write nothing."""

    def __init__(self, out_dir: str):
        path = os.path.join(out_dir, "manifest.json")
        self.manifest = {"layers_done": []}
        if os.path.exists(path):
            with open(path) as f:
                self.manifest = json.load(f)

    def layer_done(self, layer_idx: int) -> bool:
        return layer_idx in self.manifest["layers_done"]

    def write_layer(self, *a, **k):
        pass

    def close(self):
        pass


if __name__ == "__main__":
    main()
