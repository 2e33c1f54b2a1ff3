"""Check calibrated artifacts against their source checkpoint (mlx_gptq/validate_artifacts.py).

    python -m mlx_gptq_b200.validate --model DIR --calib OUT [--output report.json]

Per artifact, on the device: dequantize (gq_dequantize), require finite values, and
require every 32-column group's largest magnitude to stay within 32 x the source's
(or 2^-126): the range guard the MXFP solver applies (gptq.py:170-176), so a violation
means a corrupted or mismatched artifact. Same report and exit status as the reference.
"""

from __future__ import annotations

import argparse
import json

import torch

from .artifacts import ArtifactReader
from .grid import MX_GROUP_SIZE, dequantize_artifact
from .sequential import RawShardIndex


def _group_max(value: torch.Tensor) -> torch.Tensor:
    rows, columns = value.shape
    return value.reshape(rows, columns // MX_GROUP_SIZE, MX_GROUP_SIZE).abs().amax(dim=-1)


@torch.no_grad()
def validate(model_path: str, calib_path: str, device="cuda") -> dict:
    """validate_artifacts.py:21-76: {model, calibration, tensors, failures, worst, status}."""
    device = torch.device(device)
    reader = ArtifactReader(calib_path)
    shards = RawShardIndex(model_path)
    failures: list[dict[str, str]] = []
    worst: list[dict[str, float | str]] = []
    for name, info in reader.tensors.items():
        if not shards.has(name):
            failures.append({"name": name, "error": "missing source tensor"})
            continue
        source = shards.get(name).to(device, torch.float32)
        q, scales, biases, artifact_info = reader.get(name)
        mode = artifact_info.get("mode", info.get("mode", "affine"))
        group_size = int(artifact_info.get("group_size", info["group_size"]))
        if tuple(source.shape) != tuple(q.shape):
            failures.append({"name": name, "error": f"shape {tuple(source.shape)} != {tuple(q.shape)}"})
            continue
        dq = dequantize_artifact(q.to(device), scales.to(device), None if biases is None else biases.to(device),
                                 mode, group_size)
        if not bool(torch.isfinite(dq).all()):
            failures.append({"name": name, "error": "non-finite dequantized values"})
            continue
        source_max = _group_max(source).double()
        artifact_max = _group_max(dq).double()
        limit = torch.maximum(source_max * 32.0, torch.full_like(source_max, 2.0 ** -126))
        ratio = float((artifact_max / limit).max())
        if bool((artifact_max > limit).any()):
            failures.append({"name": name, "error": f"group range ratio {ratio:.6g}"})
        worst.append({"name": name, "ratio": round(ratio, 6), "source_max": float(source.abs().max()),
                      "artifact_max": float(dq.abs().max())})
    worst.sort(key=lambda item: float(item["ratio"]), reverse=True)
    return {"model": model_path, "calibration": calib_path, "tensors": len(reader.tensors), "failures": failures,
            "worst": worst[:20], "status": "verified" if not failures else "failed"}


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--model", required=True)
    parser.add_argument("--calib", required=True)
    parser.add_argument("--output")
    parser.add_argument("--device", default="cuda")
    args = parser.parse_args(argv)
    result = validate(args.model, args.calib, args.device)
    text = json.dumps(result, indent=2, sort_keys=True)
    if args.output:
        with open(args.output, "w", encoding="utf-8") as handle:
            handle.write(text + "\n")
    print(text)
    return 0 if result["status"] == "verified" else 1


if __name__ == "__main__":
    raise SystemExit(main())
