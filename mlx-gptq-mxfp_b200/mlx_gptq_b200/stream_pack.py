"""Stage B streaming packer on the GPU (mlx_gptq/stream_pack.py, same flags and output).

    python -m mlx_gptq_b200.stream_pack --hf-path HF_DIR --calib STAGE_A_OUT --mlx-path OUT

Assembles the MLX checkpoint one unit (one decoder layer, or the top-level tensors)
at a time, like the reference: the unit's source tensors are read from the
safetensors shards, renamed to the MLX module tree, per-expert tensors are stacked
into `switch_mlp`, Stage A codes are injected where artifacts exist and every other
quantizable weight is rounded to the grid (RTN). The difference is where the work
runs: each unit's tensors go to the device once, the uint32 word packing of codes
(gq_pack_q) and the RTN quantization (gq_rtn_mxfp) run there, and the packed unit
comes back to the host once to be written. The output files, index and config are
the reference's, tensor for tensor.
"""

from __future__ import annotations

import argparse
import json
import logging
import os
import re
import shutil
from collections import OrderedDict, defaultdict
from pathlib import Path

import torch

from .artifacts import ArtifactReader
from .grid import SUPPORTED_MODES, mode_defaults, rtn_quantize_mxfp
from .packing import pack_q

log = logging.getLogger("mlx_gptq_b200")

NGRAM_SHARD_RE = re.compile(r"\.ngram_embedding\.shard_(\d+)\.")
PER_EXPERT_RE = re.compile(r"(.*)\.mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj|gate_up_proj)\.weight$")

# norm weights stored as (w - 1) by some checkpoints: folded back (stream_pack.py:42-51)
FOLD_ONE = ("q_layernorm.weight", "k_layernorm.weight", "q_norm.weight", "k_norm.weight", "hc_norm.weight",
            "norm_key.weight", "norm_query.weight", "norm_conv.weight")
DEFAULT_EXCLUDE = r"(^|\.)(gate|router)$|shared_expert_gate|e_score|(^|\.)ple($|\.)"


def sanitize_name(k: str, fold: bool) -> str | None:
    """Hugging Face checkpoint key -> MLX module-tree key, None to drop (stream_pack.py:54-66)."""
    if k.startswith(("mtp.", "model.mtp.", "model.visual.", "visual.", "vision_tower.")):
        return None
    if k.startswith("model.language_model."):
        k = "model." + k[len("model.language_model."):]
    elif k.startswith("language_model."):
        k = k[len("language_model."):]
    return NGRAM_SHARD_RE.sub(r".ngram_embedding.shards.\1.", k)


def fold_applies(key: str) -> bool:
    return key.endswith(FOLD_ONE)


def _words(q: torch.Tensor, bits: int) -> torch.Tensor:
    """Codes -> uint32 MLX words, packed on the codes' device and carried as int32 (the
    same bits) until they reach the host."""
    w = pack_q(q, bits)
    return w.view(torch.int32) if w.dtype != torch.int32 else w


def unit_of(mlx_key: str) -> str:
    m = re.match(r"^model\.layers\.(\d+)\.", mlx_key)
    return f"layer.{int(m.group(1)):04d}" if m else "top"


class StreamingPacker:
    """stream_pack.py:77-390 (emit, plan, pack_unit, run, write_metadata)."""

    def __init__(self, hf_path: str, calib: str, out_path: str, mode: str, bits: int, group_size: int,
                 exclude: str | None, storage_dtype: str = "bfloat16", device="cuda"):
        self.hf = Path(hf_path)
        self.out = Path(out_path)
        self.mode = mode
        self.bits = bits
        self.group_size = group_size
        self.exclude = re.compile(exclude) if exclude else None
        self.device = torch.device(device)
        # the reference writes affine scales/biases as float16 unless float32 storage is asked
        self.storage_dtype = torch.float32 if storage_dtype == "float32" else torch.float16
        self.scale_dtype = torch.uint8 if mode != "affine" else self.storage_dtype
        self.torch_dtype = torch.float32 if storage_dtype == "float32" else torch.bfloat16
        self.reader = ArtifactReader(calib)
        index_path = self.hf / "model.safetensors.index.json"
        if index_path.exists():
            self.index = json.loads(index_path.read_text())
            self.weight_map: dict[str, str] = self.index["weight_map"]
        else:
            from safetensors import safe_open

            single = next(self.hf.glob("*.safetensors"))
            with safe_open(str(single), framework="pt") as f:
                self.weight_map = {k: single.name for k in list(f.keys())}
            self.index = {"weight_map": self.weight_map}
        self._open: dict[str, object] = OrderedDict()
        self._open_cap = 8
        self.stats = defaultdict(int)
        self.used_artifacts: set[str] = set()
        self._packed: set[str] = set()  # output keys holding packed words (int32 until written)

    # ---- source ----
    def _reader_for(self, fname: str):
        from safetensors import safe_open

        fh = self._open.get(fname)
        if fh is None:
            fh = safe_open(str(self.hf / fname), framework="pt", device="cpu")
            self._open[fname] = fh
            while len(self._open) > self._open_cap:
                self._open.popitem(last=False)
        else:
            self._open.move_to_end(fname)
        return fh

    def source_files_for(self, keys) -> set[str]:
        return {self.weight_map[k] for k in keys if k in self.weight_map}

    # ---- quantize ----
    def _quantizable(self, key: str, arr: torch.Tensor) -> bool:
        if not key.endswith(".weight") or arr.dim() not in (2, 3) or arr.shape[-1] % self.group_size:
            return False
        module_key = key.removesuffix(".weight")
        if module_key == "lm_head" or module_key.endswith(".lm_head") or module_key.endswith("embed_tokens"):
            return False
        if self.exclude and self.exclude.search(module_key):
            return False
        return "ngram_embedding.shards." not in key

    def _check(self, name: str, info: dict):
        if info.get("bits") != self.bits or info.get("group_size") != self.group_size:
            raise RuntimeError(f"{name}: artifact {info['bits']}b/g{info['group_size']} != config "
                               f"{self.bits}b/g{self.group_size}")

    def emit(self, mlx_key: str, arr: torch.Tensor) -> dict[str, torch.Tensor]:
        """One source tensor -> its MLX tensors (stream_pack.py:161-228); results stay on
        the device until the unit is written."""
        base = mlx_key[: -len(".weight")]
        dev = self.device
        if arr.dim() == 3 and ".switch_mlp." in mlx_key:
            artifacts = [mlx_key.replace(".switch_mlp.", f".experts.{e}.") for e in range(arr.shape[0])]
            if all(self.reader.has(a) for a in artifacts):
                qs, scale_sets = [], []
                for a in artifacts:
                    q, scales, _b, info = self.reader.get(a)
                    self._check(a, info)
                    qs.append(q)
                    scale_sets.append(scales)
                    self.used_artifacts.add(a)
                words = _words(torch.stack(qs).to(dev), self.bits)
                self._packed.add(f"{base}.weight")
                self.stats["injected"] += len(artifacts)
                return {f"{base}.weight": words, f"{base}.scales": torch.stack(scale_sets).to(self.scale_dtype)}
        if self.reader.has(mlx_key) and self._quantizable(mlx_key, arr):
            q, s, b, info = self.reader.get(mlx_key)
            self._check(mlx_key, info)
            out = {f"{base}.weight": _words(q.to(dev), self.bits), f"{base}.scales": s.to(self.scale_dtype)}
            self._packed.add(f"{base}.weight")
            if b is not None:
                out[f"{base}.biases"] = b.float().to(self.storage_dtype)
            self.stats["injected"] += 1
            self.used_artifacts.add(mlx_key)
            return out
        if self._quantizable(mlx_key, arr):
            w = arr.contiguous().to(dev, torch.float32)
            q, s, _b, _dq = rtn_quantize_mxfp(w.unsqueeze(0), self.mode)
            self.stats["rtn"] += 1
            self._packed.add(f"{base}.weight")
            return {f"{base}.weight": _words(q[0], self.bits), f"{base}.scales": s[0].to(self.scale_dtype)}
        self.stats["kept"] += 1
        return {mlx_key: arr}

    # ---- units ----
    def plan(self) -> dict[str, list[str]]:
        units: dict[str, list[str]] = defaultdict(list)
        for k in self.weight_map:
            sk = sanitize_name(k, fold=False)
            if sk is None:
                continue
            m = re.search(r"\.ngram_embedding\.shards\.(\d+)\.", sk)
            units[f"ple.shard.{int(m.group(1)):04d}" if m else unit_of(sk)].append(k)
        return units

    def pack_unit(self, unit: str, hf_keys: list[str]) -> dict[str, torch.Tensor]:
        """stream_pack.py:233-306; returns host tensors ready to write."""
        tensors: dict[str, torch.Tensor] = {}
        for hf_key in hf_keys:
            t = self._reader_for(self.weight_map[hf_key]).get_tensor(hf_key)
            tensors[hf_key] = t.contiguous().to(self.torch_dtype) if t.is_floating_point() else t.contiguous()
        per_expert: dict[str, dict[int, dict[str, torch.Tensor]]] = defaultdict(lambda: defaultdict(dict))
        out: dict[str, torch.Tensor] = {}
        fold = any(k.startswith(("model.language_model.", "language_model.")) for k in tensors)
        for hf_key, arr in tensors.items():
            k = sanitize_name(hf_key, fold)
            if k is None:
                continue
            if k.endswith("mlp.experts.gate_up_proj"):
                base = k[: -len("experts.gate_up_proj")]
                mid = arr.shape[-2] // 2
                out.update(self.emit(base + "switch_mlp.gate_proj.weight", arr[..., :mid, :]))
                out.update(self.emit(base + "switch_mlp.up_proj.weight", arr[..., mid:, :]))
                continue
            if k.endswith("mlp.experts.down_proj"):
                out.update(self.emit(k[: -len("experts.down_proj")] + "switch_mlp.down_proj.weight", arr))
                continue
            m = PER_EXPERT_RE.match(k)
            if m:
                base, idx, proj = m.group(1), int(m.group(2)), m.group(3)
                if proj == "gate_up_proj":
                    mid = arr.shape[-2] // 2
                    per_expert[base][idx]["gate_proj"] = arr[..., :mid, :]
                    per_expert[base][idx]["up_proj"] = arr[..., mid:, :]
                else:
                    per_expert[base][idx][proj] = arr
                continue
            if k.endswith("conv1d.weight") and arr.dim() == 3 and arr.shape[1] == 1:
                arr = arr.permute(0, 2, 1).contiguous()
            if fold and fold_applies(k):
                arr = (1.0 + arr).to(arr.dtype)
            out.update(self.emit(k, arr))
        for base, experts in per_expert.items():
            n = len(experts)
            for proj in ("gate_proj", "up_proj", "down_proj"):
                stacked = torch.stack([experts[i][proj] for i in range(n)], dim=0)
                out.update(self.emit(f"{base}.mlp.switch_mlp.{proj}.weight", stacked))
        host = {}
        for k, v in out.items():
            v = v.contiguous().cpu()
            host[k] = v.view(torch.uint32) if k in self._packed else v
        return host

    def run(self, shard_bytes: int = 4_500_000_000):
        """stream_pack.py:308-371: units in order, shards of about shard_bytes, index and
        config; every Stage A artifact must be consumed."""
        from safetensors.torch import save_file

        self.out.mkdir(parents=True, exist_ok=True)
        units = self.plan()
        order = ["top"] + sorted(u for u in units if u != "top")
        buf: dict[str, torch.Tensor] = {}
        buf_bytes = 0
        shards: list[str] = []

        def flush():
            nonlocal buf, buf_bytes
            if not buf:
                return
            name = f"model-{len(shards) + 1:05d}.safetensors"
            save_file(buf, str(self.out / name), metadata={"format": "mlx"})
            shards.append(name)
            log.info("wrote %s (%.2f GiB, %d tensors)", name, buf_bytes / 2**30, len(buf))
            buf, buf_bytes = {}, 0

        for unit in order:
            for k, v in self.pack_unit(unit, units[unit]).items():
                buf[k] = v
                buf_bytes += v.numel() * v.element_size()
            if buf_bytes >= shard_bytes:
                flush()
        flush()
        unused = [name for name in self.reader.tensors if name not in self.used_artifacts]
        if unused:
            raise RuntimeError(f"{len(unused)} Stage A artifacts were not consumed; first={unused[:3]}")
        self.write_metadata(shards)
        log.info("done: injected=%d rtn=%d kept=%d", self.stats["injected"], self.stats["rtn"], self.stats["kept"])

    def write_metadata(self, shards: list[str]):
        from safetensors import safe_open

        weights: dict[str, str] = {}
        total = 0
        for name in shards:
            with safe_open(str(self.out / name), framework="pt") as f:
                for k in list(f.keys()):
                    weights[k] = name
            total += os.path.getsize(self.out / name)
        (self.out / "model.safetensors.index.json").write_text(
            json.dumps({"metadata": {"total_size": total}, "weight_map": dict(sorted(weights.items()))}, indent=2)
            + "\n")
        cfg = json.loads((self.hf / "config.json").read_text())
        cfg["quantization"] = {"group_size": self.group_size, "bits": self.bits, "mode": self.mode}
        (self.out / "config.json").write_text(json.dumps(cfg, indent=2) + "\n")
        for extra in ("generation_config.json", "tokenizer.json", "tokenizer_config.json", "vocab.json", "merges.txt",
                      "preprocessor_config.json", "video_preprocessor_config.json"):
            src = self.hf / extra
            if src.exists():
                shutil.copy2(src, self.out / extra)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--hf-path", required=True)
    ap.add_argument("--calib", required=True)
    ap.add_argument("--mlx-path", required=True)
    ap.add_argument("--mode", default="mxfp4", choices=SUPPORTED_MODES)
    ap.add_argument("--bits", type=int, default=None)
    ap.add_argument("--group-size", type=int, default=None)
    ap.add_argument("--exclude", default=DEFAULT_EXCLUDE)
    ap.add_argument("--storage-dtype", default="bfloat16")
    ap.add_argument("--shard-gib", type=float, default=4.2)
    ap.add_argument("--device", default="cuda")
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s", datefmt="%H:%M:%S")
    default_group, default_bits = mode_defaults(args.mode)
    StreamingPacker(args.hf_path, args.calib, args.mlx_path, args.mode, args.bits or default_bits,
                    args.group_size or default_group, args.exclude, args.storage_dtype,
                    args.device).run(int(args.shard_gib * 2**30))


if __name__ == "__main__":
    main()
