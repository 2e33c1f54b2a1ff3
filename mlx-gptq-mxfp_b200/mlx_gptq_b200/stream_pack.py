"""Stage B streaming packer on the GPU: Hugging Face source + Stage A artifacts -> MLX model.

    python -m mlx_gptq_b200.stream_pack --hf-path HF_DIR --calib STAGE_A_OUT --mlx-path OUT

Same flags and the same output files as the reference's streaming packer
(mlx_gptq/stream_pack.py): MLX tensor names, experts stacked into ``switch_mlp``,
Stage A codes injected as uint32 MLX words where artifacts exist, every other
quantizable weight rounded to the grid (RTN), shards of about --shard-gib, the
index and the config's ``quantization`` entry. MLX loads exactly these files, so
the naming rules, the stacking order and the inject / RTN / keep decision order are
the reference's; tests compare every output tensor with the reference's bit for bit.

The work is organised around units (the top-level tensors, one decoder layer, one
per-layer-embedding shard), processed as a pipeline:

  1. a loader thread reads unit i+1's source tensors from the safetensors shards
     while unit i is being packed;
  2. ``UnitLayout`` turns a unit's source tensors into MLX-named entries (renaming,
     gate/up splits, per-expert stacking, conv1d layout, norm folding);
  3. each entry gets a ``Decision``; the unit's injected codes and RTN weights go to
     the device, where gq_pack_q packs words and gq_rtn_mxfp rounds, and the packed
     unit comes back to the host with one copy per tensor;
  4. ``ShardSink`` groups units into output shards and writes index and config.
"""

from __future__ import annotations

import argparse
import json
import logging
import os
import re
import shutil
from collections import OrderedDict
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path

import torch

from .artifacts import ArtifactReader
from .grid import SUPPORTED_MODES, mode_defaults, rtn_quantize_mxfp
from .packing import pack_q

log = logging.getLogger("mlx_gptq_b200")

# ---------------------------------------------------------------------------
# MLX naming rules (stream_pack.py:35-75 of the reference; an interface: MLX
# resolves these names)
# ---------------------------------------------------------------------------
NGRAM_SHARD_RE = re.compile(r"\.ngram_embedding\.shard_(\d+)\.")
PER_EXPERT_RE = re.compile(r"(.*)\.mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj|gate_up_proj)\.weight$")
FOLD_ONE = ("q_layernorm.weight", "k_layernorm.weight", "q_norm.weight", "k_norm.weight", "hc_norm.weight",
            "norm_key.weight", "norm_query.weight", "norm_conv.weight")
DEFAULT_EXCLUDE = r"(^|\.)(gate|router)$|shared_expert_gate|e_score|(^|\.)ple($|\.)"
_DROPPED = ("mtp.", "model.mtp.", "model.visual.", "visual.", "vision_tower.")
_WRAPPERS = (("model.language_model.", "model."), ("language_model.", ""))
_EXTRA_FILES = ("generation_config.json", "tokenizer.json", "tokenizer_config.json", "vocab.json", "merges.txt",
                "preprocessor_config.json", "video_preprocessor_config.json")


def sanitize_name(k: str, fold: bool) -> str | None:
    """Hugging Face checkpoint key -> MLX module-tree key, or None for tensors MLX does
    not load (multi-token-prediction and vision towers). `fold` is accepted for the
    reference's signature; folding is decided per unit (see UnitLayout)."""
    if k.startswith(_DROPPED):
        return None
    for wrapper, repl in _WRAPPERS:
        if k.startswith(wrapper):
            k = repl + k[len(wrapper):]
            break
    return NGRAM_SHARD_RE.sub(r".ngram_embedding.shards.\1.", k)


def fold_applies(key: str) -> bool:
    """Norm weights some checkpoints store as (w - 1)."""
    return key.endswith(FOLD_ONE)


def unit_of(mlx_key: str) -> str:
    m = re.match(r"^model\.layers\.(\d+)\.", mlx_key)
    return f"layer.{int(m.group(1)):04d}" if m else "top"


def _unit_for_source_key(hf_key: str) -> str | None:
    k = sanitize_name(hf_key, fold=False)
    if k is None:
        return None
    m = re.search(r"\.ngram_embedding\.shards\.(\d+)\.", k)
    return f"ple.shard.{int(m.group(1)):04d}" if m else unit_of(k)


# ---------------------------------------------------------------------------
# source checkpoint
# ---------------------------------------------------------------------------
class SourceShards:
    """Name -> shard map of a Hugging Face directory with a small LRU of open files."""

    def __init__(self, hf_dir: Path, open_files: int = 8):
        from safetensors import safe_open

        self.dir = hf_dir
        index_path = hf_dir / "model.safetensors.index.json"
        if index_path.exists():
            self.index = json.loads(index_path.read_text())
            self.weight_map: dict[str, str] = self.index["weight_map"]
        else:  # a single-file checkpoint: the map comes from the file itself
            single = next(hf_dir.glob("*.safetensors"))
            with safe_open(str(single), framework="pt") as f:
                self.weight_map = {k: single.name for k in f.keys()}
            self.index = {"weight_map": self.weight_map}
        self._files: OrderedDict[str, object] = OrderedDict()
        self._cap = open_files

    def _file(self, fname: str):
        from safetensors import safe_open

        fh = self._files.pop(fname, None)
        if fh is None:
            fh = safe_open(str(self.dir / fname), framework="pt", device="cpu")
        self._files[fname] = fh
        while len(self._files) > self._cap:
            self._files.popitem(last=False)
        return fh

    def read(self, key: str, float_dtype: torch.dtype) -> torch.Tensor:
        t = self._file(self.weight_map[key]).get_tensor(key).contiguous()
        return t.to(float_dtype) if t.is_floating_point() else t

    def units(self) -> dict[str, list[str]]:
        """Unit name -> its source keys, in index order."""
        out: dict[str, list[str]] = {}
        for k in self.weight_map:
            u = _unit_for_source_key(k)
            if u is not None:
                out.setdefault(u, []).append(k)
        return out


# ---------------------------------------------------------------------------
# one unit's MLX layout
# ---------------------------------------------------------------------------
class UnitLayout:
    """MLX-named entries of one unit, in the order the reference emits them: every
    source tensor in read order (fused expert params split into switch_mlp
    projections, conv1d kernels to MLX's layout, folded norms), then the per-expert
    projections stacked over experts, model by model."""

    def __init__(self):
        self.entries: list[tuple[str, torch.Tensor]] = []
        self._experts: dict[str, dict[int, dict[str, torch.Tensor]]] = {}

    @staticmethod
    def _halves(arr: torch.Tensor):
        mid = arr.shape[-2] // 2
        return arr[..., :mid, :], arr[..., mid:, :]

    def add(self, k: str, arr: torch.Tensor, fold: bool) -> None:
        if k.endswith("mlp.experts.gate_up_proj"):
            base = k[: -len("experts.gate_up_proj")] + "switch_mlp."
            gate, up = self._halves(arr)
            self.entries += [(base + "gate_proj.weight", gate), (base + "up_proj.weight", up)]
            return
        if k.endswith("mlp.experts.down_proj"):
            self.entries.append((k[: -len("experts.down_proj")] + "switch_mlp.down_proj.weight", arr))
            return
        m = PER_EXPERT_RE.match(k)
        if m:
            slot = self._experts.setdefault(m.group(1), {}).setdefault(int(m.group(2)), {})
            if m.group(3) == "gate_up_proj":
                slot["gate_proj"], slot["up_proj"] = self._halves(arr)
            else:
                slot[m.group(3)] = arr
            return
        if k.endswith("conv1d.weight") and arr.dim() == 3 and arr.shape[1] == 1:
            arr = arr.permute(0, 2, 1).contiguous()
        if fold and fold_applies(k):
            arr = (1.0 + arr).to(arr.dtype)
        self.entries.append((k, arr))

    def finish(self) -> list[tuple[str, torch.Tensor]]:
        for base, experts in self._experts.items():
            for proj in ("gate_proj", "up_proj", "down_proj"):
                stacked = torch.stack([experts[i][proj] for i in range(len(experts))], dim=0)
                self.entries.append((f"{base}.mlp.switch_mlp.{proj}.weight", stacked))
        self._experts = {}
        return self.entries


# ---------------------------------------------------------------------------
# decisions and their realisation on the device
# ---------------------------------------------------------------------------
@dataclass
class Decision:
    """How one MLX entry is produced: "stacked" (per-expert artifacts stacked),
    "single" (one artifact), "rtn" (rounded here) or "keep" (copied as is)."""
    kind: str
    key: str
    tensor: torch.Tensor
    artifacts: list[str] = field(default_factory=list)


class StreamingPacker:
    """Stage B packer with the reference's constructor, ``run``, ``stats`` and output."""

    def __init__(self, hf_path: str, calib: str, out_path: str, mode: str, bits: int, group_size: int,
                 exclude: str | None, storage_dtype: str = "bfloat16", device="cuda"):
        self.hf = Path(hf_path)
        self.out = Path(out_path)
        self.mode, self.bits, self.group_size = mode, bits, group_size
        self.exclude = re.compile(exclude) if exclude else None
        self.device = torch.device(device)
        # affine scales / biases are written as float16 unless float32 storage is asked
        self.storage_dtype = torch.float32 if storage_dtype == "float32" else torch.float16
        self.scale_dtype = torch.uint8 if mode != "affine" else self.storage_dtype
        self.read_dtype = torch.float32 if storage_dtype == "float32" else torch.bfloat16
        self.reader = ArtifactReader(calib)
        self.source = SourceShards(self.hf)
        self.weight_map = self.source.weight_map
        self.stats: dict[str, int] = {"injected": 0, "rtn": 0, "kept": 0}
        self.used_artifacts: set[str] = set()

    # ---- decisions (stream_pack.py:146-228: the order inject-stacked, inject, RTN, keep) ----
    def _quantizable(self, key: str, arr: torch.Tensor) -> bool:
        if not key.endswith(".weight") or arr.dim() not in (2, 3) or arr.shape[-1] % self.group_size:
            return False
        module = key[: -len(".weight")]
        if module == "lm_head" or module.endswith((".lm_head", "embed_tokens")):
            return False
        if self.exclude is not None and self.exclude.search(module):
            return False
        return "ngram_embedding.shards." not in key

    def decide(self, key: str, arr: torch.Tensor) -> Decision:
        if arr.dim() == 3 and ".switch_mlp." in key:
            names = [key.replace(".switch_mlp.", f".experts.{e}.") for e in range(arr.shape[0])]
            if all(self.reader.has(n) for n in names):
                return Decision("stacked", key, arr, names)
        quantizable = self._quantizable(key, arr)
        if quantizable and self.reader.has(key):
            return Decision("single", key, arr, [key])
        return Decision("rtn" if quantizable else "keep", key, arr)

    def _artifact(self, name: str):
        q, s, b, info = self.reader.get(name)
        if info.get("bits") != self.bits or info.get("group_size") != self.group_size:
            raise RuntimeError(f"{name}: artifact {info['bits']}b/g{info['group_size']} != config "
                               f"{self.bits}b/g{self.group_size}")
        self.used_artifacts.add(name)
        return q, s, b

    def _words(self, q: torch.Tensor) -> torch.Tensor:
        """Codes -> MLX uint32 words, packed on the device (carried as int32, the same
        bits, until they reach the host)."""
        w = pack_q(q.to(self.device), self.bits)
        return w.view(torch.int32) if w.dtype != torch.int32 else w

    def realize(self, d: Decision) -> dict[str, torch.Tensor]:
        base = d.key[: -len(".weight")]
        if d.kind == "stacked":
            got = [self._artifact(n) for n in d.artifacts]
            self.stats["injected"] += len(got)
            return {f"{base}.weight": self._words(torch.stack([q for q, _, _ in got])),
                    f"{base}.scales": torch.stack([s for _, s, _ in got]).to(self.scale_dtype)}
        if d.kind == "single":
            q, s, b = self._artifact(d.key)
            self.stats["injected"] += 1
            out = {f"{base}.weight": self._words(q), f"{base}.scales": s.to(self.scale_dtype)}
            if b is not None:
                out[f"{base}.biases"] = b.float().to(self.storage_dtype)
            return out
        if d.kind == "rtn":
            w = d.tensor.contiguous().to(self.device, torch.float32).unsqueeze(0)
            q, s, _, _ = rtn_quantize_mxfp(w, self.mode)
            self.stats["rtn"] += 1
            return {f"{base}.weight": self._words(q[0]), f"{base}.scales": s[0].to(self.scale_dtype)}
        self.stats["kept"] += 1
        return {d.key: d.tensor}

    # ---- units ----
    def plan(self) -> dict[str, list[str]]:
        return self.source.units()

    def load_unit(self, hf_keys: list[str]) -> dict[str, torch.Tensor]:
        return {k: self.source.read(k, self.read_dtype) for k in hf_keys}

    def pack_unit(self, unit: str, hf_keys: list[str], loaded: dict | None = None) -> dict[str, torch.Tensor]:
        """One unit, source tensors -> host tensors ready to write (stream_pack.py:233-306)."""
        tensors = self.load_unit(hf_keys) if loaded is None else loaded
        fold = any(k.startswith(("model.language_model.", "language_model.")) for k in tensors)
        layout = UnitLayout()
        for hf_key, arr in tensors.items():
            k = sanitize_name(hf_key, fold)
            if k is not None:
                layout.add(k, arr, fold)
        produced: dict[str, torch.Tensor] = {}
        packed_keys: set[str] = set()
        for key, arr in layout.finish():
            d = self.decide(key, arr)
            out = self.realize(d)
            if d.kind != "keep":
                packed_keys.add(d.key)
            produced.update(out)
        host = {}
        for k, v in produced.items():
            v = v.contiguous().cpu()
            host[k] = v.view(torch.uint32) if k in packed_keys else v
        return host

    def run(self, shard_bytes: int = 4_500_000_000):
        """Every unit in order ("top" first), the source of unit i+1 read while unit i
        is packed; then the index and config. Every Stage A artifact must be consumed
        (stream_pack.py:308-371)."""
        self.out.mkdir(parents=True, exist_ok=True)
        units = self.plan()
        order = ["top"] + sorted(u for u in units if u != "top")
        sink = ShardSink(self.out, shard_bytes)
        with ThreadPoolExecutor(max_workers=1, thread_name_prefix="gq-stage-b-read") as pool:
            nxt = pool.submit(self.load_unit, units.get(order[0], []))
            for i, unit in enumerate(order):
                loaded = nxt.result()
                if i + 1 < len(order):
                    nxt = pool.submit(self.load_unit, units.get(order[i + 1], []))
                sink.add_unit(self.pack_unit(unit, units.get(unit, []), loaded))
        sink.close()
        unused = [n for n in self.reader.tensors if n not in self.used_artifacts]
        if unused:
            raise RuntimeError(f"{len(unused)} Stage A artifacts were not consumed; first={unused[:3]}")
        self.write_metadata(sink.shards)
        log.info("done: injected=%d rtn=%d kept=%d", self.stats["injected"], self.stats["rtn"], self.stats["kept"])

    def write_metadata(self, shards: list[str]):
        write_index_and_config(self.out, self.hf, shards, self.group_size, self.bits, self.mode)


class ShardSink:
    """Collects packed units and writes a shard once it holds at least `limit` bytes
    (a unit never straddles two shards)."""

    def __init__(self, out: Path, limit: int):
        self.out, self.limit = out, limit
        self.shards: list[str] = []
        self._buf: dict[str, torch.Tensor] = {}
        self._bytes = 0

    def add_unit(self, tensors: dict[str, torch.Tensor]) -> None:
        self._buf.update(tensors)
        self._bytes += sum(v.numel() * v.element_size() for v in tensors.values())
        if self._bytes >= self.limit:
            self._write()

    def _write(self) -> None:
        from safetensors.torch import save_file

        if not self._buf:
            return
        name = f"model-{len(self.shards) + 1:05d}.safetensors"
        save_file(self._buf, str(self.out / name), metadata={"format": "mlx"})
        self.shards.append(name)
        log.info("wrote %s (%.2f GiB, %d tensors)", name, self._bytes / 2**30, len(self._buf))
        self._buf, self._bytes = {}, 0

    def close(self) -> None:
        self._write()


def write_index_and_config(out: Path, hf: Path, shards: list[str], group_size: int, bits: int, mode: str):
    """model.safetensors.index.json (sorted weight map, total bytes), config.json with the
    quantization entry, and the tokenizer / generation files copied over."""
    from safetensors import safe_open

    weight_map: dict[str, str] = {}
    for name in shards:
        with safe_open(str(out / name), framework="pt") as f:
            weight_map.update(dict.fromkeys(f.keys(), name))
    total = sum(os.path.getsize(out / name) for name in shards)
    index = {"metadata": {"total_size": total}, "weight_map": dict(sorted(weight_map.items()))}
    (out / "model.safetensors.index.json").write_text(json.dumps(index, indent=2) + "\n")
    cfg = json.loads((hf / "config.json").read_text())
    cfg["quantization"] = {"group_size": group_size, "bits": bits, "mode": mode}
    (out / "config.json").write_text(json.dumps(cfg, indent=2) + "\n")
    for extra in _EXTRA_FILES:
        if (hf / extra).exists():
            shutil.copy2(hf / extra, out / extra)


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
