"""Calibration artifact store (the per-layer format consumed by Stage B).

Same on-disk contract as mlx_gptq/artifacts.py of the reference:

    calib_dir/
      manifest.json            global settings + per-tensor metadata (atomic rewrite)
      layer_0000.safetensors   {name}.q / {name}.scales / optional {name}.biases
      ...

4-bit codes are stored nibble-packed (two per byte, low nibble first) with
meta ``q_packed = "nibble"``; other widths raw (``"raw"``). Nibble packing and
unpacking run as CUDA kernels; packing happens on the device before the
device-to-host copy, so only the packed bytes cross PCIe.
"""

from __future__ import annotations

import json
import os
import tempfile

import torch
from safetensors.torch import load_file, save_file

from . import _lib as L

_STR_TO_DTYPE = {"bfloat16": torch.bfloat16, "float16": torch.float16}


def _device_for(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("mlx_gptq_b200 packs codes on a CUDA device; none is available")
    return torch.device("cuda", torch.cuda.current_device())


def pack_nibbles(q: torch.Tensor) -> torch.Tensor:
    """artifacts.py:30-32: q[..., 2i] | q[..., 2i+1] << 4 (result on q's device)."""
    assert q.dtype == torch.uint8 and q.shape[-1] % 2 == 0
    dev = _device_for(q)
    t = L.aligned(q.to(dev))
    C = t.shape[-1]
    out = torch.empty(*t.shape[:-1], C // 2, dtype=torch.uint8, device=dev)
    rows = t.numel() // C if C else 0
    L.check(L.lib().gq_pack_nibbles(L.ptr(t), rows, C, L.ptr(out), L.stream_ptr(dev)), "pack_nibbles")
    return out if q.is_cuda else out.cpu()


def unpack_nibbles(p: torch.Tensor) -> torch.Tensor:
    """artifacts.py:35-39 (result on p's device)."""
    dev = _device_for(p)
    t = L.aligned(p.to(dev))
    n = t.shape[-1]
    out = torch.empty(*t.shape[:-1], 2 * n, dtype=torch.uint8, device=dev)
    rows = t.numel() // n if n else 0
    L.check(L.lib().gq_unpack_nibbles(L.ptr(t), rows, n, L.ptr(out), L.stream_ptr(dev)), "unpack_nibbles")
    return out if p.is_cuda else out.cpu()


class ArtifactWriter:
    """artifacts.py:42-93: per-layer safetensors + manifest.json, resumable."""

    def __init__(self, out_dir: str, header: dict):
        self.dir = out_dir
        os.makedirs(out_dir, exist_ok=True)
        self.manifest_path = os.path.join(out_dir, "manifest.json")
        if os.path.exists(self.manifest_path):
            with open(self.manifest_path) as f:
                self.manifest = json.load(f)
            for k, v in header.items():
                if k in ("mode", "bits", "group_size", "storage_dtype") and self.manifest.get(k) != v:
                    raise RuntimeError(
                        f"resume mismatch: manifest has {k}={self.manifest.get(k)}, run has {v}")
        else:
            self.manifest = dict(header)
            self.manifest["tensors"] = {}
            self.manifest["layers_done"] = []

    def layer_done(self, layer_idx: int) -> bool:
        return layer_idx in self.manifest["layers_done"]

    def layer_file(self, layer_idx: int) -> str:
        return os.path.join(self.dir, f"layer_{layer_idx:04d}.safetensors")

    def write_layer(self, layer_idx: int, tensors: dict, meta: dict):
        """tensors: name -> (q uint8 [out, in], scales, optional biases), on any device."""
        flat = {}
        for name, (q, s, b) in tensors.items():
            bits = meta[name]["bits"]
            if bits == 4:
                q = pack_nibbles(q)
                meta[name]["q_packed"] = "nibble"
            else:
                meta[name]["q_packed"] = "raw"
            flat[f"{name}.q"] = q.contiguous().cpu()
            flat[f"{name}.scales"] = s.contiguous().cpu()
            if b is not None:
                flat[f"{name}.biases"] = b.contiguous().cpu()
                meta[name]["has_biases"] = True
            else:
                meta[name]["has_biases"] = False
            meta[name]["file"] = f"layer_{layer_idx:04d}.safetensors"
        save_file(flat, self.layer_file(layer_idx))
        self.manifest["tensors"].update(meta)
        self.manifest["layers_done"].append(layer_idx)
        self._flush()

    def _flush(self):
        fd, tmp = tempfile.mkstemp(dir=self.dir, suffix=".json.tmp")
        with os.fdopen(fd, "w") as f:
            json.dump(self.manifest, f)
        os.replace(tmp, self.manifest_path)


class ArtifactReader:
    """artifacts.py:96-126."""

    def __init__(self, calib_dir: str):
        self.dir = calib_dir
        with open(os.path.join(calib_dir, "manifest.json")) as f:
            self.manifest = json.load(f)
        self.tensors = self.manifest["tensors"]
        self._cache_file = None
        self._cache = None

    @property
    def storage_dtype(self) -> torch.dtype:
        return _STR_TO_DTYPE[self.manifest["storage_dtype"]]

    def has(self, name: str) -> bool:
        return name in self.tensors

    def _load(self, fname: str) -> dict:
        if self._cache_file != fname:
            self._cache = load_file(os.path.join(self.dir, fname))
            self._cache_file = fname
        return self._cache

    def get(self, name: str):
        """Returns (q uint8 [out, in], scales, optional biases, info) on the CPU."""
        info = self.tensors[name]
        blob = self._load(info["file"])
        q = blob[f"{name}.q"]
        if info["q_packed"] == "nibble":
            q = unpack_nibbles(q)
        return q, blob[f"{name}.scales"], blob.get(f"{name}.biases"), info
