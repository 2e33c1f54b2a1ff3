"""Calibration artifact store: the per-layer files Stage A writes and Stage B reads.

The directory contract is the reference's (mlx_gptq/artifacts.py), because Stage B
and the resume path read it:

    calib_dir/
      manifest.json            header fields, "tensors" (name -> meta), "layers_done"
      layer_0000.safetensors   {name}.q / {name}.scales / optional {name}.biases
      ...

4-bit codes are stored two per byte (low nibble first), meta ``q_packed = "nibble"``;
other widths one byte per code (``"raw"``). Tensor names are the raw per-expert
checkpoint names.

How this store works is its own:

* a layer is handed over as device tensors; its 4-bit codes are nibble-packed by the
  CUDA kernel before anything leaves the device, so only packed bytes cross PCIe;
* the device-to-host copies run on a side stream into pinned buffers, and the file
  is serialized by a writer thread, so with ``overlap=True`` layer L is written to
  disk while layer L+1 is being calibrated (``flush()`` waits for the last one);
* the manifest is a small document object committed atomically (temporary file +
  rename) only after the layer's file is complete, so a crash at any point leaves a
  directory that resumes correctly;
* the reader opens a layer file lazily and reads only the tensors asked for, and can
  unpack nibbles on a CUDA device (``get(name, device=...)``).
"""

from __future__ import annotations

import json
import os
import tempfile
import threading
from concurrent.futures import Future, ThreadPoolExecutor

import torch

from . import _lib as L

_STR_TO_DTYPE = {"bfloat16": torch.bfloat16, "float16": torch.float16}
MANIFEST_NAME = "manifest.json"
# header fields that must agree when a run resumes into an existing directory
RESUME_FIELDS = ("mode", "bits", "group_size", "storage_dtype")


def layer_file_name(layer_idx: int) -> str:
    return f"layer_{layer_idx:04d}.safetensors"


def _device_for(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("mlx_gptq_b200 packs codes on a CUDA device; none is available")
    return torch.device("cuda", torch.cuda.current_device())


def pack_nibbles(q: torch.Tensor) -> torch.Tensor:
    """Two 4-bit codes per byte, q[..., 2i] in the low nibble (artifacts.py:30-32);
    computed by gq_pack_nibbles, result on q's device."""
    assert q.dtype == torch.uint8 and q.shape[-1] % 2 == 0
    dev = _device_for(q)
    t = L.aligned(q.to(dev))
    C = t.shape[-1]
    out = torch.empty(*t.shape[:-1], C // 2, dtype=torch.uint8, device=dev)
    rows = t.numel() // C if C else 0
    L.check(L.lib().gq_pack_nibbles(L.ptr(t), rows, C, L.ptr(out), L.stream_ptr(dev)), "pack_nibbles")
    return out if q.is_cuda else out.cpu()


def unpack_nibbles(p: torch.Tensor) -> torch.Tensor:
    """Inverse of pack_nibbles (artifacts.py:35-39); result on p's device."""
    dev = _device_for(p)
    t = L.aligned(p.to(dev))
    n = t.shape[-1]
    out = torch.empty(*t.shape[:-1], 2 * n, dtype=torch.uint8, device=dev)
    rows = t.numel() // n if n else 0
    L.check(L.lib().gq_unpack_nibbles(L.ptr(t), rows, n, L.ptr(out), L.stream_ptr(dev)), "unpack_nibbles")
    return out if p.is_cuda else out.cpu()


class _ManifestDoc:
    """manifest.json as an object: a header plus the per-tensor meta and the list of
    completed layers, rewritten atomically on every commit."""

    def __init__(self, path: str, doc: dict):
        self.path = path
        self.doc = doc

    @classmethod
    def load(cls, path: str) -> "_ManifestDoc":
        with open(path) as f:
            return cls(path, json.load(f))

    @classmethod
    def open_for_writing(cls, path: str, header: dict) -> "_ManifestDoc":
        if not os.path.exists(path):
            return cls(path, {**header, "tensors": {}, "layers_done": []})
        existing = cls.load(path)
        clash = [(k, existing.doc.get(k), header[k]) for k in RESUME_FIELDS
                 if k in header and existing.doc.get(k) != header[k]]
        if clash:
            k, have, want = clash[0]
            raise RuntimeError(f"resume mismatch: manifest has {k}={have}, run has {want}")
        return existing

    def record_layer(self, layer_idx: int, entries: dict) -> None:
        self.doc["tensors"].update(entries)
        self.doc["layers_done"].append(layer_idx)

    def commit(self) -> None:
        folder = os.path.dirname(self.path) or "."
        fd, tmp = tempfile.mkstemp(dir=folder, prefix=".manifest.", suffix=".tmp")
        try:
            with os.fdopen(fd, "w") as f:
                json.dump(self.doc, f)
            os.replace(tmp, self.path)
        except BaseException:
            if os.path.exists(tmp):
                os.unlink(tmp)
            raise


class ArtifactWriter:
    """Writes one safetensors file per calibrated layer plus the manifest (the
    reference's ArtifactWriter contract: same constructor, ``manifest``,
    ``layer_done``, ``layer_file``, ``write_layer``).

    overlap=False (default, the reference's behaviour): write_layer returns once the
    layer is on disk. overlap=True: write_layer returns once the layer's device work
    (packing, copy issue) is queued; the file and the manifest entry are written by a
    background thread in layer order, and the next write_layer or flush() waits for
    the previous one (and re-raises its error, if any)."""

    def __init__(self, out_dir: str, header: dict, overlap: bool = False):
        self.dir = out_dir
        os.makedirs(out_dir, exist_ok=True)
        self.manifest_path = os.path.join(out_dir, MANIFEST_NAME)
        self._doc = _ManifestDoc.open_for_writing(self.manifest_path, header)
        self.manifest = self._doc.doc
        self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="gq-artifacts") if overlap else None
        self._pending: Future | None = None
        self._streams: dict[int, torch.cuda.Stream] = {}

    def layer_done(self, layer_idx: int) -> bool:
        return layer_idx in self.manifest["layers_done"]

    def layer_file(self, layer_idx: int) -> str:
        return os.path.join(self.dir, layer_file_name(layer_idx))

    # -- staging: device tensors -> packed payloads -> pinned host copies ----------
    def _copy_stream(self, dev: torch.device) -> torch.cuda.Stream:
        s = self._streams.get(dev.index)
        if s is None:
            s = self._streams[dev.index] = torch.cuda.Stream(dev)
        return s

    @staticmethod
    def _payloads(layer_idx: int, tensors: dict, meta: dict):
        """(file key -> tensor) in write order and the manifest entries of the layer."""
        payload, entries = {}, {}
        fname = layer_file_name(layer_idx)
        for name, (q, s, b) in tensors.items():
            nibble = meta[name]["bits"] == 4
            payload[f"{name}.q"] = pack_nibbles(q) if nibble else q
            payload[f"{name}.scales"] = s
            if b is not None:
                payload[f"{name}.biases"] = b
            entries[name] = dict(meta[name], q_packed="nibble" if nibble else "raw", has_biases=b is not None,
                                 file=fname)
        return payload, entries

    def _to_host(self, payload: dict):
        """Issue every device-to-host copy on a side stream; returns the host tensors
        and the events that mark them complete."""
        host, events = {}, []
        by_dev: dict[int, list] = {}
        for k, t in payload.items():
            if t.is_cuda:
                by_dev.setdefault(t.device.index, []).append(k)
            else:
                host[k] = t.contiguous()
        for idx, keys in by_dev.items():
            dev = torch.device("cuda", idx)
            side = self._copy_stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))  # packing and solves are done
            with torch.cuda.stream(side):
                for k in keys:
                    t = payload[k].contiguous()
                    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                    h.copy_(t, non_blocking=True)
                    t.record_stream(side)
                    host[k] = h
                ev = torch.cuda.Event()
                ev.record(side)
            events.append(ev)
        return host, events

    def _finish(self, layer_idx: int, host: dict, events, entries: dict) -> None:
        from safetensors.torch import save_file

        for ev in events:
            ev.synchronize()
        save_file(host, self.layer_file(layer_idx))
        self._doc.record_layer(layer_idx, entries)
        self._doc.commit()

    def write_layer(self, layer_idx: int, tensors: dict, meta: dict):
        """tensors: name -> (q uint8 [out, in], scales, optional biases), on any device;
        meta: name -> per-tensor fields (bits, group_size, mode, ...)."""
        self.flush()  # layers reach the manifest in order; surfaces a failed write
        payload, entries = self._payloads(layer_idx, tensors, meta)
        host, events = self._to_host(payload)
        if self._pool is None:
            self._finish(layer_idx, host, events, entries)
        else:
            self._pending = self._pool.submit(self._finish, layer_idx, host, events, entries)

    def flush(self) -> None:
        """Wait until every layer handed to write_layer is on disk."""
        pending, self._pending = self._pending, None
        if pending is not None:
            pending.result()

    def close(self) -> None:
        self.flush()
        if self._pool is not None:
            self._pool.shutdown(wait=True)
            self._pool = None


class ArtifactReader:
    """Reads a Stage A directory (the reference's ArtifactReader contract: ``manifest``,
    ``tensors``, ``storage_dtype``, ``has``, ``get``). Layer files are opened lazily,
    at most a few at a time, and only the requested tensors are read."""

    _OPEN_FILES = 2

    def __init__(self, calib_dir: str):
        self.dir = calib_dir
        self.manifest = _ManifestDoc.load(os.path.join(calib_dir, MANIFEST_NAME)).doc
        self.tensors = self.manifest["tensors"]
        self._handles: dict[str, object] = {}
        self._lock = threading.Lock()

    @property
    def storage_dtype(self) -> torch.dtype:
        return _STR_TO_DTYPE[self.manifest["storage_dtype"]]

    def has(self, name: str) -> bool:
        return name in self.tensors

    def _handle(self, fname: str):
        from safetensors import safe_open

        with self._lock:
            h = self._handles.pop(fname, None)
            if h is None:
                h = safe_open(os.path.join(self.dir, fname), framework="pt", device="cpu")
            self._handles[fname] = h  # most recently used last
            while len(self._handles) > self._OPEN_FILES:
                self._handles.pop(next(iter(self._handles)))
            return h

    def get(self, name: str, device=None):
        """(q uint8 [out, in], scales, biases or None, meta) for one tensor: on the CPU,
        or on `device` (codes then cross to the device packed and are unpacked there)."""
        info = self.tensors[name]
        h = self._handle(info["file"])
        keys = set(h.keys())

        def read(suffix):
            t = h.get_tensor(f"{name}.{suffix}") if f"{name}.{suffix}" in keys else None
            return t if t is None or device is None else t.to(device)

        q, scales, biases = read("q"), read("scales"), read("biases")
        if info["q_packed"] == "nibble":
            q = unpack_nibbles(q)
        return q, scales, biases, info
