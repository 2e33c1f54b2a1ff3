"""Layer-sequential Stage A driver (mlx_gptq/sequential.py, Pipeline.run).

The model is a meta-device skeleton; each decoder layer's weights are
materialized on the forward device right before it is processed and released
after it. Per layer (sequential.py:680-770):

  1. materialize the layer's weights (from safetensors shards, or a seeded
     synthetic source for random-init benchmarks);
  2. forward every calibration batch with capture hooks (CaptureManager);
  3. solve every weight matrix (pipeline.solve_layer: grouped tcgen05 Hessians,
     batched factors, GPTQ column loops), writing W_dq back into the layer;
  4. re-forward to produce the quantized activations for the next layer;
  5. append the layer's artifacts.

Differences from the reference, all B200-first:
  * hidden states and per-layer call contexts stay in HBM between layers
    (a 524,288-token window of hidden 2048 is 2.1 GB) instead of moving to host RAM;
  * several GPUs are several processes (one per GPU, torch.distributed NCCL):
    every rank runs the same forward, experts and linears are split across ranks
    inside solve_layer, and one all-gather per task returns the quantized
    weights; rank 0 alone writes artifacts;
  * several devices in one process (``args.devices`` with more than one entry, the
    reference's own multi-device mode) spread each fused task's experts over the
    devices, one thread per device; the forward runs on the first device.
"""

from __future__ import annotations

import contextlib
import json
import logging
import os
import re
import time
import zlib
from dataclasses import dataclass, field

import torch

from .capture import CaptureManager
from .experts import install_grouped_experts
from .pipeline import LayerSolveArgs, solve_layer

log = logging.getLogger("mlx_gptq_b200")

DEFAULT_EXCLUDE = r"(^|\.)gate$|(^|\.)router($|\.)|shared_expert_gate|e_score"  # sequential.py:38


# ---------------------------------------------------------------------------
# weight sources
# ---------------------------------------------------------------------------
class ShardIndex:
    """Tensor name -> file of a Hugging Face safetensors checkpoint (the reference's
    RawShardIndex contract: ``has``, ``get``, ``get_rows``, ``names_with_prefix``).
    Files are opened on first use and kept in a small LRU; ``get_rows`` reads only the
    requested rows of a tensor (lazy per-layer embeddings)."""

    INDEX = "model.safetensors.index.json"

    def __init__(self, model_dir: str, single_file: str = "model.safetensors", open_files: int = 16):
        import glob

        self.dir = model_dir
        index = os.path.join(model_dir, self.INDEX)
        if os.path.exists(index):
            with open(index) as f:
                self.weight_map: dict[str, str] = json.load(f)["weight_map"]
        else:
            files = sorted(glob.glob(os.path.join(model_dir, single_file)))
            if not files:
                raise FileNotFoundError(f"no safetensors found in {model_dir}")
            fname = os.path.basename(files[0])
            self.weight_map = dict.fromkeys(self._open(fname).keys(), fname)
        self._handles: dict[str, object] = {}
        self._cap = open_files

    def _open(self, fname: str):
        from safetensors import safe_open

        return safe_open(os.path.join(self.dir, fname), framework="pt")

    def _handle(self, name: str):
        fname = self.weight_map[name]
        h = self._handles.pop(fname, None)
        if h is None:
            h = self._open(fname)
        self._handles[fname] = h  # most recently used last
        while len(self._handles) > self._cap:
            self._handles.pop(next(iter(self._handles)))
        return h

    def has(self, name: str) -> bool:
        return name in self.weight_map

    def get(self, name: str) -> torch.Tensor:
        return self._handle(name).get_tensor(name)

    def get_rows(self, name: str, rows: list[int]) -> torch.Tensor:
        return self._handle(name).get_slice(name)[rows]

    def names_with_prefix(self, prefix: str):
        return [n for n in self.weight_map if n.startswith(prefix)]


RawShardIndex = ShardIndex  # the reference's name (mlx_gptq/sequential.py:44-90)


class SyntheticWeights:
    """Seeded random-init stand-in for a checkpoint: every meta parameter or buffer
    of `model` is produced on demand, on `device`, from its own generator seeded by
    (seed, name), so every rank and every run sees the same weights. 1-D weights
    named like norms are ones (RMSNorm init), biases zeros, the rest N(0, std)
    (the Hugging Face initializer_range default)."""

    def __init__(self, model: torch.nn.Module, device, seed: int = 0, std: float = 0.02):
        self.device = torch.device(device)
        self.seed = int(seed)
        self.std = float(std)
        self.shapes = {}
        for n, p in model.named_parameters():
            if p.is_meta:
                self.shapes[n] = tuple(p.shape)
        for n, b in model.named_buffers():
            if b is not None and b.is_meta:
                self.shapes[n] = tuple(b.shape)

    def has(self, name: str) -> bool:
        return name in self.shapes

    def get(self, name: str) -> torch.Tensor:
        shape = self.shapes[name]
        leaf = name.rsplit(".", 1)[-1]
        if leaf == "bias":
            return torch.zeros(shape, dtype=torch.float32, device=self.device)
        if len(shape) == 1 and ("norm" in name or "layernorm" in name):
            return torch.ones(shape, dtype=torch.float32, device=self.device)
        g = torch.Generator(device=self.device)
        g.manual_seed((self.seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF)
        return torch.randn(shape, generator=g, dtype=torch.float32, device=self.device).mul_(self.std)


@contextlib.contextmanager
def empty_weights():
    """Build modules with parameters on the meta device and real buffers, the state
    calibrate.build_model gets from init_empty_weights(include_buffers=False)."""
    orig = torch.nn.Module.register_parameter

    def register(module, name, param):
        orig(module, name, param)
        if param is not None and not param.is_meta:
            p = module._parameters[name]
            module._parameters[name] = torch.nn.Parameter(p.to("meta"), requires_grad=p.requires_grad)

    torch.nn.Module.register_parameter = register
    try:
        yield
    finally:
        torch.nn.Module.register_parameter = orig


def build_model(model_or_config, dtype: torch.dtype = torch.bfloat16):
    """Meta-parameter skeleton of a Hugging Face causal LM with the eager expert loop
    (calibrate.py:29-57): a model directory, a config dict, or a PretrainedConfig."""
    from transformers import AutoConfig, AutoModelForCausalLM, PretrainedConfig

    if isinstance(model_or_config, PretrainedConfig):
        config = model_or_config
    elif isinstance(model_or_config, dict):
        cfg = dict(model_or_config)
        config = AutoConfig.for_model(cfg.pop("model_type"), **cfg)
    else:
        config = AutoConfig.from_pretrained(model_or_config)
    config._experts_implementation = "eager"  # F.linear per expert: the capture path
    with empty_weights():
        model = AutoModelForCausalLM.from_config(config, dtype=dtype, attn_implementation="sdpa")
    model.eval()
    model.config.use_cache = False
    return model


_FUSED_EXPERT_PARAM = re.compile(r"^(.*)\.(gate_up_proj|gate_proj|up_proj|down_proj)$")


def _to(t: torch.Tensor, device, dtype) -> torch.Tensor:
    """Checkpoint tensor -> device, floating point ones in the runtime dtype."""
    return (t.to(dtype) if t.is_floating_point() else t).to(device)


def _expert_sources(name: str, p: torch.Tensor):
    """For a fused 3-D expert parameter missing from the checkpoint, the per-expert
    tensors that make it up: [[gate, up] or [proj]] per expert; None otherwise."""
    m = _FUSED_EXPERT_PARAM.match(name)
    if m is None or p.dim() != 3:
        return None
    base, kind = m.groups()
    parts = ("gate_proj", "up_proj") if kind == "gate_up_proj" else (kind,)
    return [[f"{base}.{e}.{part}.weight" for part in parts] for e in range(p.shape[0])]


def _load_param(shards, name: str, p: torch.Tensor, device, dtype) -> torch.Tensor:
    if shards.has(name):
        return _to(shards.get(name), device, dtype)
    sources = _expert_sources(name, p)
    if sources is None:
        raise KeyError(f"cannot materialize parameter {name} from checkpoint")
    fused = torch.empty(p.shape, dtype=dtype, device=device)
    for e, names in enumerate(sources):  # expert e = its rows stacked ([gate; up] for gate_up)
        torch.cat([_to(shards.get(n), device, dtype) for n in names], dim=0, out=fused[e])
    return fused


def _load_buffer(shards, name: str, b: torch.Tensor, device, dtype) -> torch.Tensor:
    if shards.has(name):
        return _to(shards.get(name), device, dtype)
    if b.is_meta:
        raise KeyError(f"meta buffer {name} not in checkpoint")
    return b.to(device)  # derived buffers built at init (not checkpointed) follow the layer


def materialize_module(module: torch.nn.Module, prefix: str, shards, device, dtype) -> None:
    """Give a meta module real parameters and buffers from `shards` (sequential.py:93-145):
    checkpoint tensors by name, fused 3-D expert parameters assembled from per-expert
    checkpoint tensors (gate_up_proj [E, 2I, H] from X.{e}.gate_proj / X.{e}.up_proj,
    down_proj [E, H, I] from X.{e}.down_proj), derived buffers moved to `device`."""
    state = {n: _load_param(shards, f"{prefix}.{n}", p, device, dtype) for n, p in module.named_parameters()}
    state.update({n: _load_buffer(shards, f"{prefix}.{n}", b, device, dtype) for n, b in module.named_buffers()})
    module.load_state_dict(state, strict=False, assign=True)
    left = [n for n, p in module.named_parameters() if p.is_meta]
    if left:
        raise RuntimeError(f"parameter {prefix}.{left[0]} still on meta after materialize")


def free_module(module: torch.nn.Module):
    """Release a layer's weights by putting it back on meta (sequential.py:148-150)."""
    module.to_empty(device="meta")


class LazyShardedEmbedding(torch.nn.Module):
    """An embedding table stored as row shards in the checkpoint, read row by row on
    demand instead of materialized (sequential.py:153-190, Gemma-4 per-layer embeddings):
    each forward reads only the distinct rows its ids select, once, then places them on
    the device."""

    def __init__(self, prefix: str, shards, n_shards: int, rows_per_shard: int, dim: int, device, dtype):
        super().__init__()
        self.prefix = prefix
        self.shards = shards
        self.n_shards = n_shards
        self.rows_per_shard = rows_per_shard
        self.dim = dim
        self.device = torch.device(device)
        self.dtype = dtype
        self.weight = torch.empty(0, device=device, dtype=dtype)  # callers check its device

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        flat = ids.detach().reshape(-1).to("cpu", torch.long)
        uniq, inverse = torch.unique(flat, return_inverse=True)
        rows = torch.empty(uniq.numel(), self.dim, dtype=self.dtype)
        shard_of = uniq // self.rows_per_shard
        for shard in torch.unique(shard_of).tolist():
            sel = (shard_of == shard).nonzero().flatten()
            local = (uniq[sel] % self.rows_per_shard).tolist()
            rows[sel] = self.shards.get_rows(f"{self.prefix}.shard_{shard}.weight", local).to(self.dtype)
        return rows.to(self.device)[inverse.to(self.device)].reshape(*ids.shape, self.dim)


_PLE_TABLE = "ple.ple_embedding.ngram_embedding"
_SHARD_NO = re.compile(r"\.shard_(\d+)\.weight$")


def _ple_shard_count(shards, table_name: str) -> int:
    """Number of row shards stored for one per-layer embedding table: shard_0 ..
    shard_{n-1}, every one present."""
    found = sorted({int(m.group(1)) for n in shards.names_with_prefix(table_name + ".shard_")
                    if (m := _SHARD_NO.search(n))})
    if not found:
        raise KeyError(f"no PLE shards found for {table_name}")
    if found != list(range(len(found))):
        raise KeyError(f"PLE shards of {table_name} are not numbered 0..{len(found) - 1}: {found}")
    return len(found)


def install_lazy_ple(module: torch.nn.Module, prefix: str, shards, device, dtype):
    """Swap every fused per-layer embedding table under `module` (a module path ending
    in ple.ple_embedding.ngram_embedding, the Gemma-4 layout of sequential.py:193-229)
    for a LazyShardedEmbedding reading its rows from the checkpoint's row shards."""
    tables = [(name, child) for name, child in module.named_modules() if name.endswith(_PLE_TABLE)]
    for name, child in tables:
        rows, dim = child.weight.shape
        n = _ple_shard_count(shards, f"{prefix}.{name}")
        per, rem = divmod(rows, n)
        if rem:
            raise ValueError(f"PLE rows {rows} are not divisible by {n} shards")
        owner, attr = name.rsplit(".", 1)
        setattr(module.get_submodule(owner), attr,
                LazyShardedEmbedding(f"{prefix}.{name}", shards, n, per, dim, device, dtype))


# ---------------------------------------------------------------------------
# layer-0 inputs and per-layer call contexts
# ---------------------------------------------------------------------------
class _StopForward(Exception):
    """Raised by the last recorder: the rest of the model call is not needed."""


@dataclass
class _CallLog:
    """What one model call looks like from the decoder stack: the hidden states that
    enter layer 0 and the (args, kwargs) every layer is called with."""
    n_layers: int
    hidden: torch.Tensor | None = None
    contexts: list = field(default_factory=list)

    def __post_init__(self):
        self.contexts = [None] * self.n_layers

    def complete(self) -> bool:
        return self.hidden is not None and all(c is not None for c in self.contexts)


class _LayerRecorder(torch.nn.Module):
    """Stands in for decoder layer `index` during one model call (sequential.py:236-253):
    records its call into the log and passes the hidden states through; the last one
    ends the call."""

    def __init__(self, log: _CallLog, index: int):
        super().__init__()
        self.log, self.index = log, index

    def forward(self, hidden_states, *args, **kwargs):
        if self.index == 0:
            self.log.hidden = hidden_states.detach().clone()
        self.log.contexts[self.index] = (args, kwargs)
        if self.index == self.log.n_layers - 1:
            raise _StopForward
        return hidden_states


class _ContextDetacher:
    """Detached copy of the layer call contexts of one batch: tensors detached (they
    stay on the forward device), tuples / lists / dicts rebuilt, anything else kept as
    is, and every object mapped once, so a container that layer i mutates and layer
    i+1 reads stays one shared object across the copied contexts (the identity rule of
    sequential.py:271-293)."""

    def __init__(self):
        self._seen: dict[int, object] = {}

    def __call__(self, value):
        hit = self._seen.get(id(value), self)
        if hit is not self:
            return hit
        if isinstance(value, torch.Tensor):
            out = value.detach()
        elif isinstance(value, dict):
            out = {k: self(v) for k, v in value.items()}
        elif isinstance(value, tuple):
            out = tuple(self(v) for v in value)
        elif isinstance(value, list):
            out = [self(v) for v in value]
        else:
            out = value
        self._seen[id(value)] = out
        return out


# ---------------------------------------------------------------------------
# the driver
# ---------------------------------------------------------------------------
@dataclass
class LayerStats:
    layer: int
    linears: int
    experts: int
    capture_s: float
    solve_s: float
    reforward_s: float
    total_s: float
    solved_elems: int
    rel_err_median: float
    rel_err_max: float
    extra: dict = field(default_factory=dict)


class Pipeline:
    """Layer-sequential calibration over a meta-skeleton model (sequential.py:345-770).

    `args` carries the calibrate CLI fields: devices, dtype, layers_attr,
    checkpoint_model_prefix, artifact_layers_prefix, exclude, group_size, bits,
    mode, mxfp_algorithm, damp, clip, overrides, batch_size (and optionally
    vram_gb, experts_forward: "grouped" (default; the sort-based expert forward
    of experts.py, bit-identical to the eager loop) or "eager"). `group` is a
    torch.distributed process group whose ranks share the solves (None: this
    process alone). Every rank runs every calibration window through each layer
    unless dp=True: then rank r forwards only its contiguous share of the windows,
    Hessians are summed over ranks, and the forward scales with the ranks too (the
    result matches one process within the Hessian tolerance, not bit for bit)."""

    def __init__(self, model, shards, args, group=None, dp: bool = False):
        self.model = model
        self.shards = shards
        self.args = args
        self.group = group
        self.dp = bool(dp) and group is not None
        self.devices = [torch.device(d) for d in args.devices]
        self.dev0 = self.devices[0]  # forward device; experts spread over all of self.devices
        self.dtype = torch.bfloat16 if args.dtype == "bfloat16" else torch.float16
        self.storage_dtype = self.dtype
        inner = model
        for attr in args.layers_attr.split(".")[:-1]:
            inner = getattr(inner, attr)
        for module in model.modules():
            for name, buf in module.named_buffers(recurse=False):
                if buf is not None and not buf.is_meta:
                    setattr(module, name, buf.to(self.dev0))
        self.inner = inner
        self.layers = getattr(inner, args.layers_attr.split(".")[-1])
        self.grouped_experts = 0
        if getattr(args, "experts_forward", "grouped") == "grouped":
            self.grouped_experts = install_grouped_experts(model)
        self.runtime_model_prefix = args.layers_attr.split(".", 1)[0]
        self.checkpoint_model_prefix = args.checkpoint_model_prefix or self.runtime_model_prefix
        self.checkpoint_layers_prefix_fmt = self._checkpoint_name(args.layers_attr) + ".{}"
        self.artifact_layers_prefix_fmt = (args.artifact_layers_prefix or args.layers_attr) + ".{}"
        self.stats: list[LayerStats] = []

    @property
    def rank(self) -> int:
        if self.group is None:
            return 0
        import torch.distributed as dist

        return dist.get_rank(self.group)

    def _checkpoint_name(self, runtime_name: str) -> str:
        if runtime_name == self.runtime_model_prefix:
            return self.checkpoint_model_prefix
        prefix = self.runtime_model_prefix + "."
        if runtime_name.startswith(prefix):
            return self.checkpoint_model_prefix + runtime_name[len(self.runtime_model_prefix):]
        return runtime_name

    def _sync(self):
        if self.dev0.type == "cuda":
            torch.cuda.synchronize(self.dev0)

    # ---- layer-0 inputs ----
    @torch.no_grad()
    def catch_layer0_inputs(self, samples: torch.Tensor, batch_size: int):
        """Layer-0 hidden states and every layer's call context per batch
        (sequential.py:353-418); kept on the forward device."""
        emb = self.model.get_input_embeddings()
        emb_name = next(n for n, m in self.model.named_modules() if m is emb)
        materialize_module(emb, self._checkpoint_name(emb_name), self.shards, self.dev0, self.dtype)
        batches = []
        original = list(self.layers)
        try:
            for i in range(0, samples.shape[0], batch_size):
                log_ = _CallLog(len(original))
                for li in range(len(original)):
                    self.layers[li] = _LayerRecorder(log_, li)
                with contextlib.suppress(_StopForward):
                    self.model(input_ids=samples[i: i + batch_size].to(self.dev0), use_cache=False)
                if not log_.complete():
                    raise RuntimeError("catcher did not observe every decoder layer")
                detach = _ContextDetacher()
                contexts = [(detach(args), {k: detach(v) for k, v in kwargs.items()})
                            for args, kwargs in log_.contexts]
                batches.append((log_.hidden, contexts))
        finally:
            for li, layer in enumerate(original):
                self.layers[li] = layer
        free_module(emb)
        if not batches:
            raise RuntimeError("catcher captured nothing; layers_attr wrong?")
        return batches

    # ---- one layer ----
    @torch.no_grad()
    def forward_layer(self, layer, batches, layer_idx, capture_mgr=None):
        """Run every batch through `layer`; returns the new hidden states (sequential.py:422-437)."""
        outs = []
        for hid, contexts in batches:
            if capture_mgr is not None:
                capture_mgr.begin_batch()
            args, kwargs = contexts[layer_idx]
            out = layer(hid.to(self.dev0, self.dtype), *args, **kwargs)
            if isinstance(out, tuple):
                out = out[0]
            outs.append(out.detach())
        return outs

    def solve_args(self) -> LayerSolveArgs:
        a = self.args
        vram = getattr(a, "vram_gb", None)
        if isinstance(vram, dict):
            vram = vram.get(str(self.dev0), next(iter(vram.values())) if vram else None)
        return LayerSolveArgs(bits=a.bits, group_size=a.group_size, mode=a.mode,
                              mxfp_algorithm=getattr(a, "mxfp_algorithm", "auto"), damp=a.damp, clip=a.clip,
                              storage_dtype=self.storage_dtype, overrides=list(getattr(a, "overrides", []) or []),
                              vram_gb=vram)

    @torch.no_grad()
    def solve_layer(self, layer_idx: int, mgr: CaptureManager):
        prefix = self.artifact_layers_prefix_fmt.format(layer_idx)
        return solve_layer(prefix, mgr, self.solve_args(), self.dev0, group=self.group, on_device=True, dp=self.dp,
                           devices=self.devices)

    @torch.no_grad()
    def apply_precomputed(self, layer, layer_idx: int, reader) -> None:
        """Resume: write dequantized artifacts into a layer (sequential.py:637-679)."""
        from .grid import dequantize_artifact

        prefix = self.artifact_layers_prefix_fmt.format(layer_idx)
        for name, mod in layer.named_modules():
            if isinstance(mod, torch.nn.Linear):
                art = f"{prefix}.{name}.weight"
                if reader.has(art):
                    q, s, b, info = reader.get(art)
                    dq = dequantize_artifact(q.to(self.dev0), s.to(self.dev0), None if b is None else b.to(self.dev0),
                                             info.get("mode", "affine"), info["group_size"])
                    mod.weight.data.copy_(dq.reshape(q.shape).to(mod.weight.dtype))
            for pname, p in mod.named_parameters(recurse=False):
                if p.dim() != 3 or pname not in ("gate_up_proj", "gate_proj", "up_proj", "down_proj"):
                    continue
                E, R, _ = p.shape
                for e in range(E):
                    if pname == "gate_up_proj":
                        arts = [f"{prefix}.{name}.{e}.gate_proj.weight", f"{prefix}.{name}.{e}.up_proj.weight"]
                        rows = [(0, R // 2), (R // 2, R)]
                    else:
                        arts, rows = [f"{prefix}.{name}.{e}.{pname}.weight"], [(0, R)]
                    for art, (r0, r1) in zip(arts, rows):
                        if not reader.has(art):
                            continue
                        q, s, b, info = reader.get(art)
                        dq = dequantize_artifact(q.to(self.dev0), s.to(self.dev0),
                                                 None if b is None else b.to(self.dev0),
                                                 info.get("mode", "affine"), info["group_size"])
                        p.data[e, r0:r1].copy_(dq.reshape(q.shape).to(p.dtype))

    # ---- orchestration ----
    def run(self, samples: torch.Tensor, writer=None, reader_for_resume=None, layers=None):
        """Calibrate every decoder layer (or the first `layers`) in order
        (sequential.py:683-770). Only rank 0 writes artifacts. Returns this rank's
        batches (all of them, or its share of the windows with dp)."""
        t_start = time.time()
        if self.dp:
            import torch.distributed as dist

            world = dist.get_world_size(self.group)
            if samples.shape[0] < world:
                raise ValueError(f"dp needs at least one calibration window per rank ({samples.shape[0]} < {world})")
            n = samples.shape[0]  # balanced contiguous shares: every rank gets >= 1 window
            samples = samples[self.rank * n // world:(self.rank + 1) * n // world]
        batches = self.catch_layer0_inputs(samples, self.args.batch_size)
        log.info("caught %d forward batches for layer 0", len(batches))
        n_layers = len(self.layers) if layers is None else min(int(layers), len(self.layers))
        for li in range(n_layers):
            layer = self.layers[li]
            prefix = self.checkpoint_layers_prefix_fmt.format(li)
            t0 = time.time()
            if getattr(self.args, "lazy_ple", False):
                install_lazy_ple(layer, prefix, self.shards, self.dev0, self.dtype)
            materialize_module(layer, prefix, self.shards, self.dev0, self.dtype)
            if writer is not None and writer.layer_done(li):
                self.apply_precomputed(layer, li, reader_for_resume)
                new = self.forward_layer(layer, batches, li)
                batches = [(h, ctx) for h, (_, ctx) in zip(new, batches)]
                free_module(layer)
                log.info("layer %d: resumed from artifacts (%.1fs)", li, time.time() - t0)
                continue

            mgr = CaptureManager(layer, self.args.exclude, self.args.group_size, stash_device=self.dev0,
                                 reserve_tokens=sum(h.shape[0] * h.shape[1] for h, _ in batches))
            n_lin = len(mgr.linear_tasks)
            n_exp = sum(t.num_experts for t in mgr.fused_tasks)
            with mgr:
                self.forward_layer(layer, batches, li, capture_mgr=mgr)
            if self.dp:
                mgr.sync_token_counts(self.group, self.dev0)
            if mgr.fused_tasks:
                mgr.check_capture_happened()
                for pname, (mn, med, mx, zeros) in mgr.expert_token_stats().items():
                    log.info("layer %d %s tokens/expert min=%d med=%d max=%d zero=%d", li, pname, mn, med, mx, zeros)
                for module_name, experts in mgr.backfill_unrouted_experts().items():
                    log.warning("layer %d %s: activation-backfilled unrouted experts %s", li, module_name, experts)
                if self.dp:  # backfilled rows were added on every rank
                    mgr.sync_token_counts(self.group, self.dev0)
            self._sync()
            t_cap = time.time()

            result = self.solve_layer(li, mgr)
            mgr.drop_all()
            self._sync()
            t_solve = time.time()

            new = self.forward_layer(layer, batches, li)
            batches = [(h, ctx) for h, (_, ctx) in zip(new, batches)]
            self._sync()
            t_fwd = time.time()
            free_module(layer)  # the caching allocator keeps the blocks for the next layer
            if writer is not None and self.rank == 0:
                writer.write_layer(li, result.tensors, result.meta)
            errs = sorted(m["rel_err"] for m in result.meta.values())
            elems = sum(int(m["out_features"]) * int(m["in_features"]) for m in result.meta.values())
            st = LayerStats(li, n_lin, n_exp, t_cap - t0, t_solve - t_cap, t_fwd - t_solve, time.time() - t0, elems,
                            errs[len(errs) // 2] if errs else -1.0, errs[-1] if errs else -1.0,
                            extra={"solve_stages_s": dict(result.timing)})
            self.stats.append(st)
            log.info("layer %d done: %d linears + %d experts | rel_err med=%.4f max=%.4f | capture %.1fs "
                     "solve %.1fs reforward %.1fs total %.1fs", li, n_lin, n_exp, st.rel_err_median,
                     st.rel_err_max, st.capture_s, st.solve_s, st.reforward_s, st.total_s)
        log.info("%d layers done in %.1f min", n_layers, (time.time() - t_start) / 60)
        return batches
