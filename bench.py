"""Benchmark: GPTQ-solved weight elems/s (Hessian -> codes) on B200, 1 to 8 GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...

Workload at every N ("C3"): one MoE layer's routed expert
batch solved to MXFP4 (groupwise). 128 experts, gate_up [1536, 2048] and down
[2048, 768] bf16 ~ N(0, 0.02); X [524288, 2048] bf16 ~ N(0, 1); a top-8 router with
N(0, 1) logits plus a Zipf(1.1) bias (scaled until one expert gets no token);
down inputs silu(x Wg^T) * (x Wu^T) per routed slot (4,194,304 slots). One step =
grouped tcgen05 Hessians of every expert (gate_up over X rows, down over the slot
activations), damped 32x32 block factors, the MXFP4 column loops writing
nibble-packed codes, E8M0 scales, bf16 W_dq and rel_err, data-free RTN for the
experts without tokens, and (N > 1) the exchange: per parameter, every rank pushes
its experts' codes and scales into every peer's symmetric buffer with copy-engine
copies over NVLink (an all-gather without SM work, closed by a one-element NCCL
all-reduce), so every rank ends the step with every expert's outputs.
Under torchrun the experts are split over the ranks by longest processing time
(strong scaling: the batch is fixed, `value` = the batch's elements / step time,
max over ranks). Inputs (2.1 GB of X, 6.4 GB of slot activations) exceed the
126 MB L2, so no flush is needed between steps.

`value` is device-resident throughput (inputs already in HBM). `e2e` is the same
step through the package calls with this rank's inputs copied from pinned host
memory every step (the reference also moves its stashes host -> device,
capture.py:68-76) and every expert's codes and scales read back.

At N = 1 the line also carries the other configurations (`configs`: C1 affine,
C2 MXFP4 safe-scale-search, C4 MXFP8), a standalone packing kernel, rooflines of
the dominant kernels, and `cpu_baseline`: the numpy restatement of the reference
timed on a proportional sample of the same step (1/32 of every expert's routed rows
and of every expert's weight rows, a real run, not an extrapolation).
`--impl reference` times that same sample as the reference arm.

--workload c2 runs the previous default (C2 replicas, one per rank). --config c5
calibrates a synthetic Qwen3-30B-A3B-shaped layer stack layer by layer.
--profile-case NAME runs one small kernel case for an ncu capture.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mlx-gptq-mxfp_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "GPTQ-solved weight elems/s (Hessian->codes)"
C3_WORKLOAD = ("C3 MoE expert batch: 128 experts, gate_up [1536,2048] + down [2048,768] bf16, X [524288,2048], "
               "Zipf(1.1) top-8 routing (4,194,304 slots, >= 1 expert without tokens -> RTN); MXFP4 groupwise")
C2_WORKLOAD = ("C2 dense MLP sweep: gate/up [11008,4096] share H(K=4096), down [4096,11008] H(K=11008); "
               "X [131072,K] bf16 Student-t(4), 1% channels x30; MXFP4 safe-scale-search")
CPU_SAMPLE = 32  # the CPU sample keeps 1 of every CPU_SAMPLE routed rows and weight rows


def peaks():
    """(sustained bf16 TFLOP/s, burst bf16 TFLOP/s, HBM GB/s, source)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return p["bf16_tflops_sustained"], p["bf16_tflops"], p["hbm_gbs"], "measured"
    return 1400.0, 1590.0, 6650.0, "fallback"


def dist_env():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def hessian_executed_elems(c: int) -> int:
    """Output elements the 2-SM Hessian kernel computes per H: 256 x 256 tiles on or
    above the diagonal (the rest is mirrored); 128 x 256 tiles with GQ_HESSIAN_KERNEL=1sm."""
    if os.environ.get("GQ_HESSIAN_KERNEL", "2sm").startswith("1"):
        mt, nt = -(-c // 128), -(-c // 256)
        return 128 * 256 * sum(min(2 * tn + 2, mt) for tn in range(nt))
    t = -(-c // 256)
    return 256 * 256 * t * (t + 1) // 2


def _ev():
    return torch.cuda.Event(enable_timing=True)


def _blas_threads() -> int:
    """Threads numpy's BLAS runs with (what the CPU timings actually used)."""
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else 1
    except Exception:  # threadpoolctl missing: numpy's default is every core
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# C3: the routed expert batch, split over ranks
# ---------------------------------------------------------------------------
C3_EXPERTS, C3_H, C3_I = 128, 2048, 768
C3_ELEMS = C3_EXPERTS * (2 * C3_I * C3_H + C3_H * C3_I)


class C3Inputs:
    """This rank's share of the C3 batch, resident on the device: all of X (every rank
    holds the layer input), its experts' weights, routed token ids and down-projection
    activations."""

    def __init__(self, device, rank: int, world: int):
        from mlx_gptq_b200 import synthetic as S
        from mlx_gptq_b200.expert_batch import plan_experts

        X, gate_up, down, routing, acts = S.c3_inputs(device)
        self.counts = routing.counts.tolist()
        self.zero_experts = routing.zero_experts
        self.bias_scale = routing.bias_scale
        self.shares = plan_experts(self.counts, world, (C3_H, C3_I), 2 * C3_I * C3_H + C3_H * C3_I)
        self.mine = self.shares[rank]
        mine = torch.tensor(self.mine, dtype=torch.long, device=device)
        off = routing.offsets.tolist()
        self.X = X
        self.W_gu = gate_up.index_select(0, mine).contiguous()
        self.W_dn = down.index_select(0, mine).contiguous()
        tok = [routing.token_idx[off[e]:off[e + 1]] for e in self.mine]
        self.tok = torch.cat(tok) if tok else torch.zeros(0, dtype=torch.int32, device=device)
        rows = [acts[off[e]:off[e + 1]] for e in self.mine]
        self.acts = torch.cat(rows) if rows else torch.zeros(0, C3_I, dtype=torch.bfloat16, device=device)
        self.offsets = torch.zeros(len(self.mine) + 1, dtype=torch.int64)
        self.offsets[1:] = torch.cumsum(torch.tensor([self.counts[e] for e in self.mine], dtype=torch.int64), 0)
        self.counts_mine = [self.counts[e] for e in self.mine]
        self.hess_flop = sum(2.0 * n * (C3_H * C3_H + C3_I * C3_I) for n in self.counts_mine)
        self.hess_flop_gu = sum(2.0 * n * C3_H * C3_H for n in self.counts_mine)
        del gate_up, down, acts, routing

    def host_copy(self):
        """Pinned host copies of the step's inputs (the e2e leg)."""
        return {k: getattr(self, k).cpu().pin_memory() for k in ("X", "W_gu", "W_dn", "tok", "acts")}


class C3Step:
    """One step of the C3 batch on this rank (see the module docstring)."""

    def __init__(self, inp: C3Inputs, device, rank: int, world: int, group=None):
        from mlx_gptq_b200.expert_batch import Exchange, piece_layout

        self.inp, self.device, self.world = inp, device, world
        n = len(inp.mine)
        self.lay_gu = piece_layout(inp.tok, inp.offsets, list(range(n)), C3_H, device)
        # down inputs are laid out expert by expert: read in place as spans
        self.lay_dn = piece_layout(None, inp.offsets, list(range(n)), C3_I, device)
        self.H_gu = torch.empty(self.lay_gu.offsets.numel() - 1, C3_H, C3_H, device=device)
        self.H_dn = torch.empty(self.lay_dn.offsets.numel() - 1, C3_I, C3_I, device=device)
        self.exchange = Exchange(inp.shares, rank, group, device) if world > 1 else None
        self.all_out = None
        if world > 1:  # every expert's codes and scales on every rank, rank-major (Exchange)
            ex, u8 = self.exchange, torch.uint8
            self.all_out = {"codes_gu": ex.buffer((2 * C3_I, C3_H // 2), u8),
                            "scales_gu": ex.buffer((2 * C3_I, C3_H // 32), u8),
                            "codes_dn": ex.buffer((C3_H, C3_I // 2), u8),
                            "scales_dn": ex.buffer((C3_H, C3_I // 32), u8)}
        self.events = None
        self.last = None

    def launches(self) -> int:
        """Kernels of this library per step: per parameter the row pass (gate_up: the
        routed-row gather; down: the partial-step tails) and the Hessian, the piece merge
        when an expert was cut into pieces, dead columns, block factors, column loop,
        rel_err reduction, and RTN when this rank has experts without tokens."""
        rtn = 1 if any(c == 0 for c in self.inp.counts_mine) else 0
        merges = sum(1 for lay in (self.lay_gu, self.lay_dn) if lay.extra)
        return 2 * (2 + 4 + rtn) + merges

    def run(self, record: bool = False, X=None, W_gu=None, W_dn=None, acts=None, tok=None, ready=None):
        from mlx_gptq_b200.expert_batch import expert_hessians
        from mlx_gptq_b200.layer import solve_experts

        inp = self.inp
        X = inp.X if X is None else X
        ev = [_ev() for _ in range(6)] if record else None
        if ready is not None:
            torch.cuda.current_stream(self.device).wait_event(ready[0])
        if tok is not None and self.lay_gu.perm.numel():  # token ids copied this step: lay them out
            self.lay_gu.token_idx = tok.index_select(0, self.lay_gu.perm)
        if record:
            ev[0].record()
        H = expert_hessians(X, self.lay_gu, out=self.H_gu)
        if record:
            ev[1].record()
        gu = solve_experts(inp.W_gu if W_gu is None else W_gu, H, inp.counts_mine, "mxfp4", "groupwise",
                           torch.bfloat16, want_rel=True, check_info=False)
        if record:
            ev[2].record()
        if self.exchange is not None:
            self.exchange.start(gu.codes, self.all_out["codes_gu"])
            self.exchange.start(gu.scales, self.all_out["scales_gu"])
        if ready is not None:
            torch.cuda.current_stream(self.device).wait_event(ready[1])
        H = expert_hessians(inp.acts if acts is None else acts, self.lay_dn, out=self.H_dn)
        if record:
            ev[3].record()
        dn = solve_experts(inp.W_dn if W_dn is None else W_dn, H, inp.counts_mine, "mxfp4", "groupwise",
                           torch.bfloat16, want_rel=True, check_info=False)
        if record:
            ev[4].record()
        if self.exchange is not None:
            self.exchange.start(dn.codes, self.all_out["codes_dn"])
            self.exchange.start(dn.scales, self.all_out["scales_dn"])
            self.exchange.wait()
        if record:
            ev[5].record()
        self.events = ev
        self.last = (gu, dn)
        return gu, dn

    def outputs(self):
        """Every expert's codes and scales after the step (this rank's when N = 1)."""
        gu, dn = self.last
        if self.all_out is not None:
            return [self.exchange.expert_order(self.all_out[k]) for k in ("codes_gu", "scales_gu", "codes_dn",
                                                                          "scales_dn")]
        return [gu.codes, gu.scales, dn.codes, dn.scales]


class C3E2E:
    """The C3 step with this rank's inputs copied from pinned host memory on a side
    stream every step (X, gate_up weights and token ids first; down activations and
    weights second, overlapping the gate_up stage) and this rank's results read back.

    X, the layer input every rank needs, crosses PCIe once per step in all: with N
    ranks each copies 1/N of its rows and one all-gather over NVLink assembles it on
    every rank (the host link is the slow one). Each rank reads back the codes and
    scales of its own experts (sharded artifacts; the exchange still hands every rank
    every expert's outputs for the next layer)."""

    def __init__(self, step: C3Step, rank: int, world: int, group=None):
        self.step, self.device, self.rank, self.world, self.group = step, step.device, rank, world, group
        self.host = step.inp.host_copy()
        T = self.host["X"].shape[0]
        self.rows = T // world if world > 1 and T % world == 0 else None
        if self.rows is not None:  # only this rank's slice of X is copied from the host
            self.host["X"] = self.host["X"][rank * self.rows:(rank + 1) * self.rows].clone().pin_memory()
            self.x_full = torch.empty(T, self.host["X"].shape[1], dtype=torch.bfloat16, device=self.device)
        self.dev = {k: torch.empty_like(v, device=self.device) for k, v in self.host.items()}
        self.cs = torch.cuda.Stream(self.device)
        self.h2d_bytes = sum(v.numel() * v.element_size() for v in self.host.values())
        self.out_host = None
        self.d2h_bytes = 0

    def run(self):
        ms = torch.cuda.current_stream(self.device)
        self.cs.wait_stream(ms)  # the previous step has finished with the device buffers
        ready = []
        with torch.cuda.stream(self.cs):
            for group in (("X", "W_gu", "tok"), ("acts", "W_dn")):
                for k in group:
                    self.dev[k].copy_(self.host[k], non_blocking=True)
                e = torch.cuda.Event()
                e.record(self.cs)
                ready.append(e)
        X = self.dev["X"]
        if self.rows is not None:
            import torch.distributed as dist

            ms.wait_event(ready[0])
            dist.all_gather_into_tensor(self.x_full, self.dev["X"], group=self.group)
            X = self.x_full
            ready[0] = torch.cuda.Event()
            ready[0].record(ms)
        self.step.run(X=X, W_gu=self.dev["W_gu"], W_dn=self.dev["W_dn"], acts=self.dev["acts"],
                      tok=self.dev["tok"], ready=ready)
        gu, dn = self.step.last
        outs = [gu.codes, gu.scales, dn.codes, dn.scales]  # this rank's experts
        if self.out_host is None:
            self.out_host = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs]
            self.d2h_bytes = sum(o.numel() * o.element_size() for o in outs)
        for h, o in zip(self.out_host, outs):
            h.copy_(o, non_blocking=True)


# ---------------------------------------------------------------------------
# the CPU side: the numpy restatement of the reference on a proportional sample
# ---------------------------------------------------------------------------
class C3CpuSample:
    """1/CPU_SAMPLE of the C3 step, on the host: the first ceil(N_e / CPU_SAMPLE) routed
    rows of every expert for its Hessians (X rows for gate_up, slot activations for
    down) and every CPU_SAMPLE-th weight row of every expert for its solve (GPTQ rows
    are independent given H, so a row subset is an exact sub-problem). Every expert,
    heavy or light, is in the sample, so its mix of Hessian and solve work is the
    full step's."""

    def __init__(self, device):
        from mlx_gptq_b200 import synthetic as S

        X, gate_up, down, routing, acts = S.c3_inputs(device)
        off = routing.offsets.tolist()
        self.counts = routing.counts.tolist()
        self.x_gu, self.x_dn = [], []
        for e, n in enumerate(self.counts):
            k = -(-n // CPU_SAMPLE)
            idx = routing.token_idx[off[e]:off[e] + k].long()
            self.x_gu.append(X.index_select(0, idx).float().cpu().numpy())
            self.x_dn.append(acts[off[e]:off[e] + k].float().cpu().numpy())
        self.W_gu = gate_up[:, ::CPU_SAMPLE].float().cpu().numpy()
        self.W_dn = down[:, ::CPU_SAMPLE].float().cpu().numpy()
        self.elems = self.W_gu.size + self.W_dn.size
        del X, gate_up, down, acts

    def run(self):
        from oracle import gptq as ogptq
        from oracle import grid as ogrid
        from oracle import hessian as ohess

        zero = [e for e, n in enumerate(self.counts) if n == 0]
        for xs, W in ((self.x_gu, self.W_gu), (self.x_dn, self.W_dn)):
            C = W.shape[-1]
            H = np.stack([ohess.hessian(x) if x.shape[0] else np.zeros((C, C), np.float32) for x in xs])
            ogptq.solve_gptq(W, H, 4, 32, mode="mxfp4", mxfp_algorithm="groupwise")
            if zero:
                ogrid.rtn_quantize_mxfp(W[zero], "mxfp4")


def time_cpu_sample(sample: C3CpuSample, reps: int):
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        sample.run()
        ts.append(time.perf_counter() - t0)
    return ts


def cpu_sample_record(sample: C3CpuSample, secs: list[float]) -> dict:
    t = statistics.median(secs)
    return {"value": sample.elems / t, "unit": "elems/s", "cores": _blas_threads(), "kind": "port",
            "sample": (f"numpy restatement of the reference (oracle/), timed as run: 1/{CPU_SAMPLE} of the C3 step "
                       f"= the first ceil(N_e/{CPU_SAMPLE}) routed rows of every expert (Hessians) and every "
                       f"{CPU_SAMPLE}th weight row of every expert (MXFP4 groupwise solves, {sample.elems} elems), "
                       f"median of {len(secs)} runs of {t:.2f} s; numpy BLAS threads = cores"),
            "seconds_per_sample": t}


def run_reference_arm(args, ws, rank):
    """The reference's CPU path (its numpy restatement) on the host cores: the C3 sample
    per step, K timed steps after W warm-up ones. At N > 1 rank 0 alone runs it (the
    reference's CPU path uses no GPU); the other ranks exit without work."""
    if rank != 0:
        return
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    sample = C3CpuSample(dev)
    if dev == "cuda":
        torch.cuda.empty_cache()
    time_cpu_sample(sample, args.warmup)
    t0 = time.perf_counter()
    secs = time_cpu_sample(sample, args.steps)
    total = time.perf_counter() - t0
    rec = cpu_sample_record(sample, secs)
    v = sample.elems * args.steps / total
    rec["value"] = v
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "elems/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": C3_WORKLOAD, "sample": f"1/{CPU_SAMPLE} of every expert's rows (see cpu_baseline)",
                       "parallelism": "host cores (the reference's CPU path uses no GPU; the same at every N)"},
            "cpu_baseline": rec,
            "e2e": {"value": v, "unit": "elems/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the other configurations at N = 1
# ---------------------------------------------------------------------------
def _timed(fn, steps: int, warmup: int):
    """Mean ms of fn() over `steps` launches after `warmup`, CUDA events on the current stream."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = _ev(), _ev()
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / steps


def extra_c2(device, steps, warmup, peak_tf, peak_hbm, src):
    """C2 (configs[1], seed 0): both Hessians + factors + the three MXFP4
    safe-scale-search column loops."""
    from mlx_gptq_b200 import hessian_accumulate
    from mlx_gptq_b200 import synthetic as S
    from mlx_gptq_b200.layer import mxfp_factors, solve_mxfp_packed

    wl = S.c2_inputs(0, device)
    H_gu = torch.empty(4096, 4096, device=device)
    H_dn = torch.empty(11008, 11008, device=device)
    ev = {}

    def step(record=False):
        e = [_ev() for _ in range(4)] if record else None
        if record:
            e[0].record()
        hessian_accumulate(wl["X_gu"], H_gu, 1.0, 0.0)
        if record:
            e[1].record()
        hessian_accumulate(wl["X_down"], H_dn, 1.0, 0.0)
        if record:
            e[2].record()
        f_gu, f_dn = mxfp_factors(H_gu.unsqueeze(0)), mxfp_factors(H_dn.unsqueeze(0))
        for name, f in (("gate", f_gu), ("up", f_gu), ("down", f_dn)):
            solve_mxfp_packed(wl[name], f, "mxfp4", "safe-scale-search", torch.bfloat16, True, check_info=False)
        if record:
            e[3].record()
            ev.setdefault("steps", []).append(e)

    ms = _timed(step, steps, warmup)
    step(record=True)
    for _ in range(2):
        step(record=True)
    torch.cuda.synchronize()
    big = statistics.mean(e[1].elapsed_time(e[2]) for e in ev["steps"])
    solve = statistics.mean(e[2].elapsed_time(e[3]) for e in ev["steps"])
    elems = 3 * 11008 * 4096
    flop_big = 2.0 * 131072 * 11008 ** 2
    ach = flop_big / (big / 1e3) / 1e12
    col_bytes = sum(r * c * 4.5 + r * c // 32 + 4 * 32 * c for r, c in ((11008, 4096),) * 2 + ((4096, 11008),))
    return {"workload": C2_WORKLOAD + " (seed 0)", "value": elems / (ms / 1e3), "unit": "elems/s",
            "ms_per_step": ms, "hessian_ms_k11008": big, "factors_and_solves_ms": solve,
            "roofline_hessian": {"kernel": "hessian2_kernel (K=11008)", "bound": "tensor", "achieved": ach,
                                 "peak": peak_tf, "unit": "TFLOP/s", "frac": ach / peak_tf,
                                 "executed_frac": 2.0 * 131072 * hessian_executed_elems(11008) / (big / 1e3) / 1e12
                                 / peak_tf, "peak_source": f"{src} bf16_tflops_sustained"},
            "roofline_column_loop": {"kernel": "mx_gptq_kernel x3 (+ factors)", "bound": "compute (FP32 + tensor)",
                                     "achieved": col_bytes / (solve / 1e3) / 1e9, "peak": peak_hbm, "unit": "GB/s",
                                     "frac": col_bytes / (solve / 1e3) / 1e9 / peak_hbm,
                                     "bytes_per_step": col_bytes, "peak_source": f"{src} hbm_gbs"}}


def trailing_update_roofline(device, steps, peak_hbm, src):
    """The affine trailing update W[:, i2:] -= Err U[i1:i2, i2:] alone (tc_gemm_kernel through
    the gq_gemm_f32 hook, the engine solve_gptq uses) at a C1-sized block: M = 4096 rows,
    N = 3072 columns, K = 128; W rotates over four 64 MB matrices so the slice is not
    L2-resident between launches. HBM roofline on the W slice read and written once."""
    import ctypes

    from mlx_gptq_b200 import _lib as L

    R, C, K, i2 = 4096, 4096, 128, 1024
    N = C - i2
    g = torch.Generator(device=device).manual_seed(3)
    Ws = [torch.randn(R, C, generator=g, device=device) for _ in range(4)]
    Err = torch.randn(R, K, generator=g, device=device) * 1e-3
    Ub = torch.randn(K, C, generator=g, device=device)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    it = [0]

    def launch():
        W = Ws[it[0] % 4]
        it[0] += 1
        L.check(L.lib().gq_gemm_f32(p(Err), p(Ub[:, i2:]), p(W[:, i2:]), R, N, K, K, C, C, 0, 0, 1, 1, 0, 0, 0, 0, 0, 0,
                                    -1.0, 1.0, None, 1, L.ptr(L.status_word(device)), L.stream_ptr(device)),
                "trailing update")

    ms = _timed(launch, steps, 4)
    L.raise_on_device_timeout(device)
    nbytes = 2.0 * R * N * 4
    return {"kernel": "tc_gemm_kernel (tcgen05 kind::tf32 3xTF32, TMA reduce-add into W), M 4096 N 3072 K 128",
            "bound": "hbm", "achieved": nbytes / (ms / 1e3) / 1e9, "peak": peak_hbm, "unit": "GB/s",
            "frac": nbytes / (ms / 1e3) / 1e9 / peak_hbm, "bytes_per_launch": nbytes, "ms_per_launch": ms,
            "tflops": 2.0 * R * N * K / (ms / 1e3) / 1e12, "peak_source": f"{src} hbm_gbs",
            "l2": "W rotates over four 64 MB matrices (256 MB > L2)"}


def extra_c1(device, steps, warmup, peak_tf, src):
    """C1: H from X [524288, 4096], then solve_gptq affine 4-bit g64 mse
    (factor, column loop, lazy trailing update)."""
    from mlx_gptq_b200 import hessian_accumulate, solve_gptq
    from mlx_gptq_b200 import synthetic as S

    W, X = S.c1_inputs(device)
    Wf = W.float().unsqueeze(0)
    H = torch.empty(4096, 4096, device=device)
    hess_ms = _timed(lambda: hessian_accumulate(X, H, 1.0, 0.0), steps, warmup)
    Hb = H.unsqueeze(0)
    solve_ms = _timed(lambda: solve_gptq(Wf, Hb.clone(), 4, 64, mode="affine"), max(2, steps // 2), 1)
    del X
    trailing = sum(2.0 * 4096 * 128 * (4096 - i2) for i2 in range(128, 4096, 128))
    flop = 2.0 * 524288 * 4096 ** 2
    return {"workload": "C1 dense linear: W [4096,4096], X [524288,4096] 16 outlier channels x20; affine 4b g64 mse",
            "value": 4096 * 4096 / ((hess_ms + solve_ms) / 1e3), "unit": "elems/s",
            "ms_per_step": hess_ms + solve_ms, "hessian_ms": hess_ms, "solve_ms": solve_ms,
            "roofline_hessian": {"achieved": flop / (hess_ms / 1e3) / 1e12, "peak": peak_tf, "unit": "TFLOP/s",
                                 "frac": flop / (hess_ms / 1e3) / 1e12 / peak_tf},
            "roofline_affine": {"kernel": "gq_gptq_affine + gq_prepare_hinv (whole solve_gptq)",
                                "bound": "hbm (tcgen05 3xTF32 trailing update, TMA reduce-add into W) / latency (factor chain)",
                                "trailing_update_flop": trailing,
                                "achieved": trailing / (solve_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                                "note": "trailing-update FLOP over the whole solve's time (factor + column loop + "
                                        "trailing update): a lower bound on the GEMM's own rate"}}


def extra_c4(device, steps, warmup):
    """C4: Hessians of X_qkv [262144, 2048] and X_o [262144, 4096], MXFP8
    groupwise solves of q / k / v / o."""
    from mlx_gptq_b200 import hessian_accumulate
    from mlx_gptq_b200 import synthetic as S
    from mlx_gptq_b200.layer import mxfp_factors, solve_mxfp_packed

    wl = S.c4_inputs(device)
    Hq = torch.empty(2048, 2048, device=device)
    Ho = torch.empty(4096, 4096, device=device)

    def step():
        hessian_accumulate(wl["X_qkv"], Hq, 1.0, 0.0)
        hessian_accumulate(wl["X_o"], Ho, 1.0, 0.0)
        fq, fo = mxfp_factors(Hq.unsqueeze(0)), mxfp_factors(Ho.unsqueeze(0))
        for n in ("q_proj", "k_proj", "v_proj"):
            solve_mxfp_packed(wl[n], fq, "mxfp8", "groupwise", torch.bfloat16, True, check_info=False)
        solve_mxfp_packed(wl["o_proj"], fo, "mxfp8", "groupwise", torch.bfloat16, True, check_info=False)

    ms = _timed(step, steps, warmup)
    elems = 4096 * 2048 + 2 * 512 * 2048 + 2048 * 4096
    return {"workload": "C4 attention: q [4096,2048], k/v [512,2048] share H(K=2048), o [2048,4096] H(K=4096); "
                        "X [262144,K] N(0,1) x LogNormal(0,0.5); MXFP8 groupwise",
            "value": elems / (ms / 1e3), "unit": "elems/s", "ms_per_step": ms,
            "hessian_tflop": (2.0 * 262144 * (2048 ** 2 + 4096 ** 2)) / 1e12}


def extra_pack(device, peak_hbm, src, codes: torch.Tensor):
    """Stage B's uint32 word packing (gq_pack_q, packing.py:15-39) of the C3 batch's
    MXFP4 codes: algorithmic bytes R*C*(1 + bits/8) per launch."""
    from mlx_gptq_b200 import _lib as L

    q = codes
    rows, C = q.numel() // q.shape[-1], q.shape[-1]
    out = torch.empty(rows, C // 8, dtype=torch.int32, device=device)

    def launch():
        L.check(L.lib().gq_pack_q(q.data_ptr(), rows, C, 4, out.data_ptr(), L.stream_ptr(device)), "pack_q")

    ms = _timed(launch, 20, 3)
    nbytes = rows * C * 1.5
    ach = nbytes / (ms / 1e3) / 1e9
    return {"kernel": "pack_q_kernel (4-bit, C3 codes [128 x 3584 rows, 2048/768 cols as one batch])",
            "bound": "hbm", "achieved": ach, "peak": peak_hbm, "unit": "GB/s", "frac": ach / peak_hbm,
            "bytes_per_launch": nbytes, "ms_per_launch": ms, "peak_source": f"{src} hbm_gbs (burst copy)"}


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi samples every 50 ms from before the warm-up on; the summary keeps the
    samples whose timestamps fall inside the timed region (begin()/end())."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        deadline = time.time() + 5.0
        while time.time() < deadline and os.path.getsize(self.path) == 0:  # first sample written
            time.sleep(0.02)

    def begin(self):
        self.t0 = time.time()

    def end(self):
        self.t1 = time.time()

    @staticmethod
    def _when(stamp: str):
        import datetime

        try:
            return datetime.datetime.strptime(stamp.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10:
                rows.append((self._when(parts[0]), parts[1:]))
        os.unlink(self.path)
        if not rows:
            return None
        inside = rows
        if self.t0 is not None and self.t1 is not None:
            inside = [r for r in rows if r[0] is not None and self.t0 - 0.06 <= r[0] <= self.t1 + 0.06]
            if not inside:  # a region shorter than the sampling period: the nearest sample after it began
                after = [r for r in rows if r[0] is not None and r[0] >= self.t0]
                inside = after[:1] or rows[-1:]
        rows = [r[1] for r in inside]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}



# ---------------------------------------------------------------------------
# C5: Qwen3-30B-A3B-shaped MoE layer stack, layer-sequential, experts sharded over ranks
# ---------------------------------------------------------------------------
QWEN3_30B_A3B = dict(model_type="qwen3_moe", vocab_size=151936, hidden_size=2048, intermediate_size=6144,
                     moe_intermediate_size=768, num_hidden_layers=48, num_attention_heads=32,
                     num_key_value_heads=4, head_dim=128, num_experts=128, num_experts_per_tok=8,
                     decoder_sparse_step=1, norm_topk_prob=True, rms_norm_eps=1e-6, rope_theta=1e6,
                     max_position_embeddings=40960, tie_word_embeddings=False, hidden_act="silu")


def run_c5(args, ws, rank, local):
    """Synthetic Qwen3-30B-A3B stack (random init, seed 0; 256 x 2048 uniform tokens,
    seed 1) calibrated layer by layer to MXFP4 (safe-scale-search) through the
    package's Pipeline. By default every rank runs the layer forwards and the solves are
    split across ranks (one exchange of packed codes per task); with --c5-dp each rank
    forwards its share of the windows and Hessians are summed over ranks. Reports the
    solve stage (Hessians, factors, column loops, exchange) and the whole layer time, max
    over ranks."""
    import types

    from mlx_gptq_b200 import sequential

    device = torch.device("cuda", local)
    group = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
        group = dist.group.WORLD
    cfg = dict(QWEN3_30B_A3B)
    model = sequential.build_model(cfg)
    src = sequential.SyntheticWeights(model, device, seed=0)
    sargs = types.SimpleNamespace(devices=[str(device)], dtype="bfloat16", layers_attr="model.layers",
                                  checkpoint_model_prefix=None, artifact_layers_prefix=None,
                                  exclude=sequential.DEFAULT_EXCLUDE, group_size=32, bits=4, mode="mxfp4",
                                  mxfp_algorithm="safe-scale-search", damp=0.01, clip="mse", overrides=[],
                                  batch_size=args.c5_batch, experts_forward=args.c5_experts_forward)
    g = torch.Generator().manual_seed(1)
    samples = torch.randint(0, cfg["vocab_size"], (args.c5_samples, args.c5_seqlen), generator=g)
    pipe = sequential.Pipeline(model, src, sargs, group=group, dp=args.c5_dp)
    t0 = time.time()
    pipe.run(samples, writer=None, layers=args.layers)
    torch.cuda.synchronize()
    wall = time.time() - t0
    def stages(st):
        d = st.extra.get("solve_stages_s", {})
        return [d.get("expert_rows", 0.0) + d.get("expert_hessians", 0.0) + d.get("expert_solves", 0.0),
                d.get("linears", 0.0), d.get("all_gather", 0.0)]

    mid = len(pipe.stats) // 2
    my_mid = {k: round(v * 1e3, 2) for k, v in pipe.stats[mid].extra.get("solve_stages_s", {}).items()}
    per_rank_mid = [my_mid]
    if group is not None:
        import torch.distributed as dist

        per_rank_mid = [None] * ws
        dist.all_gather_object(per_rank_mid, my_mid, group=group)

    rows = [[s.capture_s, s.solve_s, s.reforward_s, s.total_s] + stages(s) for s in pipe.stats]
    t = torch.tensor(rows + [[wall, 0, 0, 0, 0, 0, 0]], dtype=torch.float64, device=device)
    if group is not None:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.destroy_process_group()
    if rank != 0:
        return
    t = t.cpu().tolist()
    per_layer, wall = t[:-1], t[-1][0]
    elems = sum(s.solved_elems for s in pipe.stats)
    solve_s = sum(r[1] for r in per_layer[1:]) or per_layer[0][1]  # layer 0 carries one-time set-up
    n_solve = max(1, len(per_layer) - 1) if len(per_layer) > 1 else 1
    elems_timed = elems / len(per_layer) * n_solve
    tokens = args.c5_samples * args.c5_seqlen
    H, I, E, k = cfg["hidden_size"], cfg["moe_intermediate_size"], cfg["num_experts"], cfg["num_experts_per_tok"]
    qd, kvd = cfg["num_attention_heads"] * cfg["head_dim"], cfg["num_key_value_heads"] * cfg["head_dim"]
    hess_flop = 2.0 * tokens * (H * H + qd * qd) + 2.0 * tokens * k * (H * H + I * I)
    line = {"metric": "C5 layer stack: GPTQ-solved weight elems/s (solve stage: Hessians -> codes, all-gather)",
            "value": elems_timed / solve_s, "unit": "elems/s", "n_gpus": ws, "layers": len(per_layer),
            "higher_is_better": True, "scaling": "strong (one layer's experts split over ranks)" + (
                ", windows split over ranks (dp)" if args.c5_dp else ", forward on every rank"),
            "dtype": "bf16 x bf16 -> f32 (Hessian), f32 (solve)", "data": "synthetic (random init seed 0, "
            "uniform tokens seed 1)",
            "config": {"workload": "C5 Qwen3-30B-A3B-shaped stack, MXFP4 safe-scale-search",
                       "tokens": tokens, "batch_size": args.c5_batch,
                       "experts_forward": {"grouped": "sort-based, bit-identical to the eager loop",
                                           "eager": "eager F.linear loop"}[args.c5_experts_forward],
                       "artifacts": "kept on the device, not written to disk"},
            "solved_elems_per_layer": elems // len(per_layer),
            "stack_elems_per_s": elems_timed / sum(r[3] for r in (per_layer[1:] or per_layer)),
            "layer_ms_mean": statistics.mean(r[3] for r in (per_layer[1:] or per_layer)) * 1e3,
            "hessian_tflop_per_layer": hess_flop / 1e12,
            "solve_ms_per_layer": solve_s / n_solve * 1e3,
            "layer_s": [round(r[3], 3) for r in per_layer],
            "capture_s": [round(r[0], 3) for r in per_layer],
            "solve_s": [round(r[1], 3) for r in per_layer],
            "reforward_s": [round(r[2], 3) for r in per_layer],
            "wall_s": wall,
            "expert_stage_ms_per_layer": statistics.mean(r[4] for r in per_layer[1:] or per_layer) * 1e3,
            "linears_ms_per_layer": statistics.mean(r[5] for r in per_layer[1:] or per_layer) * 1e3,
            "all_gather_ms_per_layer": statistics.mean(r[6] for r in per_layer[1:] or per_layer) * 1e3,
            "solve_stages_ms_per_rank_layer_mid": per_rank_mid,
            "stage_note": "max over ranks per layer; expert stage = grouped expert Hessians + batched "
                          "expert solves; layer 0 (one-time set-up) excluded from the means",
            "rel_err_median": [round(s.rel_err_median, 5) for s in pipe.stats],
            "rel_err_max": [round(s.rel_err_max, 5) for s in pipe.stats]}
    print(json.dumps(line), flush=True)




# ---------------------------------------------------------------------------
# small cases for ncu captures
# ---------------------------------------------------------------------------
def profile_case(case, device):
    """Small, self-contained launches for ncu captures (a few launches, inputs > L2)."""
    from mlx_gptq_b200 import hessian_accumulate, hessian_grouped, layer, solve_gptq
    from mlx_gptq_b200 import synthetic as S
    from mlx_gptq_b200.gptq import _prepare_hinv

    def show(name, fn, n=3, units=None):
        for i in range(n):
            a, b = _ev(), _ev()
            a.record()
            fn()
            b.record()
            b.synchronize()
            ms = a.elapsed_time(b)
            print(f"{name} launch {i}: {ms:.3f} ms" + (f", {units(ms)}" if units else ""))

    if case in ("hessian", "hessian-full"):
        n, k = (16384, 4096) if case == "hessian" else (131072, 11008)
        X = S.student_t_bf16(n, k, 7, device)
        H = torch.empty(k, k, device=device)
        show(f"hessian N={n} C={k}", lambda: hessian_accumulate(X, H, 1.0, 0.0), 4,
             lambda ms: f"{2.0 * n * k * k / ms / 1e9:.1f} TFLOP/s (2*N*C^2)")
    elif case == "solve":
        X = S.student_t_bf16(8192, 4096, 7, device)
        H = torch.empty(4096, 4096, device=device)
        hessian_accumulate(X, H, 1.0, 0.0)
        W = S.weights_bf16((11008, 4096), 8, device)
        f = layer.mxfp_factors(H.unsqueeze(0))
        show("solve [11008, 4096] safe-scale-search", lambda: layer.solve_mxfp_packed(
            W, f, "mxfp4", "safe-scale-search", torch.bfloat16, True, check_info=False), 4,
             lambda ms: f"{W.numel() / ms / 1e6:.2f} G elems/s")
    elif case == "affine":
        X = S.outlier_normal_bf16(32768, 4096, 7, device)
        H = torch.empty(4096, 4096, device=device)
        hessian_accumulate(X, H, 1.0, 0.0)
        W = S.weights_bf16((1, 4096, 4096), 8, device)
        show("affine factor C=4096", lambda: _prepare_hinv(H.unsqueeze(0).clone(), 0.01), 2)
        show("affine solve_gptq [4096, 4096] g64", lambda: solve_gptq(W, H.unsqueeze(0).clone(), 4, 64,
                                                                      mode="affine"), 2)
    elif case in ("moe", "moe-small"):
        T = 524288 if case == "moe" else 32768
        X = torch.randn(T, 2048, generator=torch.Generator(device=device).manual_seed(1),
                        device=device).to(torch.bfloat16)
        r = S.zipf_routing(T, 128, 8, device)
        H = torch.empty(128, 2048, 2048, device=device)
        flop = 2.0 * float(r.counts.double().sum()) * 2048 * 2048
        print(f"routed slots {int(r.offsets[-1])}, max {int(r.counts.max())}, zero {len(r.zero_experts)}")
        show("grouped hessian", lambda: hessian_grouped(X, r.token_idx, r.offsets, 128, H=H), 3,
             lambda ms: f"{flop / ms / 1e9:.1f} TFLOP/s (sum 2*N_e*C^2)")
        W = S.weights_bf16((128, 1536, 2048), 0, device)
        show("batched solve (128 experts gate_up, groupwise)",
             lambda: layer.solve_experts(W, H.clone(), r.counts.tolist(), "mxfp4", "groupwise", torch.bfloat16,
                                         True, check_info=False), 3)
    elif case == "solve-groupwise":
        X = S.student_t_bf16(8192, 2048, 7, device)
        H = torch.empty(2048, 2048, device=device)
        hessian_accumulate(X, H, 1.0, 0.0)
        W = S.weights_bf16((32, 1536, 2048), 8, device)  # 32 experts' gate_up: 200 MB bf16 in
        Hb = H.unsqueeze(0).repeat(32, 1, 1)
        f = layer.mxfp_factors(Hb)
        show("solve [32, 1536, 2048] groupwise", lambda: layer.solve_mxfp_packed(
            W, f, "mxfp4", "groupwise", torch.bfloat16, True, check_info=False), 4,
             lambda ms: f"{W.numel() / ms / 1e6:.2f} G elems/s")
    elif case == "c3-step":
        inp = C3Inputs(device, 0, 1)
        step = C3Step(inp, device, 0, 1)
        for _ in range(3):
            step.run()
        torch.cuda.synchronize()
    elif case == "pack":
        q = torch.randint(0, 16, (128 * 1536, 2048), dtype=torch.uint8, device=device)
        print(extra_pack(device, peaks()[2], peaks()[3], q))
    else:
        raise SystemExit(f"unknown profile case {case}")
    torch.cuda.synchronize()
    print(f"profile case {case} done")


# ---------------------------------------------------------------------------
# the default run: C3 at N ranks
# ---------------------------------------------------------------------------
def _max_over_ranks(x: float, pg, device) -> float:
    if pg is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def _per_rank(vals: list[float], pg, device, ws) -> list[list[float]]:
    if pg is None:
        return [vals]
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    out = [torch.empty_like(t) for _ in range(ws)]
    pg.all_gather(out, t)
    return [o.tolist() for o in out]


def c2_replicas(device, rank, ws, pg, steps):
    """Every rank solves its own copy of C2 (seed rank % 3), no collective: the previous
    default multi-GPU workload, kept as an extra key."""
    from mlx_gptq_b200 import hessian_accumulate
    from mlx_gptq_b200 import synthetic as S
    from mlx_gptq_b200.layer import mxfp_factors, solve_mxfp_packed

    wl = S.c2_inputs(rank % 3, device)
    H_gu, H_dn = torch.empty(4096, 4096, device=device), torch.empty(11008, 11008, device=device)

    def step():
        hessian_accumulate(wl["X_gu"], H_gu, 1.0, 0.0)
        hessian_accumulate(wl["X_down"], H_dn, 1.0, 0.0)
        f_gu, f_dn = mxfp_factors(H_gu.unsqueeze(0)), mxfp_factors(H_dn.unsqueeze(0))
        for name, f in (("gate", f_gu), ("up", f_gu), ("down", f_dn)):
            solve_mxfp_packed(wl[name], f, "mxfp4", "safe-scale-search", torch.bfloat16, True, check_info=False)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    ms = _max_over_ranks(_timed(step, steps, 0), pg, device)
    return {"workload": C2_WORKLOAD + ", one copy per rank (seed rank % 3), no collective",
            "value": ws * 3 * 11008 * 4096 / (ms / 1e3), "unit": "elems/s", "ms_per_step": ms, "scaling": "weak"}


def run_c3(args, ws, rank, local):
    from mlx_gptq_b200 import _lib as L

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    pg, group = None, None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        pg, group = dist, dist.group.WORLD
    args.warmup = max(args.warmup, 3)
    peak_tf, peak_burst, peak_hbm, src = peaks()

    inp = C3Inputs(device, rank, ws)
    step = C3Step(inp, device, rank, ws, group)
    torch.cuda.empty_cache()
    clocks = ClockSampler(local)
    clocks.start()  # sampling from before the warm-up; the summary keeps the timed region
    for _ in range(args.warmup):
        step.run()
    torch.cuda.synchronize()
    L.raise_on_device_timeout(device)
    gu, dn = step.last
    assert bool(torch.isfinite(gu.rel_err).all()) and bool(torch.isfinite(dn.rel_err).all())

    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    clocks.begin()
    t0, t1 = _ev(), _ev()
    evs = []
    t0.record()
    for _ in range(args.steps):
        step.run(record=True)
        evs.append(step.events)
    t1.record()
    torch.cuda.synchronize()
    clocks.end()
    if pg:
        pg.barrier()
    clk = clocks.stop()
    ms_step = _max_over_ranks(t0.elapsed_time(t1) / args.steps, pg, device)
    stage = [statistics.mean(e[i].elapsed_time(e[i + 1]) for e in evs) for i in range(5)]
    stages_by_rank = _per_rank(stage + [float(len(inp.mine)), float(sum(inp.counts_mine))], pg, device, ws)

    e2e = None
    if not args.no_e2e:
        leg = C3E2E(step, rank, ws, group)
        for _ in range(2):
            leg.run()
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        a, b = _ev(), _ev()
        n = max(3, args.steps // 4)
        a.record()
        for _ in range(n):
            leg.run()
        b.record()
        torch.cuda.synchronize()
        ms_e2e = _max_over_ranks(a.elapsed_time(b) / n, pg, device)
        e2e = {"value": C3_ELEMS / (ms_e2e / 1e3), "unit": "elems/s", "ms_per_step": ms_e2e,
               "h2d_bytes_per_step": leg.h2d_bytes, "d2h_bytes_per_step": leg.d2h_bytes,
               "note": "per rank: 1/N of X's rows host->device (all-gathered over NVLink), its experts' "
                       "weights, token ids and slot activations; its experts' codes + E8M0 scales device->host"}
        del leg
    reps = None if args.no_extras else c2_replicas(device, rank, ws, pg, 5) if ws > 1 else None
    outs = step.outputs()
    if pg:
        pg.destroy_process_group()
    if rank != 0:
        return

    hess_gu_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    ach = inp.hess_flop_gu / (hess_gu_ms / 1e3) / 1e12
    executed = sum(2.0 * n * hessian_executed_elems(C3_H) for n in inp.counts_mine) / (hess_gu_ms / 1e3) / 1e12
    roofline = {"kernel": "grouped Hessian, gate_up (gather_rows_kernel + hessian2_kernel, one call)",
                "bound": "tensor", "achieved": ach, "peak": peak_burst, "unit": "TFLOP/s", "frac": ach / peak_burst,
                "peak_source": f"{src} bf16_tflops (burst; the timed region is well under a second per kernel)",
                "flop_per_launch": inp.hess_flop_gu,
                "note": "algorithmic FLOP = sum_e 2*N_e*C^2 (the reference's full per-expert X^T X); the kernel "
                        "computes tiles on/above the diagonal and mirrors them (executed_* = MMA work issued); the "
                        "time includes the row-gather pass of the same call",
                "executed_tflops": executed, "executed_frac": executed / peak_burst,
                "frac_of_sustained": ach / peak_tf, "traffic": profile_traffic("c3_gate_up")}
    solve_ms = stage[1] + stage[3]
    col_bytes = C3_EXPERTS * sum(r * c * 4.5 + r * c // 32 + 4 * 32 * c for r, c in ((2 * C3_I, C3_H), (C3_H, C3_I)))
    line = {
        "metric": METRIC, "value": C3_ELEMS / (ms_step / 1e3), "unit": "elems/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 x bf16 -> f32 (Hessian), f32 (solve)",
        "data": "synthetic",
        "config": {"workload": C3_WORKLOAD, "elems_per_step": C3_ELEMS, "tokens": 524288,
                   "zero_token_experts": inp.zero_experts, "zipf_bias_scale": inp.bias_scale,
                   "l2": "inputs larger than L2 (X 2.1 GB, slot activations 6.4 GB); no flush",
                   "parallelism": (f"experts split over {ws} ranks (LPT); per parameter codes + scales pushed to "
                                   "every rank (copy engines into symmetric buffers, NCCL all-reduce to close) "
                                   "inside the step" if ws > 1 else "1 GPU")},
        "hessian_tflops": sum(2.0 * n * (C3_H ** 2 + C3_I ** 2) for n in inp.counts) / (ms_step / 1e3) / 1e12,
        "stages_ms_rank0": {"hessian_gate_up": stage[0], "solve_gate_up": stage[1], "hessian_down": stage[2],
                            "solve_down": stage[3], "exchange_wait": stage[4]},
        "stages_ms_by_rank": [{"expert_stage": sum(r[:4]), "exchange_wait": r[4], "experts": int(r[5]),
                               "routed_rows": int(r[6])} for r in stages_by_rank],
        "roofline": roofline,
        "roofline_column_loop": {"kernel": "mx_gptq_kernel (groupwise) x2 + factors + RTN", "bound": "hbm",
                                 "achieved": col_bytes / (solve_ms / 1e3) / 1e9 if ws == 1 else None,
                                 "peak": peak_hbm, "unit": "GB/s",
                                 "frac": col_bytes / (solve_ms / 1e3) / 1e9 / peak_hbm if ws == 1 else None,
                                 "bytes_per_step": col_bytes, "peak_source": f"{src} hbm_gbs"},
        "gpu_launches": step.launches() * args.steps,
        "clocks": clk,
        "e2e": e2e,
    }
    if reps is not None:
        line["c2_replicas"] = reps
    if ws == 1 and not args.no_extras:
        n = max(3, args.steps // 4)
        configs = {}
        for key, fn in (("c2", lambda: extra_c2(device, n, 3, peak_tf, peak_hbm, src)),
                        ("c1", lambda: extra_c1(device, n, 3, peak_tf, src)),
                        ("c4", lambda: extra_c4(device, n, 3))):
            torch.cuda.empty_cache()
            configs[key] = fn()
        line["configs"] = configs
        from mlx_gptq_b200.artifacts import unpack_nibbles

        line["roofline_pack"] = extra_pack(device, peak_hbm, src, unpack_nibbles(outs[0]).reshape(-1, C3_H))
        torch.cuda.empty_cache()
        line["roofline_trailing_update"] = trailing_update_roofline(device, 20, peak_hbm, src)
    if ws == 1 and not args.no_cpu_baseline:
        del step, inp
        torch.cuda.empty_cache()
        sample = C3CpuSample(device)
        time_cpu_sample(sample, 1)
        line["cpu_baseline"] = cpu_sample_record(sample, time_cpu_sample(sample, 3))
    print(json.dumps(line), flush=True)


def profile_traffic(key: str):
    """Per-launch DRAM bytes of a kernel from the committed ncu summaries."""
    path = os.path.join(ROOT, "profiles", "hessian_traffic.json")
    if os.path.exists(path):
        return json.load(open(path)).get(key)
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the other configurations and the pack kernel")
    ap.add_argument("--profile-case", default=None,
                    choices=["hessian", "hessian-full", "solve", "solve-groupwise", "affine", "moe", "moe-small",
                             "c3-step", "pack"],
                    help="run a small case of one kernel for an ncu capture and exit")
    ap.add_argument("--config", choices=["c3", "c5"], default="c3",
                    help="c3: the routed expert batch (default); c5: the synthetic Qwen3-MoE layer stack")
    ap.add_argument("--layers", type=int, default=2, help="c5: decoder layers to calibrate")
    ap.add_argument("--c5-samples", type=int, default=256)
    ap.add_argument("--c5-seqlen", type=int, default=2048)
    ap.add_argument("--c5-batch", type=int, default=16, help="c5: sequences per forward")
    ap.add_argument("--c5-experts-forward", choices=["grouped", "eager"], default="grouped")
    ap.add_argument("--c5-dp", action="store_true",
                    help="c5: each rank forwards 1/N of the windows; Hessians summed over ranks")
    args = ap.parse_args()
    ws, rank, local = dist_env()
    if args.config == "c5":
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
        torch.cuda.set_device(local)
        run_c5(args, ws, rank, local)
        return
    if args.profile_case:
        profile_case(args.profile_case, torch.device("cuda", 0))
        return
    if args.impl == "reference":
        run_reference_arm(args, ws, rank)
        return
    run_c3(args, ws, rank, local)


if __name__ == "__main__":
    main()
