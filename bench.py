"""Benchmark: GPTQ-solved weight elems/s (Hessian -> codes) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload ("C2", seed = rank % 3): a dense MLP
projection sweep solved to MXFP4 with safe-scale-search.
  gate / up  W bf16 [11008, 4096] ~ N(0, 0.02), sharing H from X [131072, 4096]
  down       W bf16 [4096, 11008] ~ N(0, 0.02), H from X [131072, 11008]
  X bf16, i.i.d. Student-t(nu=4) per element, 1% of channels scaled x30.
One step = both Hessians (tcgen05 kernel) + damped 32x32 block factors + the
MXFP4 column loop of all three matrices, writing nibble-packed codes, E8M0
scales, bf16 W_dq and rel_err. Inputs (3.97 GB of X) exceed the 126 MB L2, so
no flush is needed between steps.

`value` is device-resident throughput (inputs already in HBM); `e2e` is the same
step through the package's public calls with X and W copied from pinned host
memory each step (chunked H2D overlapped with the Hessian) and the packed codes
+ scales + rel_err copied back. `cpu_baseline` / `--impl reference` time the
numpy oracle (a restatement of the reference's torch CPU path) on a bounded
sample and extrapolate linearly (Hessian: tokens; solve: 32-column groups,
which the reference solves independently).

Under torchrun each rank solves its own copy of the workload (weak scaling, no
data-path collective); timing is the max over ranks.

--config c5 instead calibrates a synthetic Qwen3-30B-A3B-shaped layer stack
layer by layer through the package's Pipeline and
prints per-layer stage times (--layers L, --c5-dp for data-parallel windows).
--profile-case NAME runs one small kernel case for an ncu capture.
"""

from __future__ import annotations

import argparse
import json
import math
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

TOKENS = 131072
HIDDEN, INTER = 4096, 11008
METRIC = "GPTQ-solved weight elems/s (Hessian->codes), MXFP4 safe-scale-search"
WORKLOAD = ("C2 dense MLP sweep: gate/up [11008,4096] share H(K=4096), down [4096,11008] H(K=11008); "
            "X [131072,K] bf16 Student-t(4), 1% channels x30; MXFP4 safe-scale-search")


# ---------------------------------------------------------------------------
# synthetic inputs (seeded, generated on the device in float32, rounded to bf16)
# ---------------------------------------------------------------------------
def student_t_bf16(n, k, seed, device, outlier_frac=0.01, outlier_scale=30.0, chunk=16384):
    g = torch.Generator(device=device).manual_seed(seed)
    out = torch.empty(n, k, dtype=torch.bfloat16, device=device)
    for i in range(0, n, chunk):
        m = min(chunk, n - i)
        z = torch.randn(m, k, generator=g, device=device)
        u = torch.rand(2, m, k, generator=g, device=device).clamp_(min=1e-12)
        chi2 = -2.0 * torch.log(u[0] * u[1])  # chi-square with 4 degrees of freedom
        out[i:i + m] = (z / torch.sqrt(chi2 / 4.0)).to(torch.bfloat16)
    n_out = max(1, int(round(outlier_frac * k)))
    idx = torch.randperm(k, generator=g, device=device)[:n_out]
    out[:, idx] = (out[:, idx].float() * outlier_scale).to(torch.bfloat16)
    return out


def weights_bf16(r, c, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(r, c, generator=g, device=device) * 0.02).to(torch.bfloat16)


def make_workload(seed, device):
    return {
        "X_gu": student_t_bf16(TOKENS, HIDDEN, seed + 1000, device),
        "X_down": student_t_bf16(TOKENS, INTER, seed + 2000, device),
        "gate": weights_bf16(INTER, HIDDEN, seed, device),
        "up": weights_bf16(INTER, HIDDEN, seed + 1, device),
        "down": weights_bf16(HIDDEN, INTER, seed + 2, device),
    }


ELEMS = 3 * INTER * HIDDEN  # weight elements solved per step
HESS_FLOP = 2.0 * TOKENS * (HIDDEN ** 2 + INTER ** 2)  # full X^T X, as the reference computes it


# ---------------------------------------------------------------------------
# the step (device-resident)
# ---------------------------------------------------------------------------
class Step:
    def __init__(self, wl, device):
        from mlx_gptq_b200 import layer

        self.layer = layer
        self.wl = wl
        self.H_gu = torch.empty(HIDDEN, HIDDEN, dtype=torch.float32, device=device)
        self.H_down = torch.empty(INTER, INTER, dtype=torch.float32, device=device)
        self.events = None

    def run(self, record=False):
        from mlx_gptq_b200 import hessian_accumulate

        ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)] if record else None
        if record:
            ev[0].record()
        hessian_accumulate(self.wl["X_gu"], self.H_gu, 1.0, 0.0)
        if record:
            ev[1].record()
        hessian_accumulate(self.wl["X_down"], self.H_down, 1.0, 0.0)
        if record:
            ev[2].record()
        f_gu = self.layer.mxfp_factors(self.H_gu.unsqueeze(0))
        f_dn = self.layer.mxfp_factors(self.H_down.unsqueeze(0))
        if record:
            ev[3].record()
        outs = []
        for name, f in (("gate", f_gu), ("up", f_gu), ("down", f_dn)):
            outs.append(self.layer.solve_mxfp_packed(self.wl[name], f, "mxfp4", "safe-scale-search",
                                                     torch.bfloat16, True, check_info=False))
        if record:
            ev[4].record()
        self.events = ev
        self.last = (outs, f_gu, f_dn)
        return outs


def column_loop_bytes():
    """Algorithmic HBM bytes of one step's three MXFP4 column loops: per matrix bf16 W in,
    bf16 W_dq out, nibble codes out (R*C*(2 + 2 + 0.5)), E8M0 scales (R*C/32) and the
    32x32 diagonal factor blocks read (4 * 32 * C)."""
    total = 0
    for r, c in ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER)):
        total += r * c * 4.5 + r * c // 32 + 4 * 32 * c
    return total


def column_loop_roofline(solve_ms_per_step, peak_hbm, src):
    """HBM roofline of the column loops (the north star's >= 50%-of-HBM target), stated with
    its bound: the safe-scale search makes them compute-bound on the FP32 and tensor pipes."""
    nbytes = column_loop_bytes()
    achieved = nbytes / (solve_ms_per_step / 1e3) / 1e9
    return {"kernel": "mx_gptq_kernel x3 (MXFP4 safe-scale-search)", "bound": "compute (FP32 + tensor pipes)",
            "achieved": achieved, "peak": peak_hbm, "unit": "GB/s", "frac": achieved / peak_hbm,
            "bytes_per_step": nbytes, "peak_source": f"{src} hbm_gbs",
            "note": "7 candidate E8M0 scales per group with e^T H e objectives on the tensor cores make the "
                    "loop compute-bound (ncu: DRAM 2.6%, tensor pipe 27%, FMA pipe 16%, 12 warp instructions "
                    "per weight element), so its HBM fraction is low by construction"}


def hessian_executed_elems(c):
    """Output elements the Hessian kernel computes per launch: 256x256 tiles on or above
    the diagonal (2-SM kernel, the default), 128x256 ones with GQ_HESSIAN_KERNEL=1sm."""
    if os.environ.get("GQ_HESSIAN_KERNEL", "2sm").startswith("1"):
        mt, nt = -(-c // 128), -(-c // 256)
        return 128 * 256 * sum(min(2 * tn + 2, mt) for tn in range(nt))
    t = -(-c // 256)
    return 256 * 256 * t * (t + 1) // 2


def launches_per_step():
    # 2 hessian + 2 x (dead columns + block factors) + 3 x (column loop + rel_err)
    return 2 + 4 + 6


# ---------------------------------------------------------------------------
# end-to-end step: pinned host inputs -> device -> host outputs
# ---------------------------------------------------------------------------
class E2EStep:
    CHUNK = 16384

    def __init__(self, wl, device):
        from mlx_gptq_b200 import layer

        self.layer = layer
        self.device = device
        self.host = {k: v.cpu().pin_memory() for k, v in wl.items()}
        self.dev_x = {k: torch.empty_like(wl[k]) for k in ("X_gu", "X_down")}
        self.dev_w = {k: torch.empty_like(wl[k]) for k in ("gate", "up", "down")}
        self.H = {"X_gu": torch.empty(HIDDEN, HIDDEN, device=device),
                  "X_down": torch.empty(INTER, INTER, device=device)}
        self.copy_stream = torch.cuda.Stream(device)
        self.out_host = None
        self.h2d_bytes = sum(v.numel() * v.element_size() for v in self.host.values())
        self.d2h_bytes = 0

    def run(self):
        from mlx_gptq_b200 import hessian_accumulate

        cs, ms = self.copy_stream, torch.cuda.current_stream(self.device)
        cs.wait_stream(ms)  # device buffers are free only once the previous step's kernels are done
        # weights first (small), then X in chunks; Hessian of chunk i overlaps copy of chunk i+1
        with torch.cuda.stream(cs):
            for k in ("gate", "up", "down"):
                self.dev_w[k].copy_(self.host[k], non_blocking=True)
        w_ready = torch.cuda.Event()
        w_ready.record(cs)
        for k in ("X_gu", "X_down"):
            src, dst, H = self.host[k], self.dev_x[k], self.H[k]
            first = True
            for i in range(0, TOKENS, self.CHUNK):
                with torch.cuda.stream(cs):
                    dst[i:i + self.CHUNK].copy_(src[i:i + self.CHUNK], non_blocking=True)
                    e = torch.cuda.Event()
                    e.record(cs)
                ms.wait_event(e)
                hessian_accumulate(dst[i:i + self.CHUNK], H, 1.0, 0.0 if first else 1.0)
                first = False
        ms.wait_event(w_ready)
        f_gu = self.layer.mxfp_factors(self.H["X_gu"].unsqueeze(0))
        f_dn = self.layer.mxfp_factors(self.H["X_down"].unsqueeze(0))
        outs = [self.layer.solve_mxfp_packed(self.dev_w[n], f, "mxfp4", "safe-scale-search", torch.bfloat16,
                                             True, check_info=False)
                for n, f in (("gate", f_gu), ("up", f_gu), ("down", f_dn))]
        if self.out_host is None:
            self.out_host = [(torch.empty(o.codes.shape, dtype=torch.uint8, pin_memory=True),
                              torch.empty(o.scales.shape, dtype=torch.uint8, pin_memory=True),
                              torch.empty(o.rel_err.shape, dtype=torch.float32, pin_memory=True)) for o in outs]
            self.d2h_bytes = sum(a.numel() + b.numel() + 4 * c.numel() for a, b, c in self.out_host)
        for o, (hc, hs, hr) in zip(outs, self.out_host):
            hc.copy_(o.codes, non_blocking=True)
            hs.copy_(o.scales, non_blocking=True)
            hr.copy_(o.rel_err, non_blocking=True)
        return outs


# ---------------------------------------------------------------------------
# CPU baseline: the numpy oracle on a bounded sample, extrapolated
# ---------------------------------------------------------------------------
def cpu_baseline(wl, n_tokens=4096, n_groups=4):
    from oracle import gptq as ogptq
    from oracle import hessian as ohess

    t_h = 0.0
    Hs = {}
    for k, K in (("X_gu", HIDDEN), ("X_down", INTER)):
        xs = wl[k][:n_tokens].float().cpu().numpy()
        t0 = time.perf_counter()
        Hs[k] = ohess.hessian(xs)
        t_h += (time.perf_counter() - t0) * (TOKENS / n_tokens)
    t_s = 0.0
    cols = n_groups * 32
    for name, hk, K in (("gate", "X_gu", HIDDEN), ("up", "X_gu", HIDDEN), ("down", "X_down", INTER)):
        W = wl[name][:, :cols].float().cpu().numpy()[None]
        H = Hs[hk][:cols, :cols][None].copy()
        t0 = time.perf_counter()
        ogptq.solve_gptq(W, H, 4, 32, mode="mxfp4", mxfp_algorithm="safe-scale-search")
        t_s += (time.perf_counter() - t0) * (K / cols)
    total = t_h + t_s
    cores = torch.get_num_threads()
    return {
        "value": ELEMS / total,
        "unit": "elems/s",
        "cores": cores,
        "kind": "port",
        "sample": (f"numpy oracle: Hessians on {n_tokens}/{TOKENS} tokens x (tokens ratio), MXFP4 "
                   f"safe-scale-search on {n_groups} of the K/32 column groups of each matrix (all rows) x "
                   f"(groups ratio); extrapolated step {total:.1f} s (hessian {t_h:.1f} s, solve {t_s:.1f} s)"),
    }


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


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return p["bf16_tflops_sustained"], p["hbm_gbs"], "measured"
    return 1400.0, 6650.0, "fallback"


def profile_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "hessian_traffic.json")
    if os.path.exists(path):
        return json.load(open(path)).get("dram_bytes_per_launch_k11008")
    return None


# ---------------------------------------------------------------------------
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference_arm(args, ws, rank):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    wl = make_workload(0, dev)
    small = {k: v for k, v in wl.items()}
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(small, n_tokens=4096, n_groups=4)
        if i >= args.warmup:
            vals.append(r["value"])
    v = statistics.mean(vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "elems/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ELEMS / v * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": WORKLOAD, "seed": 0},
            "cpu_baseline": {"kind": r["kind"], "cores": r["cores"], "sample": r["sample"], "value": v,
                             "unit": "elems/s"},
            "e2e": {"value": v, "unit": "elems/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def moe_routing(tokens, experts, topk, seed, device):
    """C3 router: softmax logits N(0,1) + per-expert Zipf(1.1) bias -1.1*ln(rank), top-k.
    Returns (token_idx int32 [tokens*topk] grouped by expert, offsets int64 [E+1] on CPU)."""
    g = torch.Generator(device=device).manual_seed(seed)
    rank = torch.randperm(experts, generator=g, device=device).float() + 1.0
    logits = torch.randn(tokens, experts, generator=g, device=device) - 1.1 * torch.log(rank)
    top = logits.topk(topk, dim=1).indices.reshape(-1)
    order = torch.sort(top, stable=True).indices
    token_idx = (order // topk).to(torch.int32)
    counts = torch.bincount(top, minlength=experts).cpu()
    offsets = torch.zeros(experts + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, 0)
    return token_idx, offsets


def profile_case(case, device):
    """Small, self-contained launches for ncu captures (a few launches, inputs > L2)."""
    from mlx_gptq_b200 import hessian_accumulate, layer

    if case in ("hessian", "hessian-full"):
        n, k = (16384, HIDDEN) if case == "hessian" else (TOKENS, INTER)
        X = student_t_bf16(n, k, 7, device)  # small case: 128 MiB > L2
        H = torch.empty(k, k, device=device)
        for i in range(4):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            hessian_accumulate(X, H, 1.0, 0.0)
            b.record()
            b.synchronize()
            flop = 2.0 * n * k * k
            print(f"hessian launch {i} [{os.environ.get('GQ_HESSIAN_KERNEL', '2sm')}] N={n} C={k}: "
                  f"{a.elapsed_time(b):.3f} ms, {flop / a.elapsed_time(b) / 1e9:.1f} TFLOP/s (2*N*C^2)")
    elif case == "solve":
        X = student_t_bf16(8192, HIDDEN, 7, device)
        H = torch.empty(HIDDEN, HIDDEN, device=device)
        hessian_accumulate(X, H, 1.0, 0.0)
        W = weights_bf16(INTER, HIDDEN, 8, device)  # 90 MB bf16 in, 90 MB bf16 out
        f = layer.mxfp_factors(H.unsqueeze(0))
        for i in range(4):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            layer.solve_mxfp_packed(W, f, "mxfp4", "safe-scale-search", torch.bfloat16, True, check_info=False)
            b.record()
            b.synchronize()
            print(f"solve launch {i}: {a.elapsed_time(b):.3f} ms ({W.numel() / a.elapsed_time(b) / 1e6:.2f} G elems/s)")
    elif case == "affine":
        from mlx_gptq_b200 import solve_gptq
        from mlx_gptq_b200.gptq import _prepare_hinv

        X = student_t_bf16(32768, HIDDEN, 7, device)
        H = torch.empty(HIDDEN, HIDDEN, device=device)
        hessian_accumulate(X, H, 1.0, 0.0)
        W = weights_bf16(HIDDEN, HIDDEN, 8, device).unsqueeze(0)
        for i in range(3):
            a, m, b = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            a.record()
            _prepare_hinv(H.unsqueeze(0).clone(), 0.01)
            m.record()
            solve_gptq(W, H.unsqueeze(0).clone(), 4, 64, mode="affine")
            b.record()
            b.synchronize()
            print(f"affine C1 [4096x4096] g64: factor {a.elapsed_time(m):.2f} ms, full solve_gptq "
                  f"{m.elapsed_time(b):.2f} ms ({W.numel() / m.elapsed_time(b) / 1e6:.2f} G elems/s)")
    elif case in ("moe", "moe-small"):
        from mlx_gptq_b200 import hessian_grouped

        T, E, K, I = (524288 if case == "moe" else 32768), 128, 2048, 768
        X = (torch.randn(T, K, generator=torch.Generator(device=device).manual_seed(1), device=device)
             .to(torch.bfloat16))
        token_idx, offsets = moe_routing(T, E, 8, 2, device)
        cnt = (offsets[1:] - offsets[:-1])
        print(f"routed slots {int(offsets[-1])}, tokens/expert min {int(cnt.min())} median "
              f"{int(cnt.median())} max {int(cnt.max())} zero {int((cnt == 0).sum())}")
        H = torch.empty(E, K, K, device=device)
        flop = 2.0 * float((cnt.double() * K * K).sum())
        for i in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            hessian_grouped(X, token_idx, offsets, E, H=H)
            b.record()
            b.synchronize()
            print(f"grouped hessian launch {i}: {a.elapsed_time(b):.3f} ms, {flop / a.elapsed_time(b) / 1e9:.1f} "
                  f"TFLOP/s (2*N_e*C^2 summed over experts)")
        W = (torch.randn(E, 2 * I, K, generator=torch.Generator(device=device).manual_seed(0), device=device)
             * 0.02).to(torch.bfloat16)
        for i in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            f = layer.mxfp_factors(H)
            layer.solve_mxfp_packed(W, f, "mxfp4", "groupwise", torch.bfloat16, True, check_info=False)
            b.record()
            b.synchronize()
            print(f"batched solve (128 experts gate_up, groupwise) {i}: {a.elapsed_time(b):.3f} ms, "
                  f"{W.numel() / a.elapsed_time(b) / 1e6:.1f} G elems/s")
    else:
        raise SystemExit(f"unknown profile case {case}")
    torch.cuda.synchronize()
    print(f"profile case {case} done")


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile-case", choices=["hessian", "hessian-full", "solve", "affine", "moe", "moe-small"],
                    default=None,
                    help="run a small case of one kernel for an ncu capture and exit")
    ap.add_argument("--config", choices=["c2", "c5"], default="c2",
                    help="c2: the headline MLP sweep (default); c5: the synthetic Qwen3-MoE layer stack")
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
        # per-layer buffers vary in size with the routing: let the allocator grow segments
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
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    pg = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        pg = dist
    args.warmup = max(args.warmup, 3)

    wl = make_workload(rank % 3, device)
    step = Step(wl, device)
    clocks = ClockSampler(local)
    clocks.start()  # sampling from before the warm-up; the summary keeps the timed region
    for _ in range(args.warmup):
        step.run()
    torch.cuda.synchronize()
    outs, f_gu, f_dn = step.last
    assert not bool((f_gu.info != 0).any()) and not bool((f_dn.info != 0).any()), "factorization failed"

    # timed region: K steps, events on the launching stream, barrier + sync on both sides
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    clocks.begin()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    hess_ms, solve_ms, hess_big_ms = [], [], []
    t0.record()
    for _ in range(args.steps):
        step.run(record=True)
        ev = step.events
        hess_ms.append(ev)
    t1.record()
    torch.cuda.synchronize()
    clocks.end()
    if pg:
        pg.barrier()
    clk = clocks.stop()
    ms_total = t0.elapsed_time(t1)
    per_step = []
    for ev in hess_ms:
        hess_big_ms.append(ev[1].elapsed_time(ev[2]))
        solve_ms.append(ev[3].elapsed_time(ev[4]))
        per_step.append(ev[0].elapsed_time(ev[2]))
    ms_step = ms_total / args.steps
    if pg:
        t = torch.tensor([ms_step], device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms_step = float(t.item())
    value = ws * ELEMS / (ms_step / 1e3)

    # e2e leg (public calls, host buffers)
    e2e = None
    if not args.no_e2e:
        e = E2EStep(wl, device)
        for _ in range(2):
            e.run()
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = max(3, args.steps // 2)
        a.record()
        for _ in range(n_e2e):
            e.run()
        b.record()
        torch.cuda.synchronize()
        ms_e2e = a.elapsed_time(b) / n_e2e
        if pg:
            t = torch.tensor([ms_e2e], device=device)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms_e2e = float(t.item())
        e2e = {"value": ws * ELEMS / (ms_e2e / 1e3), "unit": "elems/s", "ms_per_step": ms_e2e,
               "h2d_bytes_per_step": e.h2d_bytes, "d2h_bytes_per_step": e.d2h_bytes}
        del e

    if pg:
        pg.destroy_process_group()
    if rank != 0:
        return

    peak_tf, peak_hbm, src = peaks()
    big_ms = statistics.mean(hess_big_ms)
    flop_big = 2.0 * TOKENS * INTER ** 2
    executed_flop = 2.0 * TOKENS * hessian_executed_elems(INTER)
    achieved = flop_big / (big_ms / 1e3) / 1e12
    roofline = {"kernel": "hessian2_kernel (2-SM tcgen05, K=11008 launch)", "bound": "tensor", "achieved": achieved,
                "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                "peak_source": f"{src} bf16_tflops_sustained (kernel timed inside a long step)",
                "flop_per_launch": flop_big,
                "note": "algorithmic FLOP = 2*N*C^2 (full X^T X as the reference computes); the kernel "
                        "computes only tiles on/above the diagonal and mirrors them, so frac can exceed 1; "
                        "executed_* counts the MMA work actually issued",
                "executed_tflops": executed_flop / (big_ms / 1e3) / 1e12,
                "executed_frac": executed_flop / (big_ms / 1e3) / 1e12 / peak_tf,
                "traffic": profile_traffic()}
    hess_ms_step = statistics.mean(per_step)
    line = {
        "metric": METRIC, "value": value, "unit": "elems/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 x bf16 -> f32 (Hessian), f32 (solve)", "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens": TOKENS, "elems_per_step_per_gpu": ELEMS,
                   "seed": "rank % 3", "l2": "inputs larger than L2 (X = 3.97 GB); no flush",
                   "parallelism": f"weak x{ws} (independent replicas, no data-path collective)"},
        "hessian_tflops": HESS_FLOP / (hess_ms_step / 1e3) / 1e12 * ws,
        "hessian_ms_per_step": hess_ms_step,
        "solve_ms_per_step": statistics.mean(solve_ms),
        "roofline": roofline,
        "roofline_column_loop": column_loop_roofline(statistics.mean(solve_ms), peak_hbm, src),
        "gpu_launches": launches_per_step() * args.steps,
        "clocks": clk,
        "e2e": e2e,
    }
    if not args.no_cpu_baseline and ws == 1:
        torch.set_num_threads(os.cpu_count() or 1)
        line["cpu_baseline"] = cpu_baseline(wl)
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
