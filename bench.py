#!/usr/bin/env python
"""Benchmark of the hackable-lm fused-operator hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload d12|lm_head]

Prints ONE JSON line (rank 0).  For N > 1 launch one process per GPU with
torch.distributed.run; timing is on the device (CUDA events), bracketed by a
barrier + synchronize, and the max over ranks is reported.

Workloads (synthetic, seeded):
  d12      (default) depth-12 decoder data-parallel training step, BASELINE
           config 5: global batch 2^20 tokens (micro-batch 16 x 2048 per GPU,
           gradient accumulation 32/N), DDP bf16 buckets over NCCL, Muon+AdamW
           step; all hot-path operators on the B200 kernels, attention via SDPA.
           At N=1 the line also carries the LM-head C4 measurement
           ("lm_head_c4") and per-operator rooflines ("ops").
  lm_head  fused LM-head + cross-entropy forward+backward, hidden [32768,768],
           W [32768,768], 2% targets = ignore_index -1 (one step = one call on
           one batch).  With N > 1 each rank processes its own batch and the
           bf16 grad_weight is all-reduced (data-parallel exchange).

--impl reference times the reference algorithm's CPU implementation (the
oracle restatement, all host threads) on a bounded sample of the same
workload and prints the same line with "impl": "reference".
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
# stdout carries exactly one JSON line: NCCL's own log lines go to stderr
# unless the caller chose a log file (NCCL ignores the file at the VERSION log
# level, hence also the descriptor switch in main())
os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:  # noqa: BLE001
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def traffic_table() -> dict:
    """DRAM bytes per launch from committed ncu summaries (profiles/ncu_traffic.txt):
    lines "<workload> <kernel> <bytes_per_launch> <note...>"."""
    out = {}
    p = ROOT / "profiles" / "ncu_traffic.txt"
    if p.exists():
        for line in p.read_text().splitlines():
            parts = line.split()
            if len(parts) >= 3 and not line.startswith("#"):
                try:
                    out[(parts[0], parts[1])] = float(parts[2])
                except ValueError:
                    pass
    return out


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.enabled = self.world > 1

    def init(self, backend="nccl"):
        if self.enabled and not dist.is_initialized():
            import datetime

            if backend == "nccl":
                torch.cuda.set_device(self.local_rank)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))

    def barrier(self):
        if self.enabled:
            dist.barrier()

    def max(self, x: float) -> float:
        if not self.enabled:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.enabled and dist.is_initialized():
            dist.destroy_process_group()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.dev), "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cuda_time(fn, steps: int, warmup: int, d: Dist, flush=None, label: str = "timed"):
    """Run warmup steps, then time exactly `steps` steps with CUDA events,
    bracketed by barrier + synchronize; returns (max-over-ranks total ms)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    d.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    torch.cuda.nvtx.range_push(label)  # ncu --nvtx --nvtx-include "timed/" selects these launches
    for _ in range(steps):
        if flush is not None:
            flush()
        fn()
    torch.cuda.nvtx.range_pop()
    stop.record()
    torch.cuda.synchronize()
    d.barrier()
    torch.cuda.synchronize()
    return d.max(start.elapsed_time(stop))


# ---------------------------------------------------------------------------
# LM head workload
# ---------------------------------------------------------------------------
LM = {"M": 32768, "C": 768, "V": 32768, "ignore_frac": 0.02, "ignore_index": -1}


def lm_inputs(seed: int, device):
    g = torch.Generator().manual_seed(seed)
    M, C, V = LM["M"], LM["C"], LM["V"]
    hidden = torch.randn(M, C, generator=g).to(torch.bfloat16)
    weight = (torch.randn(V, C, generator=g) * 0.02).to(torch.bfloat16)
    targets = torch.randint(0, V, (M,), generator=g)
    targets[torch.randperm(M, generator=g)[: int(LM["ignore_frac"] * M)]] = LM["ignore_index"]
    return hidden, weight, targets


def lm_cpu_sample(n_tokens: int, seed: int = 0):
    import oracle

    hidden, weight, targets = lm_inputs(seed, "cpu")
    h = hidden[:n_tokens].float()
    w = weight.float()
    t = targets[:n_tokens]
    t0 = time.perf_counter()
    oracle.lm_head_ce(h, w, t, LM["ignore_index"], 4096)
    return time.perf_counter() - t0


def cpu_baseline_lm(target_seconds: float = 15.0) -> dict:
    torch.set_num_threads(os.cpu_count() or 1)
    n = 256
    lm_cpu_sample(n)  # warm-up
    dt = lm_cpu_sample(n)
    per_rep = max(1.0, target_seconds / 3)
    n = int(min(8192, max(256, n * per_rep / max(dt, 1e-3))) // 256 * 256)
    times = [lm_cpu_sample(n) for _ in range(3)]
    med = statistics.median(times)
    return {"value": n / med, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"oracle (torch CPU fp32) LM-head+CE fwd+bwd on {n} of the 32768 tokens, full "
                      f"V=32768, C=768; median of 3 reps ({med:.2f} s each)"}


def bench_lm_head(args, d: Dist, device) -> dict:
    from hackable_lm_b200 import _lib, kernels

    peaks, peak_src = load_peaks()
    hidden, weight, targets = lm_inputs(1000 + d.rank, device)
    h = hidden.to(device).requires_grad_(True)
    w = weight.to(device).requires_grad_(True)
    t = targets.to(device)
    M, C, V = LM["M"], LM["C"], LM["V"]

    def step():
        loss = kernels.fused_linear_cross_entropy_with_weight(h, w, None, t, "b200",
                                                              ignore_index=LM["ignore_index"])
        gh, gw = torch.autograd.grad(loss, (h, w))
        if d.enabled:
            dist.all_reduce(gw)
        return loss

    # ---- device-timed value, with the library timing its own kernels
    clocks = ClockSampler(device.index)
    kernels_to_time = ("lm_logits", "lm_dlogits", "lm_dx", "lm_dw")
    timers = {k: _lib.KernelTimer(k, 4 * args.steps) for k in kernels_to_time}
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks.start()
    n0 = _lib.launch_count()
    for k in kernels_to_time:
        timers[k].__enter__()
    total_ms = cuda_time(step, args.steps, 0, d)
    for k in kernels_to_time:
        timers[k].__exit__(None, None, None)
    launches = _lib.launch_count() - n0
    clk = clocks.stop()
    ms_per_step = total_ms / args.steps
    value = M * d.world / (ms_per_step / 1e3)

    kt = {k: timers[k].times_ms() for k in kernels_to_time}
    # per step (= per call): a kernel may launch more than once (the dlogits pass
    # and grad_hidden GEMM run in two row halves), and the second dlogits half
    # overlaps the first grad_hidden GEMM on a side stream, so shares can sum
    # above 1
    flops = {"lm_logits": 2.0 * M * C * V, "lm_dx": 2.0 * M * C * V, "lm_dw": 2.0 * M * C * V}
    bytes_ = {"lm_dlogits": 4.0 * M * V}  # bf16 logits read + dlogits written in place
    per_step = {k: sum(ts) / args.steps for k, ts in kt.items() if ts}
    breakdown = {}
    for k, ms in per_step.items():
        entry = {"ms": round(ms, 4), "launches_per_step": len(kt[k]) // args.steps,
                 "share_of_step": round(ms / ms_per_step, 4)}
        if k in flops:
            entry["tflops"] = round(flops[k] / (ms / 1e3) / 1e12, 1)
        if k in bytes_:
            entry["gbs"] = round(bytes_[k] / (ms / 1e3) / 1e9, 1)
        breakdown[k] = entry
    dominant = max(per_step, key=per_step.get)
    dom_ms = per_step[dominant]
    tr = traffic_table().get(("lm_head", dominant))
    if dominant in flops:
        achieved = flops[dominant] / (dom_ms / 1e3) / 1e12
        peak = peaks["bf16_tflops"]
        roofline = {"kernel": dominant, "bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                    "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": tr,
                    "peak_source": f"{peak_src} bf16_tflops (burst: kernel timed inside a ~5 ms step)",
                    "algorithmic_per_step": f"2*M*C*V = {flops[dominant]:.4e} FLOP"}
    else:
        achieved = bytes_[dominant] / (dom_ms / 1e3) / 1e9
        peak = peaks["hbm_gbs"]
        roofline = {"kernel": dominant, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                    "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": tr,
                    "peak_source": f"{peak_src} hbm_gbs"}

    # ---- end to end through the public API with host-resident inputs
    h_host = hidden.pin_memory()
    t_host = targets.pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    h_dev = torch.empty_like(h)
    t_dev = torch.empty_like(t)

    def e2e_step():
        h_dev.copy_(h_host, non_blocking=True)
        t_dev.copy_(t_host, non_blocking=True)
        hd = h_dev.requires_grad_(True)
        loss = kernels.fused_linear_cross_entropy_with_weight(hd, w, None, t_dev, "b200",
                                                              ignore_index=LM["ignore_index"])
        gh, gw = torch.autograd.grad(loss, (hd, w))
        if d.enabled:
            dist.all_reduce(gw)
        loss_host.copy_(loss.detach(), non_blocking=True)
        hd.requires_grad_(False)

    e2e_ms = cuda_time(e2e_step, args.steps, args.warmup, d, label="e2e") / args.steps
    e2e = {"value": M * d.world / (e2e_ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": h_host.numel() * 2 + t_host.numel() * 8, "d2h_bytes_per_step": 4,
           "ms_per_step": round(e2e_ms, 4)}

    out = {
        "metric": "LM-head+CE fwd/bwd tokens/s", "value": value, "unit": "tokens/s", "n_gpus": d.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: hidden~N(0,1), W~N(0,0.02), uniform targets, 2% ignore_index=-1 (seeded)",
        "config": {"workload": f"lm_head_ce C4: hidden [{M},{C}] x W [{V},{C}], fwd+bwd",
                   "tokens_per_gpu": M, "hidden": C, "vocab": V, "ignore_index": -1,
                   "parallelism": f"dp{d.world} (grad_weight all-reduce)" if d.enabled else "single GPU",
                   "l2": "working set per step ~2.2 GB (bf16 logits) >> 126 MB L2; no flush"},
        "roofline": roofline, "kernel_breakdown": breakdown, "e2e": e2e, "gpu_launches": launches,
        "gpu_launches_per_step": launches / args.steps, "clocks": clk,
    }
    return out


# ---------------------------------------------------------------------------
# Depth-12 data-parallel training step
# ---------------------------------------------------------------------------
D12_FLOPS_PER_TOKEN = 887_095_296  # config.estimate_flops_per_token, full causal attention

# operator calls per micro-step: per-layer kernels once per layer, LM-head kernels once
D12_KERNELS = {"lm_logits": 1, "lm_dlogits": 1, "lm_dx": 1, "lm_dw": 1, "gate_up": 12, "qkv_fwd": 12, "qkv_bwd_norm": 12,
               "qkv_dx": 12, "qkv_dw": 12, "swiglu_fwd": 12, "swiglu_bwd": 12, "swiglu_down_bwd": 12,
               "proj_norm": 24, "rmsnorm_fwd": 1, "rmsnorm_bwd": 25}


def d12_flops_per_token(window: int) -> int:
    if not window:
        return D12_FLOPS_PER_TOKEN
    from hackable_lm_b200 import config as hcfg

    n_embd, _ = hcfg.depth_dimensions(12)
    return hcfg.estimate_flops_per_token(12, n_embd, 2048, hcfg.scaling_params_for_depth(12, 32768),
                                         attention_window=window,
                                         attention_full_every=hcfg.DEFAULTS["attention_full_every"])


def d12_config(world: int, accum: int, max_grad_norm: float = 1.0, window: int = 0) -> dict:
    attention = ("torch SDPA, full causal" if not window else
                 f"sliding window {window} (the reference's default pattern: every 4th and the last layer "
                 "full causal): windowed layers on the tcgen05 forward and backward, "
                 "full layers on SDPA")
    return {"workload": "d12 DP training step: depth 12, C=768, 6x128 heads, SwiGLU 2048, vocab 32768, "
                        "seq 2048, micro-batch 16/GPU, global batch 2^20 tokens, global grad-norm clip "
                        f"{max_grad_norm}, Muon+AdamW step",
            "model": "hackable-lm d12 (random init)", "global_batch": 2**20, "seq_len": 2048,
            "micro_batch_per_gpu": 16, "grad_accum_per_rank": accum,
            "parallelism": f"dp{world}" + (" (DDP, bf16 25 MB buckets, NCCL)" if world > 1 else ""),
            "attention": attention,
            "l2": "working set per micro-step >> 126 MB L2 (activations ~GBs); no flush"}


def bench_d12(args, d: Dist, device) -> dict:
    from hackable_lm_b200 import _lib
    from hackable_lm_b200 import train as tr

    peaks, peak_src = load_peaks()
    window = int(args.attention_window or 0)
    s = tr.build(device, world=d.world, attention_window=window or None)
    # fresh data: one distinct micro-batch for every micro-step of the run (warm-up, timed
    # steps and the end-to-end pass), cycling only beyond 1024 micro-batches (268 MB)
    n_micro = min(1024, s.accum * (args.warmup + 2 * args.steps + 1))
    batches = tr.synthetic_batches(n_micro, s.micro_batch, s.seq_len, s.config.vocab_size, d.rank, device)
    tokens_per_step = s.accum * s.micro_batch * s.seq_len * d.world
    cursor = [0]

    def next_batch(i):
        b = batches[cursor[0] % len(batches)]
        cursor[0] += 1
        return b

    def step(mark=None):
        return tr.train_step(s, batches, fetch=next_batch, max_grad_norm=args.max_grad_norm, mark=mark)

    first_loss = None
    for i in range(args.warmup):
        l = step()
        if i == 0:
            first_loss = float(l.float().item())
    torch.cuda.synchronize()
    # per-kernel timing of the library's own launches during the first timed step
    # capacity: up to two launches per operator call (LM dlogits / grad_hidden run in row halves)
    timers = {k: _lib.KernelTimer(k, 2 * n * s.accum) for k, n in D12_KERNELS.items()}
    clocks = ClockSampler(device.index)
    clocks.start()
    d.barrier()
    torch.cuda.synchronize()
    n0 = _lib.launch_count()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    first = torch.cuda.Event(enable_timing=True)
    phase_events: list[tuple[str, torch.cuda.Event]] = []

    def mark(tag):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        phase_events.append((tag, ev))

    start.record()
    torch.cuda.nvtx.range_push("timed")  # ncu --nvtx --nvtx-include "timed/" selects these launches
    for i in range(args.steps):
        if i == 0:
            for t in timers.values():
                t.__enter__()
        loss = step(mark if i == 0 else None)
        if i == 0:
            for t in timers.values():
                t.__exit__(None, None, None)
            first.record()
    torch.cuda.nvtx.range_pop()
    stop.record()
    torch.cuda.synchronize()
    d.barrier()
    torch.cuda.synchronize()
    total_ms = d.max(start.elapsed_time(stop))
    step0_ms = start.elapsed_time(first)
    launches = _lib.launch_count() - n0
    clk = clocks.stop()
    # per-phase breakdown of the first timed step (this rank): micro-steps, the exposed
    # part of the gradient all-reduce (the last micro-step waits for DDP's final
    # buckets), gradient clipping and the optimizer step
    prev, micro = start, []
    phases = {}
    for tag, ev in phase_events:
        ms = prev.elapsed_time(ev)
        if tag == "micro":
            micro.append(ms)
        else:
            phases[tag] = ms
        prev = ev
    plain = micro[:-1] if len(micro) > 1 else micro
    step_phases = {"micro_step_ms": round(statistics.mean(plain), 3),
                   "last_micro_step_ms": round(micro[-1], 3),
                   "exposed_allreduce_ms": round(micro[-1] - statistics.mean(plain), 3) if d.world > 1 else 0.0,
                   "clip_ms": round(phases.get("clip", 0.0), 3), "optimizer_ms": round(phases.get("opt", 0.0), 3),
                   "note": "first timed step on rank 0; the optimizer's Muon work is sharded over the ranks"}
    ms_per_step = total_ms / args.steps
    value = tokens_per_step / (ms_per_step / 1e3)

    M = s.micro_batch * s.seq_len
    C, V, Hd = s.config.n_embd, s.config.vocab_size, 3 * s.config.n_head * s.config.head_dim
    Hm, Dq = s.config.mlp_hidden, s.config.n_head * s.config.head_dim
    # algorithmic FLOPs / HBM bytes per operator call (bf16 = 2 bytes)
    flops = {"lm_logits": 2.0 * M * C * V, "lm_dx": 2.0 * M * C * V, "lm_dw": 2.0 * M * C * V,
             "qkv_fwd": 2.0 * M * C * Hd, "qkv_dx": 2.0 * M * C * Hd, "qkv_dw": 2.0 * M * C * Hd,
             "gate_up": 2.0 * M * C * 2 * s.config.mlp_hidden,
             # o_proj (K = C) and down (K = H) calls alternate: the mean per call
             "proj_norm": 2.0 * M * C * (Dq + s.config.mlp_hidden) / 2}
    n_fwd = D12_KERNELS["rmsnorm_fwd"]
    bytes_ = {
        "swiglu_fwd": 2.0 * M * 3 * Hm,           # read gate_up [M,2H], write [M,H]
        "swiglu_bwd": 2.0 * M * 5 * Hm,           # read gate_up + grad [M,H], write [M,2H]
        # the input norm (read x, write norm); the residual variants run inside proj_norm
        "rmsnorm_fwd": 2.0 * M * C * (2 + 4 * (n_fwd - 1)) / n_fwd,
        # input norm: read x + grad_norm, write grad; residual variants also read the residual grad
        "rmsnorm_bwd": 2.0 * M * C * (3 + 4 * (D12_KERNELS["rmsnorm_bwd"] - 1)) / D12_KERNELS["rmsnorm_bwd"],
        "qkv_bwd_norm": 2.0 * M * Dq * 6,         # read q, k, dq, dk; write dq_in, dk_in
        "lm_dlogits": 4.0 * M * V,                # bf16 logits read + dlogits written in place
        # down grad_h GEMM + SwiGLU backward: read grad_y [M,C], gate_up [M,2H], W_down [C,H];
        # write grad_gate_up [M,2H] (HBM-bound: 2*M*C*H FLOP over these bytes is below the ridge)
        "swiglu_down_bwd": 2.0 * (M * C + 4 * M * Hm + C * Hm),
    }
    breakdown, totals = {}, {}
    for k, t in timers.items():
        ts = t.times_ms()
        if not ts:
            continue
        totals[k] = sum(ts)
        # per operator call (D12_KERNELS calls per micro-step; a call may be two launches)
        avg = sum(ts) / (D12_KERNELS[k] * s.accum)
        e = {"launches_in_step": t.launches, "calls_in_step": D12_KERNELS[k] * s.accum,
             "avg_ms_per_call": round(avg, 4), "total_ms": round(sum(ts), 3),
             "share_of_step": round(sum(ts) / step0_ms, 4)}
        if k in flops:
            e["tflops"] = round(flops[k] / (avg / 1e3) / 1e12, 1)
        if k in bytes_:
            e["gbs"] = round(bytes_[k] / (avg / 1e3) / 1e9, 1)
        breakdown[k] = e
    dominant = max((k for k in totals if k in flops or k in bytes_), key=totals.get)
    dom_avg = breakdown[dominant]["avg_ms_per_call"]
    roofline = {"kernel": dominant, "traffic": traffic_table().get(("d12", dominant))}
    if dominant in flops:
        achieved = flops[dominant] / (dom_avg / 1e3) / 1e12
        peak = peaks["bf16_tflops_sustained"]
        roofline.update({"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_src} bf16_tflops_sustained (kernel inside a seconds-long step)"})
    else:
        achieved = bytes_[dominant] / (dom_avg / 1e3) / 1e9
        roofline.update({"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_source": f"{peak_src} hbm_gbs"})

    # ---- end to end: every micro-batch copied from pinned host memory, loss read back per step
    host = [(x.cpu().pin_memory(), y.cpu().pin_memory()) for x, y in batches]
    xd = torch.empty_like(batches[0][0])
    yd = torch.empty_like(batches[0][1])
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def fetch(i):
        hx, hy = host[cursor[0] % len(host)]
        cursor[0] += 1
        xd.copy_(hx, non_blocking=True)
        yd.copy_(hy, non_blocking=True)
        return xd, yd

    def e2e_step():
        l = tr.train_step(s, batches, fetch=fetch, max_grad_norm=args.max_grad_norm)
        loss_host.copy_(l.float(), non_blocking=True)

    e2e_ms = cuda_time(e2e_step, args.steps, 1, d, label="e2e") / args.steps
    bytes_in = s.accum * (host[0][0].numel() + host[0][1].numel()) * 8
    e2e = {"value": tokens_per_step / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": bytes_in,
           "d2h_bytes_per_step": 4, "ms_per_step": round(e2e_ms, 3)}
    flops_per_token = d12_flops_per_token(window)
    mfu = flops_per_token * value / (peaks["bf16_tflops"] * 1e12 * d.world)
    return {
        "metric": "d12 step tok/s", "value": value, "unit": "tokens/s", "n_gpus": d.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: uniform token ids (seeded per rank), targets = ids shifted by one",
        "config": d12_config(d.world, s.accum, args.max_grad_norm, window), "roofline": roofline,
        "kernel_breakdown": breakdown,
        "mfu": round(mfu, 4), "mfu_basis": f"{flops_per_token} FLOP/token / measured bf16 burst peak",
        "loss_first_step": first_loss, "loss": float(loss.float().item()),
        "loss_note": f"mean micro-batch loss of the first warm-up step and of the last timed step; "
                     f"{n_micro} distinct micro-batches over the run; random-init loss is ln(32768) = 10.40",
        "step_phases": step_phases, "e2e": e2e, "gpu_launches": launches,
        "gpu_launches_per_step": launches / args.steps, "clocks": clk,
    }


def d12_cpu_sample(seq_len: int = 2048, seed: int = 0) -> float:
    from oracle import model as om

    p = om.init_params(seed=seed)
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 32768, (1, seq_len + 1), generator=g)
    t0 = time.perf_counter()
    om.train_step_cpu(p, ids[:, :-1], ids[:, 1:])
    return time.perf_counter() - t0


def cpu_baseline_d12(reps: int = 2) -> dict:
    torch.set_num_threads(os.cpu_count() or 1)
    d12_cpu_sample()  # warm-up
    times = [d12_cpu_sample() for _ in range(reps)]
    med = statistics.median(times)
    return {"value": 2048 / med, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"port: oracle d12 model (torch CPU fp32, a restatement of the reference LanguageModel) "
                      f"forward+backward on 1x2048 tokens, median of {reps} ({med:.2f} s each); the optimizer "
                      f"step is excluded"}


# ---------------------------------------------------------------------------
# per-operator roofline measurements (rank 0, after the headline)
# ---------------------------------------------------------------------------
def bench_ops(device, iters: int = 20, only: str | None = None) -> dict:
    """Per-operator rooflines at the BASELINE operator configs.

    L2 policy: inputs larger than L2.  Each operator cycles through enough
    private copies of its inputs that one cycle reads more than twice the L2
    size of distinct input bytes, so no call finds its inputs in L2; the time
    per call is the CUDA-event time of the whole timed loop divided by the
    number of calls (each call also pays the write-back of the previous call's
    outputs, as inside a training step).  `only`: run just the operators whose
    name starts with it (small, known launch sequences for ncu captures: one
    untimed pass over the copies, then `iters` timed calls)."""
    from hackable_lm_b200 import ops
    from hackable_lm_b200.model import RotaryEmbedding

    peaks, _ = load_peaks()

    def timed(fn, inputs, in_bytes, n=iters):
        copies = max(2, -(-2 * L2_BYTES // max(1, in_bytes)))
        sets = [inputs] + [tuple(t.clone() if isinstance(t, torch.Tensor) else t for t in inputs)
                           for _ in range(copies - 1)]
        for st in sets:  # untimed pass (allocations, first-launch work)
            fn(*st)
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        # a spin kernel ahead of the timed loop keeps the GPU busy while the host
        # queues the calls, so host-side call overhead cannot open gaps between them
        torch.cuda._sleep(int(n * 400_000))
        a.record()
        for i in range(n):
            fn(*sets[i % copies])
        b.record()
        torch.cuda.synchronize()
        del sets
        return a.elapsed_time(b) / n

    res = {}

    def want(name):
        return only is None or name.startswith(only)

    def nbytes_of(inputs):
        return sum(t.numel() * t.element_size() for t in inputs if isinstance(t, torch.Tensor))

    def hbm(name, fn, inputs, nbytes):
        if not want(name):
            return
        ms = timed(fn, inputs, nbytes_of(inputs))
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1), "bytes": nbytes,
                     "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4)}

    def tensor(name, fn, inputs, flop):
        if not want(name):
            return
        ms = timed(fn, inputs, nbytes_of(inputs))
        tf = flop / (ms / 1e3) / 1e12
        res[name] = {"us": round(ms * 1e3, 2), "TFLOP/s": round(tf, 1), "flop": flop,
                     "frac_of_bf16": round(tf / peaks["bf16_tflops"], 4)}

    g = torch.Generator().manual_seed(0)
    gu = torch.randn(16384, 4096, generator=g).to(torch.bfloat16).to(device)
    go = torch.randn(16384, 2048, generator=g).to(torch.bfloat16).to(device)
    hbm("swiglu_fwd [16384,4096]", lambda a: ops.swiglu(a), (gu,), 201_326_592)
    hbm("swiglu_bwd [16384,4096]", lambda a, b: ops.swiglu_backward(a, b), (gu, go), 335_544_320)
    del gu, go
    x = torch.randn(32768, 768, generator=g).to(torch.bfloat16).to(device)
    r = torch.randn(32768, 768, generator=g).to(torch.bfloat16).to(device)
    gn = torch.randn(32768, 768, generator=g).to(torch.bfloat16).to(device)
    hbm("residual_rmsnorm_fwd [32768,768]", lambda a, b: ops.residual_rms_norm(a, b, None, 1e-6), (r, x),
        201_326_592)
    hbm("rmsnorm_bwd [32768,768]", lambda a, b, c: ops.rms_norm_backward(a, None, b, c, 1e-6), (x, r, gn),
        201_326_592)
    del x, r, gn
    B, T, H, D = 8, 2048, 6, 128
    q = torch.randn(B, T, H, D, generator=g).to(torch.bfloat16).to(device)
    k = torch.randn(B, T, H, D, generator=g).to(torch.bfloat16).to(device)
    c1, s1 = RotaryEmbedding(D, 10_000.0, 0.25)(T, device, torch.bfloat16)
    cos = c1.transpose(1, 2).contiguous()
    sin = s1.transpose(1, 2).contiguous()
    dq = torch.randn_like(q)
    dk = torch.randn_like(k)
    hbm("qk_norm_rope_fwd [8,2048,6,128]", lambda a, b: ops.qk_norm_rope(a, b, cos, sin, 1e-6), (q, k),
        100_663_296)
    hbm("qk_norm_rope_bwd [8,2048,6,128]",
        lambda a, b, c, d: ops.qk_norm_rope_backward(a, b, c, d, cos, sin, 1e-6), (q, k, dq, dk), 150_994_944)
    xq = torch.randn(8, 2048, 768, generator=g).to(torch.bfloat16).to(device)
    wq = (torch.randn(2304, 768, generator=g) * 0.02).to(torch.bfloat16).to(device)
    tensor("qkv_rope_fwd X[16384,768] W[2304,768]", lambda a: ops.qkv_rope(a, wq, c1, s1, 6, 6, 1e-6), (xq,),
           57_982_058_496)
    xg = torch.randn(32768, 768, generator=g).to(torch.bfloat16).to(device)
    wg = (torch.randn(4096, 768, generator=g) * 0.02).to(torch.bfloat16).to(device)
    tensor("gate_up_swiglu X[32768,768] W[4096,768]", lambda a: ops.gate_up_swiglu(a, wg), (xg,),
           2 * 32768 * 768 * 4096)
    del xg, wg
    # o_proj / down projection with the residual add + RMSNorm in the GEMM epilogue (d12 shapes),
    # beside the unfused chain it replaces (cuBLAS GEMM + residual_rms_norm kernel).  Bound: the
    # slower of the FLOPs at the bf16 peak and the bytes (read y, W, residual; write out, norm)
    # at the HBM peak: o_proj is HBM-bound, down is tensor-bound.
    for name, K in (("o_proj", 768), ("down", 2048)):
        key = f"proj_norm {name} y[32768,{K}] W[768,{K}]"
        if not want(key):
            continue
        yd = torch.randn(32768, K, generator=g).to(torch.bfloat16).to(device)
        wd = (torch.randn(768, K, generator=g) * 0.02).to(torch.bfloat16).to(device)
        rd = torch.randn(32768, 768, generator=g).to(torch.bfloat16).to(device)
        flop = 2 * 32768 * 768 * K
        nbytes = 2 * (32768 * K + 768 * K + 3 * 32768 * 768 + 32768 * 768)
        ms = timed(lambda a, b: ops.proj_residual_norm(a, wd, b, 1e-6), (yd, rd), nbytes_of((yd, rd)))
        ms_ref = timed(lambda a, b: ops.residual_rms_norm(b, torch.nn.functional.linear(a, wd), None, 1e-6),
                       (yd, rd), nbytes_of((yd, rd)))
        t_tensor = flop / (peaks["bf16_tflops"] * 1e12) * 1e3
        t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9) * 1e3
        res[key] = {"us": round(ms * 1e3, 2), "TFLOP/s": round(flop / (ms / 1e3) / 1e12, 1),
                    "GB/s": round(nbytes / (ms / 1e3) / 1e9, 1), "flop": flop, "bytes": nbytes,
                    "bound": "tensor" if t_tensor >= t_hbm else "hbm",
                    "frac_of_roofline": round(max(t_tensor, t_hbm) / ms, 4),
                    "unfused_us": round(ms_ref * 1e3, 2)}
        del yd, wd, rd
    # down projection backward with the SwiGLU backward in its epilogue (d12 shape): HBM-bound,
    # 2*M*C*H = 103 GFLOP against 590 MB (read grad_y, gate_up, W_down; write grad_gate_up)
    if want("swiglu_down_bwd"):
        gyd = torch.randn(32768, 768, generator=g).to(torch.bfloat16).to(device)
        gud = torch.randn(32768, 4096, generator=g).to(torch.bfloat16).to(device)
        wdn = (torch.randn(768, 2048, generator=g) * 0.02).to(torch.bfloat16).to(device)
        outd = torch.empty_like(gud)
        hbm("swiglu_down_bwd dY[32768,768] W[768,2048] gate_up[32768,4096]",
            lambda a, b: ops.swiglu_down_grad(a, wdn, b, out=outd), (gyd, gud),
            2 * (32768 * 768 + 2 * 32768 * 4096 + 768 * 2048))
        del gyd, gud, wdn, outd
    # attention forward (tcgen05 kernel) at the d12 shape, full causal, beside torch SDPA (cuDNN) on
    # the same inputs: tensor-bound, 4*D FLOPs per causal (query, key) pair (Q K^T and P V)
    key = "attention_fwd [16,2048,6,128] causal"
    if want(key):
        qa, ka, va = (torch.randn(16, 2048, 6, 128, generator=g).to(torch.bfloat16).to(device) for _ in range(3))
        flop = 4 * 128 * (2048 * 2049 // 2) * 16 * 6
        ms = timed(lambda a, b, c: ops.attention(a, b, c, 0, 128 ** -0.5), (qa, ka, va), nbytes_of((qa, ka, va)))
        ms_ref = timed(lambda a, b, c: torch.nn.functional.scaled_dot_product_attention(
            a.transpose(1, 2), b.transpose(1, 2), c.transpose(1, 2), is_causal=True), (qa, ka, va),
            nbytes_of((qa, ka, va)))
        tf = flop / (ms / 1e3) / 1e12
        res[key] = {"us": round(ms * 1e3, 2), "TFLOP/s": round(tf, 1), "flop": flop,
                    "frac_of_bf16": round(tf / peaks["bf16_tflops"], 4), "sdpa_us": round(ms_ref * 1e3, 2)}
        del qa, ka, va
    # attention backward (tcgen05 kernel) at the d12 shape with the reference's 512-key window
    # (where it runs) and full causal, beside the library backward on the same inputs
    # (flash_attn's windowed backward; cuDNN's SDPA backward): 10*D FLOPs per unmasked
    # (query, key) pair (S, dP, dV, dK, dQ)
    key = "attention_bwd [16,2048,6,128] window 512"
    if want(key):
        qa, ka, va, ga = (torch.randn(16, 2048, 6, 128, generator=g).to(torch.bfloat16).to(device) for _ in range(4))
        sc = 128 ** -0.5
        entry = {}
        old = ops.ATTENTION_BWD["mode"]
        try:
            for w, tag in ((512, ""), (0, "causal_")):
                oa, la = ops.attention(qa, ka, va, w, sc)
                for mode, name in (("native", "us"), ("library", "library_us")):
                    ops.ATTENTION_BWD["mode"] = mode
                    ms = timed(lambda a, b, c, d_, o=oa, l=la, w=w: ops.attention_backward(d_, a, b, c, o, l, w, sc),
                               (qa, ka, va, ga), nbytes_of((qa, ka, va, ga)))
                    entry[tag + name] = round(ms * 1e3, 2)
                del oa, la
        finally:
            ops.ATTENTION_BWD["mode"] = old
        pairs = 512 * 513 // 2 + (2048 - 512) * 512
        flop = 10 * 128 * pairs * 16 * 6
        tf = flop / (entry["us"] / 1e6) / 1e12
        res[key] = {"us": entry["us"], "TFLOP/s": round(tf, 1), "flop": flop,
                    "frac_of_bf16": round(tf / peaks["bf16_tflops"], 4), "flash_attn_us": entry["library_us"],
                    "causal_us": entry["causal_us"], "causal_cudnn_us": entry["causal_library_us"]}
        del qa, ka, va, ga
    if not want("qkv_rope_bwd"):
        return res
    qo, ko, vo, rs = ops.qkv_rope(xq, wq, c1, s1, 6, 6, 1e-6)
    gv = torch.randn_like(vo)
    tensor("qkv_rope_bwd (dX+dW)",
           lambda a, b, c, d, e, f, h: ops.qkv_rope_backward(a, wq, b, c, d, c1, s1, e, f, h, 6, 6, 1e-6, True,
                                                             True),
           (xq, qo, ko, rs, dq, dk, gv), 115_964_116_992)
    return res


# ---------------------------------------------------------------------------
# reference arm: the reference algorithm on the host cores
# ---------------------------------------------------------------------------
def run_reference(args, d: Dist) -> dict | None:
    if d.rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    if args.workload == "lm_head":
        n = args.ref_tokens
        for _ in range(args.warmup):
            lm_cpu_sample(n)
        times = [lm_cpu_sample(n) for _ in range(args.steps)]
        total = sum(times)
        value = n * args.steps / total
        sample = (f"oracle (torch CPU fp32) LM-head+CE fwd+bwd, {n} tokens per step of the 32768-token "
                  "batch, full V=32768, C=768")
        metric = "LM-head+CE fwd/bwd tokens/s"
        cfg = {"workload": "lm_head_ce C4: hidden [32768,768] x W [32768,768], fwd+bwd",
               "tokens_per_gpu": LM["M"], "hidden": LM["C"], "vocab": LM["V"], "ignore_index": -1}
    else:
        for _ in range(args.warmup):
            d12_cpu_sample()
        times = [d12_cpu_sample() for _ in range(args.steps)]
        total = sum(times)
        value = 2048 * args.steps / total
        sample = ("port: oracle d12 model (torch CPU fp32; a restatement of the reference LanguageModel, "
                  "which does not travel to the GPU box; the package's torch formulation equals the "
                  "reference model on its golden fixture to 1e-5) forward+backward, 1x2048 tokens per "
                  "step of the 2^20-token global batch; optimizer step excluded")
        metric = "d12 step tok/s"
        cfg = d12_config(1, 32)
    ms = total / args.steps * 1e3
    return {"impl": "reference", "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": d.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "config": cfg,
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def _claim_stdout():
    """Keep the process's stdout for the result line alone: file descriptor 1
    is pointed at stderr for the rest of the run (so a library that prints to
    stdout, such as NCCL's version banner, lands on stderr) and the returned
    stream writes to the original stdout."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def main() -> None:
    result_out = _claim_stdout()

    def emit(obj) -> None:
        result_out.write(json.dumps(obj) + "\n")
        result_out.flush()

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", choices=("lm_head", "d12"), default="d12")
    ap.add_argument("--max-grad-norm", type=float, default=1.0,
                    help="global gradient-norm clip in the d12 step (the reference's --max-grad-norm; "
                         "its default 0 skips the clip, this bench includes it so the step does all of "
                         "the reference's per-step work)")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-operator section")
    ap.add_argument("--attention-window", type=int, default=0,
                    help="d12 variant: sliding window on every layer but each 4th and the last "
                         "(the reference's default pattern); 0 (default, BASELINE config 5) = full causal")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-tokens", type=int, default=1024, help="tokens per reference-arm step")
    ap.add_argument("--tokens", type=int, default=None,
                    help="override the LM-head token count (smaller cases for ncu captures)")
    ap.add_argument("--op", default=None,
                    help="run only the per-operator section for operators starting with this name "
                         "('all' for every operator) and print {\"ops\": ...}; for ncu captures")
    ap.add_argument("--op-iters", type=int, default=1, help="timed calls per operator with --op")
    args = ap.parse_args()
    if args.tokens is not None:
        LM["M"] = args.tokens
    if args.warmup < 3 and args.impl == "b200":
        ap.error("--warmup must be >= 3")

    d = Dist()
    if args.impl == "reference":
        d.init(backend="gloo")
        out = run_reference(args, d)
        if out is not None:
            emit(out)
        d.close()
        return

    d.init()
    device = torch.device("cuda", d.local_rank)
    torch.cuda.set_device(device)
    if args.op is not None:
        if d.rank == 0:
            res = bench_ops(device, iters=args.op_iters, only=None if args.op == "all" else args.op)
            emit({"ops": res})
        d.close()
        return
    if args.workload == "lm_head":
        out = bench_lm_head(args, d, device)
    else:
        out = bench_d12(args, d, device)
    if d.rank == 0:
        if not args.no_ops and d.world == 1:
            if args.workload == "d12":
                lm = bench_lm_head(argparse.Namespace(steps=10, warmup=3), d, device)
                out["lm_head_c4"] = {k: lm[k] for k in ("metric", "value", "unit", "ms_per_step", "config",
                                                        "roofline", "kernel_breakdown", "e2e", "gpu_launches")}
            out["ops"] = bench_ops(device)
        if not args.no_cpu_baseline and d.world == 1:
            out["cpu_baseline"] = cpu_baseline_lm() if args.workload == "lm_head" else cpu_baseline_d12()
        emit(out)
    d.close()


if __name__ == "__main__":
    main()
