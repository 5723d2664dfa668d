#!/usr/bin/env python
"""Benchmark of Sion's operator hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]

Default workload: HGEMM fp16 M=N=K=4096, A row-major, B column-major (stored
N x K, the reference's "nt" kernel), fp32 accumulate, fp16 output, seed 1 —
the configuration the headline metric (HGEMM/FlashAttn/SGEMM TFLOPS) is quoted
on. Other workloads: sgemm_f32_1024, hgemm_f16_128x8192x16384_nt,
flash_attn_fwd_f16_4x32x8192x128, hgemm_f16_16384_nt.

A step is one operator call on one synthetic batch. Each rank runs its own
copy of the workload (independent units, no data-path collective: weak
scaling). Steps are timed one by one with CUDA events on the launching stream;
between steps a 512 MiB buffer is written to flush the 126 MB L2 (outside the
events). Workloads whose inputs are larger than the L2 also read a 256 MiB
buffer after that write, so that the L2 holds clean lines: a streaming kernel
would otherwise be charged the write-back of the flush buffer (measured: the
skinny HGEMM 74 us after the write alone, 64 us after write + read). The
reported time is the max over ranks of the mean step time.

`e2e` times the same call through the C ABI with pinned HOST buffers: every
step copies its inputs host-to-device, runs the kernel and copies its output
device-to-host, all inside the timed region. Steps are pipelined the way a
serving loop would run them: copy-in, compute and copy-out on three streams
with two device buffer sets, so step k+1's inputs cross PCIe while step k
computes and step k-1's output comes back (PCIe is full duplex). The time is
the whole K-step loop divided by K (max over ranks).

--impl reference: the reference's host path (BASELINE: LibTorch CPU
torch.matmul / naive fp32 softmax attention, the reference tests' comparison
path) timed on the host cores on a bounded row sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from sion_b200 import workloads as W  # noqa: E402

DEFAULT_WORKLOAD = W.HGEMM_4096.name
METRIC = "HGEMM/FlashAttn/SGEMM TFLOPS per B200 and % of peak; 1/2/4/8-GPU aggregate"
L2_FLUSH_BYTES = 512 << 20
L2_CLEAN_BYTES = 256 << 20


L2_BYTES = 126 * 10**6


class L2Flush:
    """Evicts the L2 between timed steps: a write larger than the L2; with
    clean=True also a read larger than the L2 after it, so that the next step
    starts from cold, clean lines."""

    def __init__(self, device, clean: bool = False):
        import torch
        self.w = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        self.r = torch.zeros(L2_CLEAN_BYTES // 4, dtype=torch.float32, device=device) \
            if clean else None
        self.acc = torch.zeros((), dtype=torch.float32, device=device)

    def __call__(self, i):
        import torch
        self.w.fill_(float(i))
        if self.r is not None:
            torch.sum(self.r, dim=0, out=self.acc)

    @property
    def description(self) -> str:
        if self.r is None:
            return "flushed between steps (512 MiB write outside the timed events)"
        return ("inputs larger than L2; flushed between steps (512 MiB write, then 256 MiB "
                "read so the L2 holds clean lines, outside the timed events)")


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d["bf16_tflops"],
                "tflops_sustained": d.get("bf16_tflops_sustained"),
                "sm_max_mhz": d.get("sm_max_mhz", 1965.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0,
            "sm_max_mhz": 1965.0, "source": "fallback"}


def _ncu_traffic(workload: str):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get(workload)
    return None


class ClockSampler:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) > 8
                          for i in range(4) if r[5 + i].lower().startswith("active")})
        loaded = [s for s in sm if s > 0.5 * (max(mx) if mx else 1)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


# ----------------------------------------------------------------- workloads
class GemmRunner:
    def __init__(self, cfg: W.GemmConfig, device, shard_rank=None, world=1):
        from sion_b200 import abi
        self.abi = abi
        self.cfg = cfg
        A, B = W.gemm_inputs(cfg)
        self.work_fraction = 1.0
        if shard_rank is not None:
            # strong scaling: this rank owns a contiguous column block of C
            from sion_b200.shard import gemm_column_shard
            n0, n1 = gemm_column_shard(cfg.N, world, shard_rank)
            B = (B[n0:n1] if cfg.b_layout == "nk" else B[:, n0:n1]).contiguous()
            self.work_fraction = (n1 - n0) / cfg.N
            cfg = W.GemmConfig(cfg.name, cfg.M, n1 - n0, cfg.K, cfg.dtype, cfg.b_layout, cfg.dist,
                               cfg.std, cfg.seed)
            self.cfg = cfg
        self.hA = A.pin_memory()
        self.hB = B.pin_memory()
        self.dA = self.hA.to(device)
        self.dB = self.hB.to(device)
        dt = torch.float32 if cfg.dtype == "f32" else torch.float16
        self.dC = torch.empty(cfg.M, cfg.N, dtype=dt, device=device)
        self.hC = torch.empty(cfg.M, cfg.N, dtype=dt).pin_memory()
        self.launches_per_step = 1
        # end-to-end pipeline: host buffers and two device buffer sets
        self.h_in, self.h_out = [self.hA, self.hB], [self.hC]
        self.d_in = [[self.dA, self.dB], [torch.empty_like(self.dA), torch.empty_like(self.dB)]]
        self.d_out = [[self.dC], [torch.empty_like(self.dC)]]

    def compute(self, slot):
        c = self.cfg
        (A, B), (C,) = self.d_in[slot], self.d_out[slot]
        if c.dtype == "f32":
            self.abi.sgemm(A, B, C)
        else:
            self.abi.hgemm(A, B, C, b_layout=self.abi.B_NK if c.b_layout == "nk" else self.abi.B_KN)

    def step(self):
        self.compute(0)

    @property
    def h2d_bytes(self):
        return self.hA.numel() * self.hA.element_size() + self.hB.numel() * self.hB.element_size()

    @property
    def d2h_bytes(self):
        return self.hC.numel() * self.hC.element_size()

    def algorithmic(self):
        c = self.cfg
        if c.name == W.HGEMM_SKINNY.name:
            return "hbm", float(c.io_bytes)
        return "tensor" if c.dtype == "f16" else "ffma", c.flops


class AttnRunner:
    def __init__(self, cfg: W.AttnConfig, device, shard_rank=None, world=1):
        from sion_b200 import abi
        self.abi = abi
        self.cfg = cfg
        Q, K, V = W.attn_inputs(cfg)
        self.work_fraction = 1.0
        if shard_rank is not None:
            # strong scaling: this rank owns a contiguous group of (b, h) pairs
            from sion_b200.shard import attention_shard
            s0, s1 = attention_shard(cfg.B, cfg.H, world, shard_rank)
            Q, K, V = [t.reshape(cfg.B * cfg.H, cfg.S, cfg.D)[s0:s1].reshape(1, s1 - s0, cfg.S,
                                                                            cfg.D).contiguous()
                       for t in (Q, K, V)]
            self.work_fraction = (s1 - s0) / (cfg.B * cfg.H)
            cfg = W.AttnConfig(cfg.name, 1, s1 - s0, cfg.S, cfg.D, cfg.seed, cfg.causal,
                               cfg.backward)
            self.cfg = cfg
        self.h = [t.pin_memory() for t in (Q, K, V)]
        self.d = [t.to(device) for t in self.h]
        self.dO = torch.empty_like(self.d[0])
        self.dL = torch.empty(cfg.B, cfg.H, cfg.S, device=device)
        self.hO = torch.empty_like(self.h[0]).pin_memory()
        self.hL = torch.empty(cfg.B, cfg.H, cfg.S).pin_memory()
        self.launches_per_step = 1
        if cfg.backward:
            # forward outputs and the incoming gradient are inputs of the step
            abi.flash_attn_fwd(self.d[0], self.d[1], self.d[2], self.dO, self.dL,
                               causal=cfg.causal)
            g = W.attn_grad_input(W.CONFIGS[cfg.name])
            if shard_rank is not None:
                g = g.reshape(-1, cfg.S, cfg.D)[s0:s1].reshape(self.d[0].shape).contiguous()
            self.h += [self.dO.cpu().pin_memory(), self.dL.cpu().pin_memory(), g.pin_memory()]
            self.d += [self.dO, self.dL, g.to(device)]
            self.grads = [torch.empty_like(self.d[0]) for _ in range(3)]
            self.hgrads = [torch.empty_like(self.h[0]).pin_memory() for _ in range(3)]
            self.ws = torch.empty(abi.flash_attn_bwd_workspace_size(cfg.H, cfg.B, cfg.S, cfg.D),
                                  dtype=torch.uint8, device=device)
            self.launches_per_step = 3  # Delta, backward, dQ conversion

    def step(self):
        if self.cfg.backward:
            Q, K, V, O, L, dO = self.d
            self.abi.flash_attn_bwd(Q, K, V, O, dO, L, *self.grads, causal=self.cfg.causal,
                                    workspace=self.ws)
            return
        self.abi.flash_attn_fwd(self.d[0], self.d[1], self.d[2], self.dO, self.dL,
                                causal=self.cfg.causal)

    def _e2e_sets(self):
        # end-to-end pipeline: host buffers and two device buffer sets
        if self.cfg.backward:
            self.h_in, self.h_out = self.h, self.hgrads
            outs = self.grads
        else:
            self.h_in, self.h_out = self.h, [self.hO, self.hL]
            outs = [self.dO, self.dL]
        self.d_in = [list(self.d), [torch.empty_like(t) for t in self.d]]
        self.d_out = [list(outs), [torch.empty_like(t) for t in outs]]

    def compute(self, slot):
        if not hasattr(self, "d_in"):
            self._e2e_sets()
        ins, outs = self.d_in[slot], self.d_out[slot]
        if self.cfg.backward:
            Q, K, V, O, L, dO = ins
            self.abi.flash_attn_bwd(Q, K, V, O, dO, L, *outs, causal=self.cfg.causal,
                                    workspace=self.ws)
        else:
            self.abi.flash_attn_fwd(ins[0], ins[1], ins[2], outs[0], outs[1],
                                    causal=self.cfg.causal)

    @property
    def h2d_bytes(self):
        return sum(t.numel() * t.element_size() for t in self.h)

    @property
    def d2h_bytes(self):
        if self.cfg.backward:
            return sum(t.numel() * t.element_size() for t in self.hgrads)
        return self.hO.numel() * 2 + self.hL.numel() * 4

    def algorithmic(self):
        return "tensor", self.cfg.flops


def e2e_pipeline(runner, steps, world):
    """Per-step time (ms, max over ranks) of `steps` end-to-end steps: H2D of
    the step's inputs from pinned host memory, the kernel, D2H of its output.
    Copy-in, compute and copy-out run on three streams over two device buffer
    sets; a buffer set is refilled only after the compute that read it, and a
    compute writes an output set only after that set's previous copy-out."""
    if hasattr(runner, "_e2e_sets") and not hasattr(runner, "d_in"):
        runner._e2e_sets()
    s_in, s_cmp, s_out = (torch.cuda.Stream() for _ in range(3))
    ev = lambda: torch.cuda.Event()
    in_ready, cmp_done, out_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    used = [False, False]

    def one(k):
        slot = k % 2
        with torch.cuda.stream(s_in):
            if used[slot]:
                s_in.wait_event(cmp_done[slot])
            for d, h in zip(runner.d_in[slot], runner.h_in):
                d.copy_(h, non_blocking=True)
            in_ready[slot].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(in_ready[slot])
            if used[slot]:
                s_cmp.wait_event(out_done[slot])
            runner.compute(slot)
            cmp_done[slot].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(cmp_done[slot])
            for h, d in zip(runner.h_out, runner.d_out[slot]):
                h.copy_(d, non_blocking=True)
            out_done[slot].record(s_out)
        used[slot] = True

    for k in range(2):
        one(k)
    torch.cuda.synchronize()
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    s_cmp.wait_stream(s_in)
    s_out.wait_stream(s_in)
    for k in range(steps):
        one(k)
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_cmp)
    t1.record(s_out)
    torch.cuda.synchronize()
    return max_over_ranks(t0.elapsed_time(t1) / steps, world)


def make_runner(name, device, shard_rank=None, world=1):
    cfg = W.CONFIGS[name]
    cls = AttnRunner if isinstance(cfg, W.AttnConfig) else GemmRunner
    return cls(cfg, device, shard_rank, world)


# ----------------------------------------------------------------- CPU host path
def cpu_sample(cfg, budget_s: float = 10.0):
    """Time the reference's host path on a bounded row sample; returns
    (TFLOPS, threads, description)."""
    threads = torch.get_num_threads()
    if isinstance(cfg, W.AttnConfig):
        Q, K, V = W.attn_inputs(W.AttnConfig(cfg.name, 1, 1, cfg.S, cfg.D, cfg.seed))
        q, k, v = Q[0, 0].float(), K[0, 0].float(), V[0, 0].float()
        rows = 1024
        flops_per = 4.0 * rows * cfg.S * cfg.D
        def fn():
            s = (q[:rows] @ k.t()) / (cfg.D ** 0.5)
            p = torch.softmax(s, dim=-1)
            return p @ v
        desc = (f"naive fp32 softmax(QK^T/sqrt(D))V, {rows} query rows x {cfg.S} keys of one "
                f"(b,h) per call, torch CPU, repeated for ~{budget_s:.0f} s")
        if cfg.backward:
            g = torch.randn(rows, cfg.D, generator=torch.Generator().manual_seed(cfg.seed))
            flops_per = 10.0 * rows * cfg.S * cfg.D
            def fn():  # noqa: F811
                p = torch.softmax((q[:rows] @ k.t()) / (cfg.D ** 0.5), dim=-1)
                dv = p.t() @ g
                dp = g @ v.t()
                ds = p * (dp - (dp * p).sum(-1, keepdim=True))
                return ds @ k, ds.t() @ q[:rows], dv
            desc = (f"naive fp32 attention backward (P recomputed; dV, dP, dS, dQ, dK), "
                    f"{rows} query rows x {cfg.S} keys of one (b,h) per call, torch CPU, "
                    f"repeated for ~{budget_s:.0f} s")
    else:
        rows = min(cfg.M, 512)
        A, B = W.gemm_inputs(cfg, M=rows)
        a = A.float()
        b = B.float()
        if cfg.b_layout == "nk":
            b = b.t()
        flops_per = 2.0 * rows * cfg.N * cfg.K
        def fn():
            return torch.matmul(a, b)
        upcast = "fp32 inputs" if A.dtype == torch.float32 else "fp16 inputs upcast"
        desc = (f"torch.matmul fp32 on CPU ({upcast}), {rows} rows of A x full B "
                f"per call, repeated for ~{budget_s:.0f} s")
    fn()
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return flops_per * n / el / 1e12, threads, desc


# ----------------------------------------------------------------- main
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reference_gpu_timing(cfg, steps: int, warmup: int):
    """Time the reference's own kernels (oracle/_ref, built from the unmodified
    reference sources for sm_100a) on this workload, same protocol as our arm
    (L2 flushed between steps, CUDA events). None when unavailable."""
    try:
        from oracle import reference as ref
    except Exception:
        return None
    if not (ref.available() and torch.cuda.is_available()):
        return None
    dev = torch.device("cuda", 0)
    if isinstance(cfg, W.AttnConfig) and (cfg.backward or cfg.causal):
        return {"unavailable": "the reference has no backward or masked attention kernel"}
    if isinstance(cfg, W.AttnConfig):
        Q, K, V = [t.to(dev) for t in W.attn_inputs(cfg)]
        O = torch.empty_like(Q)
        step = lambda: ref.flash_attn(Q, K, V, O)  # noqa: E731
    else:
        A, B = [t.to(dev) for t in W.gemm_inputs(cfg)]
        if cfg.dtype == "f32":
            C = torch.empty(cfg.M, cfg.N, device=dev)
            step = lambda: ref.sgemm(A, B, C)  # noqa: E731
        else:
            C = torch.empty(cfg.M, cfg.N, dtype=torch.half, device=dev)
            step = lambda: ref.hgemm(A, B, C, nt=cfg.b_layout == "nk")  # noqa: E731
    flush = L2Flush(dev, clean=cfg.io_bytes > L2_BYTES)
    for _ in range(warmup):
        step()
    times = []
    for i in range(steps):
        flush(i)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        step()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    ms = statistics.mean(times)
    return {"value": cfg.flops / (ms * 1e-3) / 1e12, "unit": "TFLOPS", "ms_per_step": ms,
            "what": "the reference's own kernels (fp16-accumulate HGEMM/attention, SIMT "
                    "SGEMM) built unmodified for sm_100a, timed on the same B200"}


def run_reference(args, world, rank):
    if rank != 0:
        return 0
    cfg = W.CONFIGS[args.workload]
    torch.set_num_threads(os.cpu_count() or 1)
    vals = []
    for _ in range(args.warmup):
        cpu_sample(cfg, budget_s=1.0)
    desc, threads = "", 1
    for _ in range(args.steps):
        v, threads, desc = cpu_sample(cfg, budget_s=max(2.0, 20.0 / max(args.steps, 1)))
        vals.append(v)
    value = statistics.mean(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded torch CPU generator)",
        "config": {"workload": cfg.name, "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    try:
        line["reference_gpu"] = reference_gpu_timing(cfg, max(args.steps, 5), args.warmup)
    except Exception as e:  # the comparator is informative only
        line["reference_gpu"] = {"unavailable": str(e)[:200]}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(W.CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard", action="store_true",
                    help="strong scaling: split one workload over the ranks (GEMM N-column "
                         "blocks, attention (b, h) groups) instead of one copy per rank")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world, rank, local = init_dist() if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    if args.impl == "reference":
        return run_reference(args, world, rank)

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    runner = make_runner(args.workload, device, rank if args.shard else None, world)
    full_cfg = W.CONFIGS[args.workload]
    flush = L2Flush(device, clean=full_cfg.io_bytes > L2_BYTES)
    stream = torch.cuda.current_stream()

    for _ in range(args.warmup):
        runner.step()
    torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(torch.cuda.current_device() if world == 1 else local)
    barrier(world)
    torch.cuda.synchronize()
    with sampler:
        time.sleep(0.25)
        t_wall = time.perf_counter()
        for i in range(args.steps):
            flush(i)
            starts[i].record(stream)
            runner.step()
            ends[i].record(stream)
        torch.cuda.synchronize()
        t_wall = time.perf_counter() - t_wall
    barrier(world)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    mean_ms = statistics.mean(step_ms)
    ms = max_over_ranks(mean_ms, world)

    bound, work = runner.algorithmic()
    job_flops = full_cfg.flops if args.shard else world * full_cfg.flops
    value = job_flops / (ms * 1e-3) / 1e12

    # e2e through the C ABI with host buffers, steps pipelined over three streams
    e2e_ms = e2e_pipeline(runner, args.steps, world)
    e2e_val = job_flops / (e2e_ms * 1e-3) / 1e12

    peaks = _peaks()
    if bound == "hbm":
        achieved = work / (mean_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                "unit": "GB/s"}
    elif bound == "ffma":
        ffma_peak = 148 * 128 * 2 * peaks["sm_max_mhz"] * 1e6 / 1e12
        achieved = work / (mean_ms * 1e-3) / 1e12
        roof = {"bound": "ffma", "achieved": achieved, "peak": ffma_peak, "unit": "TFLOP/s"}
    else:
        achieved = work / (mean_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["tflops"],
                "unit": "TFLOP/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["peak_source"] = peaks["source"] + (" (148 SM x 128 FFMA x 2 x max clock)"
                                             if bound == "ffma" else "")
    roof["traffic"] = _ncu_traffic(runner.cfg.name)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        v, threads, desc = cpu_sample(runner.cfg, budget_s=10.0)
        cpu = {"value": v, "unit": "TFLOPS", "cores": threads, "kind": "port", "sample": desc}

    clocks = sampler.summary()
    if rank == 0:
        cfg = full_cfg
        par = (f"shards x{world} (N-column / (b,h) blocks, no collective)" if args.shard
               else f"replicas x{world} (independent units)")
        conf = {"workload": cfg.name, "parallelism": par,
                "l2": flush.description}
        if isinstance(cfg, W.GemmConfig):
            conf.update({"M": cfg.M, "N": cfg.N, "K": cfg.K, "b_layout": cfg.b_layout})
        else:
            conf.update({"B": cfg.B, "H": cfg.H, "S": cfg.S, "D": cfg.D})
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if args.shard else "weak",
            "vs_baseline": None,
            "dtype": "f32" if getattr(cfg, "dtype", "f16") == "f32" else "f16 (fp32 accumulate)",
            "data": "synthetic (seeded torch CPU generator)", "config": conf,
            "frac_of_peak": value / world / (roof["peak"] if bound != "hbm" else 1) if bound != "hbm" else None,
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "TFLOPS", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": runner.h2d_bytes,
                    "d2h_bytes_per_step": runner.d2h_bytes,
                    "pipeline": "copy-in / compute / copy-out streams, 2 device buffer sets"},
            "gpu_launches": args.steps * runner.launches_per_step,
            "clocks": clocks, "wall_s_timed": t_wall,
            "step_ms_min": min(step_ms), "step_ms_median": statistics.median(step_ms),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
