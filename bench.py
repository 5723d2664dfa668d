#!/usr/bin/env python
"""Benchmark of Sion's operator hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--shard]

Default (the suite): the headline is HGEMM fp16 M=N=K=16384 (A row-major, B
column-major = stored N x K, fp32 accumulate, fp16 output, seed 4), sharded by
N-column blocks over the ranks (strong scaling: N=1 computes the whole
product, N=8 one eighth of the columns per GPU; no data-path collective). The
optional NCCL all-gather of C over NVLink is timed after the compute as its own
field (`allgather`) and kept out of `value`. The same JSON line carries one
sub-record per other configuration (`configs`): SGEMM 1024^3 (FFMA roofline),
HGEMM 4096^3 (tensor roofline), skinny HGEMM 128x8192x16384 (HBM roofline) and
flash-attention forward 4x32x8192x128 (tensor roofline). Attention is sharded
over (b, h) groups like the headline (strong scaling); the three smaller GEMMs
run one copy per rank (weak scaling, said in each sub-record).

--workload NAME runs one workload alone (one copy per rank, or split over the
ranks with --shard); the profiles use this form.

A step is one operator call on one synthetic batch. Steps are timed one by one
with CUDA events on the launching stream; between steps a 512 MiB buffer is
written to flush the 126 MB L2 (outside the events). Workloads whose inputs
are larger than the L2 also read a 256 MiB buffer after that write, so that the
L2 holds clean lines: a streaming kernel would otherwise be charged the
write-back of the flush buffer (measured: the skinny HGEMM 74 us after the
write alone, 64 us after write + read). The reported time is the max over
ranks of the mean step time.

`e2e` times the same call through the C ABI with pinned HOST buffers: every
step copies its inputs host-to-device, runs the kernel and copies its output
device-to-host, all inside the timed region. Two figures: `value` /
`ms_per_step_pipelined` run the steps the way a serving loop would (copy-in,
compute and copy-out on three streams with two device buffer sets, so step
k+1's inputs cross PCIe while step k computes and step k-1's output comes back)
and divide the loop time by K; `serial_ms_per_step` is one step with the three
phases back to back (latency). Both are max over ranks.

--impl reference: the reference's host path (LibTorch CPU torch.matmul /
naive fp32 softmax attention, the reference tests' comparison path) timed on
the host cores on a bounded row sample of the same workload, with the same
`config` as this arm; `ms_per_step` is the sample's time scaled to the whole
workload. Under torchrun every rank times its own shard with its share of the
host cores, and `value` is the sum over ranks.
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

    @staticmethod
    def describe(clean: bool) -> str:
        if not clean:
            return "flushed between steps (512 MiB write outside the timed events)"
        return ("inputs larger than L2; flushed between steps (512 MiB write, then 256 MiB "
                "read so the L2 holds clean lines, outside the timed events)")

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
        rows = min(1024, cfg.S)
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


def e2e_serial(runner, steps, world):
    """Latency (ms, max over ranks) of one end-to-end step with copy-in,
    compute and copy-out back to back on one stream (mean of `steps`)."""
    if hasattr(runner, "_e2e_sets") and not hasattr(runner, "d_in"):
        runner._e2e_sets()
    s = torch.cuda.Stream()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for k in range(steps + 1):
        barrier(world)
        torch.cuda.synchronize()
        with torch.cuda.stream(s):
            t0.record(s)
            for d, h in zip(runner.d_in[0], runner.h_in):
                d.copy_(h, non_blocking=True)
            runner.compute(0)
            for h, d in zip(runner.h_out, runner.d_out[0]):
                h.copy_(d, non_blocking=True)
            t1.record(s)
        torch.cuda.synchronize()
        if k:  # the first pass is a warm-up
            times.append(t0.elapsed_time(t1))
    return max_over_ranks(statistics.mean(times), world)


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
    dev = torch.device("cuda", torch.cuda.current_device())
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
            "n_gpus": 1,
            "what": "the reference's own kernels (fp16-accumulate HGEMM/attention, SIMT "
                    "SGEMM) built unmodified for sm_100a, timed on one B200 of the same box"}


HEADLINE = W.HGEMM_16384.name
# (workload, split over the ranks?) of the sub-records, in the order printed
SUITE = [(W.SGEMM_1024.name, False), (W.HGEMM_4096.name, False),
         (W.HGEMM_SKINNY.name, False), (W.FA_8192.name, True)]


def config_dict(cfg, world: int, shard: bool, l2: str | None = None) -> dict:
    if shard:
        how = ("N-column blocks of C" if isinstance(cfg, W.GemmConfig) else "(b, h) groups")
        par = f"shards x{world} ({how}, no data-path collective)"
    else:
        par = f"replicas x{world} (one independent copy per rank)"
    conf = {"workload": cfg.name, "parallelism": par}
    if l2:
        conf["l2"] = l2
    if isinstance(cfg, W.GemmConfig):
        conf.update({"M": cfg.M, "N": cfg.N, "K": cfg.K, "b_layout": cfg.b_layout,
                     "seed": cfg.seed})
    else:
        conf.update({"B": cfg.B, "H": cfg.H, "S": cfg.S, "D": cfg.D, "seed": cfg.seed,
                     "causal": cfg.causal, "backward": cfg.backward})
    return conf


def _dtype(cfg) -> str:
    return "f32" if getattr(cfg, "dtype", "f16") == "f32" else "f16 (fp32 accumulate)"


def measure(name: str, shard: bool, args, world: int, rank: int, local: int, device,
            cpu_budget: float, want_cpu: bool = True):
    """One workload: device-timed steps, e2e (pipelined and serial), roofline,
    clocks and (rank 0, N=1) the CPU host-path sample. Returns (record, runner)."""
    runner = make_runner(name, device, rank if shard else None, world)
    full_cfg = W.CONFIGS[name]
    flush = L2Flush(device, clean=full_cfg.io_bytes > L2_BYTES)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        runner.step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(local)
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
    del flush

    bound, work = runner.algorithmic()
    job_flops = full_cfg.flops if shard else world * full_cfg.flops
    value = job_flops / (ms * 1e-3) / 1e12

    e2e_ms = e2e_pipeline(runner, args.steps, world)
    serial_ms = e2e_serial(runner, max(2, min(args.steps, 5)), world)

    peaks = _peaks()
    # the roofline is this rank's dominant kernel: its own work over its own time
    if bound == "hbm":
        roof = {"bound": "hbm", "achieved": work / (mean_ms * 1e-3) / 1e9,
                "peak": peaks["hbm_gbs"], "unit": "GB/s"}
    elif bound == "ffma":
        roof = {"bound": "ffma", "achieved": work / (mean_ms * 1e-3) / 1e12,
                "peak": 148 * 128 * 2 * peaks["sm_max_mhz"] * 1e6 / 1e12, "unit": "TFLOP/s"}
    else:
        roof = {"bound": "tensor", "achieved": work / (mean_ms * 1e-3) / 1e12,
                "peak": peaks["tflops"], "unit": "TFLOP/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["peak_source"] = peaks["source"] + (" (148 SM x 128 FFMA x 2 x max clock)"
                                             if bound == "ffma" else " (burst)")
    tr = _ncu_traffic(full_cfg.name)
    roof["traffic"] = None if tr is None else tr * runner.work_fraction
    if tr is not None and runner.work_fraction != 1.0:
        roof["traffic_note"] = "full-workload capture scaled by this rank's share of the work"

    cpu = None
    if want_cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        v, threads, desc = cpu_sample(runner.cfg, budget_s=cpu_budget)
        cpu = {"value": v, "unit": "TFLOPS", "cores": threads, "kind": "port", "sample": desc}

    rec = {
        "value": value, "unit": "TFLOPS", "ms_per_step": ms,
        "scaling": "strong" if shard else "weak", "dtype": _dtype(full_cfg),
        "config": config_dict(full_cfg, world, shard, runner_l2(full_cfg)),
        "frac_of_peak": None if bound == "hbm" else value / world / roof["peak"],
        "roofline": roof, "cpu_baseline": cpu,
        "e2e": {"value": job_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
                "ms_per_step_pipelined": e2e_ms, "serial_ms_per_step": serial_ms,
                "serial_value": job_flops / (serial_ms * 1e-3) / 1e12,
                "h2d_bytes_per_step": runner.h2d_bytes, "d2h_bytes_per_step": runner.d2h_bytes,
                "pipeline": "copy-in / compute / copy-out streams, 2 device buffer sets"},
        "gpu_launches": args.steps * runner.launches_per_step,
        "clocks": sampler.summary(), "wall_s_timed": t_wall,
        "step_ms_min": min(step_ms), "step_ms_median": statistics.median(step_ms),
    }
    return rec, runner


def runner_l2(cfg) -> str:
    return L2Flush.describe(cfg.io_bytes > L2_BYTES)


def allgather_timing(runner, world: int, iters: int = 5):
    """NCCL all-gather of every rank's C column block (the optional
    reassembly of C over NVLink), timed alone after the compute. Blocks are
    gathered as [rank][M][N/ranks] (equal widths); GB/s counts the bytes each
    rank receives."""
    if world == 1:
        return None
    block = runner.d_out[0][0] if hasattr(runner, "d_out") else runner.dC
    out = torch.empty((world,) + tuple(block.shape), dtype=block.dtype, device=block.device)
    for _ in range(2):
        dist.all_gather_into_tensor(out, block.contiguous())
    torch.cuda.synchronize()
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(iters):
        dist.all_gather_into_tensor(out, block)
    t1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(t0.elapsed_time(t1) / iters, world)
    recv = block.numel() * block.element_size() * (world - 1)
    return {"ms": ms, "bytes_received_per_rank": recv,
            "gbs_per_rank": recv / (ms * 1e-3) / 1e9,
            "what": "NCCL all_gather_into_tensor of the C column blocks over NVLink, "
                    "timed separately; not part of value"}


def run_reference(args, world, rank):
    """The reference's host path on this arm's workload. Under torchrun every
    rank times its own shard with cores / world threads at the same time, and
    the values add up (gloo); rank 0 prints."""
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("gloo")
    cores = os.cpu_count() or 1
    threads = max(1, cores // world)
    torch.set_num_threads(threads)
    names = [args.workload] if args.workload else [HEADLINE] + [n for n, _ in SUITE]
    shard_of = {HEADLINE: True, **dict(SUITE)}
    recs = []
    for name in names:
        full = W.CONFIGS[name]
        shard = args.shard if args.workload else shard_of[name]
        cfg = full
        if shard and world > 1:
            if isinstance(full, W.GemmConfig):
                from sion_b200.shard import gemm_column_shard
                n0, n1 = gemm_column_shard(full.N, world, rank)
                cfg = W.GemmConfig(full.name, full.M, n1 - n0, full.K, full.dtype,
                                   full.b_layout, full.dist, full.std, full.seed)
            else:
                from sion_b200.shard import attention_shard
                s0, s1 = attention_shard(full.B, full.H, world, rank)
                cfg = W.AttnConfig(full.name, 1, s1 - s0, full.S, full.D, full.seed,
                                   full.causal, full.backward)
        budget = 20.0 / max(args.steps, 1) if name == names[0] else 4.0 / max(args.steps, 1)
        for _ in range(min(args.warmup, 3)):
            cpu_sample(cfg, budget_s=0.5)
        vals, desc = [], ""
        for _ in range(args.steps):
            v, _t, desc = cpu_sample(cfg, budget_s=max(0.5, budget))
            vals.append(v)
        mine = statistics.mean(vals)
        total = mine
        if world > 1:
            # every rank ran its own shard (or, for replicated workloads, its own
            # copy, as each rank of our arm does) on its share of the host cores
            t = torch.tensor([mine], dtype=torch.float64)
            dist.all_reduce(t)
            total = float(t.item())
        job_flops = full.flops if shard else world * full.flops
        ms = job_flops / (total * 1e12) * 1e3
        l2 = runner_l2(full)
        rec = {"value": total, "unit": "TFLOPS", "ms_per_step": ms,
               "ms_per_step_how": "host sample's throughput scaled to the whole workload",
               "scaling": "strong" if shard else "weak", "dtype": "f32",
               "config": config_dict(full, world, shard, l2),
               "cpu_baseline": {"value": total, "unit": "TFLOPS", "cores": threads * world,
                                "kind": "port", "sample": desc +
                                (f"; {world} ranks x {threads} threads, each on its own shard"
                                 if world > 1 else "")},
               "e2e": {"value": total, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}}
        recs.append(rec)
    if rank != 0:
        dist.destroy_process_group()
        return 0
    head = recs[0]
    line = {"impl": "reference", "metric": METRIC, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "vs_baseline": None,
            "data": "synthetic (seeded torch CPU generator)", **head}
    if len(recs) > 1:
        line["configs"] = {r["config"]["workload"]: r for r in recs[1:]}
    try:
        line["reference_gpu"] = reference_gpu_timing(W.CONFIGS[names[0]], 5, args.warmup)
    except Exception as e:  # the comparator is informative only
        line["reference_gpu"] = {"unavailable": str(e)[:200]}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=None, choices=sorted(W.CONFIGS),
                    help="one workload alone (default: the suite, headline HGEMM 16384^3)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-suite", action="store_true",
                    help="headline only (skip the sub-records of the other configs)")
    ap.add_argument("--shard", action="store_true",
                    help="with --workload: split it over the ranks (GEMM N-column blocks, "
                         "attention (b, h) groups) instead of one copy per rank")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, world, rank)

    world, rank, local = init_dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    if args.workload:
        head_name, head_shard, subs = args.workload, args.shard, []
    else:
        head_name, head_shard = HEADLINE, True
        subs = [] if args.no_suite else SUITE

    rec, runner = measure(head_name, head_shard, args, world, rank, local, device,
                          cpu_budget=10.0)
    launches = rec["gpu_launches"]
    ag = allgather_timing(runner, world) if (head_shard and isinstance(
        W.CONFIGS[head_name], W.GemmConfig)) else None
    del runner
    torch.cuda.empty_cache()
    sub_recs = {}
    for name, shard in subs:
        r, run = measure(name, shard, args, world, rank, local, device, cpu_budget=5.0)
        launches += r["gpu_launches"]
        sub_recs[name] = r
        del run
        torch.cuda.empty_cache()

    if rank == 0:
        line = {"metric": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "vs_baseline": None,
                "data": "synthetic (seeded torch CPU generator)", **rec}
        line["gpu_launches"] = launches
        line["gpu_launches_note"] = ("this repository's kernels launched in the timed device "
                                     "regions of the headline and every sub-record")
        if ag is not None:
            line["allgather"] = ag
        if sub_recs:
            line["configs"] = sub_recs
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
