"""Seeded synthetic inputs for the benchmark configurations.

Inputs are drawn on the host with torch's CPU generator (torch.manual_seed(seed),
draws in the order A then B, or Q then K then V, in fp32, then cast to fp16
where the config is fp16), so the CUDA kernels, the CPU oracle and the CPU
baseline all consume identical bits. There is no public dataset for this path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class GemmConfig:
    name: str
    M: int
    N: int
    K: int
    dtype: str       # "f32" or "f16"
    b_layout: str    # "kn" (B stored K x N) or "nk" (B stored N x K)
    dist: str        # "normal" or "uniform"
    std: float
    seed: int

    @property
    def flops(self) -> float:
        return 2.0 * self.M * self.N * self.K

    @property
    def io_bytes(self) -> int:
        es = 4 if self.dtype == "f32" else 2
        return es * (self.M * self.K + self.K * self.N + self.M * self.N)


@dataclass(frozen=True)
class AttnConfig:
    name: str
    B: int
    H: int
    S: int
    D: int
    seed: int
    causal: bool = False
    backward: bool = False

    @property
    def flops(self) -> float:
        # reference convention (bench/flash_attention/fa_bench.cpp:93-95): 4*B*H*S^2*D
        # for the forward (QK^T and PV). The backward does five such products
        # (S recomputed, dP, dV, dK, dQ): 10*B*H*S^2*D. A causal mask halves the
        # work actually required.
        f = (10.0 if self.backward else 4.0) * self.B * self.H * self.S * self.S * self.D
        return f / 2 if self.causal else f

    @property
    def io_bytes(self) -> int:
        t = 2 * self.B * self.H * self.S * self.D
        rows = 4 * self.B * self.H * self.S
        # backward: reads Q, K, V, O, dO, LSE; writes dQ, dK, dV
        return 8 * t + rows if self.backward else 4 * t + rows


# The five configurations of the headline metric.
SGEMM_1024 = GemmConfig("sgemm_f32_1024", 1024, 1024, 1024, "f32", "kn", "normal", 1.0, 0)
HGEMM_4096 = GemmConfig("hgemm_f16_4096_nt", 4096, 4096, 4096, "f16", "nk", "uniform", 1.0, 1)
HGEMM_SKINNY = GemmConfig("hgemm_f16_128x8192x16384_nt", 128, 8192, 16384, "f16", "nk",
                          "normal", 0.02, 2)
FA_8192 = AttnConfig("flash_attn_fwd_f16_4x32x8192x128", 4, 32, 8192, 128, 3)
FA_8192_CAUSAL = AttnConfig("flash_attn_fwd_causal_f16_4x32x8192x128", 4, 32, 8192, 128, 3,
                            causal=True)
FA_BWD_8192 = AttnConfig("flash_attn_bwd_f16_4x32x8192x128", 4, 32, 8192, 128, 3,
                         backward=True)
# a smaller backward case for detailed ncu captures (1/8 of the (b, h, query) rows)
FA_BWD_4096 = AttnConfig("flash_attn_bwd_f16_2x16x4096x128", 2, 16, 4096, 128, 3,
                         backward=True)
# a smaller forward case for detailed ncu captures (1/4 of the (b, h) pairs;
# Q, K, V, O still 4 x 128 MiB, larger than the L2)
FA_FWD_2x16 = AttnConfig("flash_attn_fwd_f16_2x16x8192x128", 2, 16, 8192, 128, 3)
HGEMM_16384 = GemmConfig("hgemm_f16_16384_nt", 16384, 16384, 16384, "f16", "nk", "uniform", 1.0,
                         4)

CONFIGS = {c.name: c for c in (SGEMM_1024, HGEMM_4096, HGEMM_SKINNY, FA_8192, HGEMM_16384,
                               FA_8192_CAUSAL, FA_BWD_8192, FA_BWD_4096, FA_FWD_2x16)}


def _draw(gen: torch.Generator, shape, dist: str, std: float) -> torch.Tensor:
    if dist == "normal":
        return torch.randn(*shape, generator=gen, dtype=torch.float32) * std
    return torch.rand(*shape, generator=gen, dtype=torch.float32) * 2.0 - 1.0


def gemm_inputs(cfg: GemmConfig, M: int | None = None):
    """Host (CPU) tensors A, B for a GEMM config; M overrides the row count
    (row-sampled runs draw the full B and the first M rows of A)."""
    gen = torch.Generator().manual_seed(cfg.seed)
    m = cfg.M if M is None else M
    A = _draw(gen, (cfg.M, cfg.K), cfg.dist, cfg.std)[:m]
    bshape = (cfg.K, cfg.N) if cfg.b_layout == "kn" else (cfg.N, cfg.K)
    B = _draw(gen, bshape, cfg.dist, cfg.std)
    if cfg.dtype == "f16":
        A, B = A.half(), B.half()
    return A.contiguous(), B.contiguous()


def attn_inputs(cfg: AttnConfig):
    gen = torch.Generator().manual_seed(cfg.seed)
    shape = (cfg.B, cfg.H, cfg.S, cfg.D)
    Q = torch.randn(*shape, generator=gen, dtype=torch.float32).half()
    K = torch.randn(*shape, generator=gen, dtype=torch.float32).half()
    V = torch.randn(*shape, generator=gen, dtype=torch.float32).half()
    return Q, K, V


def attn_grad_input(cfg: AttnConfig):
    """dO for a backward config: drawn after Q, K, V from the same seed."""
    gen = torch.Generator().manual_seed(cfg.seed + 1000)
    return torch.randn(cfg.B, cfg.H, cfg.S, cfg.D, generator=gen, dtype=torch.float32).half()
