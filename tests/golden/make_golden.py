"""Generate the golden fixtures in tests/golden/*.npz.

The reference's own tests take their expected values from torch
(`torch::addmm` for SGEMM/HGEMM, tests/sgemm/sgemm_test.cpp:15-18 and
tests/hgemm/hgemm_test.cpp:3-21; `at::scaled_dot_product_attention` for
attention, tests/flash_attention/fa_test.cpp:8-15). This script evaluates those
same torch functions on the CPU in float64 over small seeded inputs, so the C
oracle can be pinned against them without a GPU. LSE is pinned with
torch.logsumexp over the float64 scores.

Run from the repo root: python tests/golden/make_golden.py
"""
from __future__ import annotations

import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def sgemm_case(name, M, N, K, alpha, beta, seed):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g)
    B = torch.randn(K, N, generator=g)
    C0 = torch.randn(M, N, generator=g)
    ref = torch.addmm(C0.double(), A.double(), B.double(), beta=beta, alpha=alpha)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), A=A.numpy(), B=B.numpy(),
                        C0=C0.numpy(), alpha=alpha, beta=beta, ref=ref.numpy())


def hgemm_case(name, M, N, K, nt, alpha, beta, seed):
    g = torch.Generator().manual_seed(seed)
    A = (torch.rand(M, K, generator=g) * 2 - 1).half()
    B = (torch.rand(N, K, generator=g) * 2 - 1).half() if nt else \
        (torch.rand(K, N, generator=g) * 2 - 1).half()
    C0 = (torch.rand(M, N, generator=g) * 2 - 1).half()
    Bk = B.double().t() if nt else B.double()
    ref = torch.addmm(C0.double(), A.double(), Bk, beta=beta, alpha=alpha)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), A=A.numpy(), B=B.numpy(),
                        C0=C0.numpy(), nt=nt, alpha=alpha, beta=beta, ref=ref.numpy())


def attn_case(name, Bn, H, S, D, seed, causal=False):
    g = torch.Generator().manual_seed(seed)
    Q = torch.randn(Bn, H, S, D, generator=g).half()
    K = torch.randn(Bn, H, S, D, generator=g).half()
    V = torch.randn(Bn, H, S, D, generator=g).half()
    q, k, v = Q.double(), K.double(), V.double()
    O = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=None, dropout_p=0.0,
                                                         is_causal=causal)
    scores = (q @ k.transpose(-1, -2)) / (D ** 0.5)
    if causal:
        scores = scores.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
    lse = torch.logsumexp(scores, dim=-1)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), Q=Q.numpy(), K=K.numpy(),
                        V=V.numpy(), O=O.numpy(), lse=lse.numpy())


def attn_bwd_case(name, Bn, H, S, D, seed, causal):
    # gradients of SDPA by torch autograd in float64
    g = torch.Generator().manual_seed(seed)
    Q, K, V, dO = [torch.randn(Bn, H, S, D, generator=g).half() for _ in range(4)]
    q, k, v = [t.double().requires_grad_(True) for t in (Q, K, V)]
    O = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal)
    O.backward(dO.double())
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), Q=Q.numpy(), K=K.numpy(),
                        V=V.numpy(), dO=dO.numpy(), dQ=q.grad.numpy(), dK=k.grad.numpy(),
                        dV=v.grad.numpy(), causal=causal)


def main():
    sgemm_case("sgemm_67x45x33", 67, 45, 33, 0.7, 0.3, 10)
    sgemm_case("sgemm_128x128x128", 128, 128, 128, 1.0, 0.0, 11)
    hgemm_case("hgemm_nt_128x256x64", 128, 256, 64, True, 1.0, 0.0, 12)
    hgemm_case("hgemm_nn_200x136x72", 200, 136, 72, False, 0.5, 0.25, 13)
    attn_case("attn_1x2x80x64", 1, 2, 80, 64, 14)
    attn_case("attn_1x1x130x128", 1, 1, 130, 128, 15)
    attn_case("attn_causal_1x2x150x64", 1, 2, 150, 64, 16, causal=True)
    attn_bwd_case("attn_bwd_1x2x70x64", 1, 2, 70, 64, 17, causal=False)
    attn_bwd_case("attn_bwd_causal_1x1x90x128", 1, 1, 90, 128, 18, causal=True)


if __name__ == "__main__":
    main()
