"""felix_sgemm_noalloc: the SGEMM entry point that allocates nothing.

It is meant for callers that cannot call cudaMalloc inside an operator call
(hosts that own all device memory through their own pool or budget, plugin
runtimes that forbid allocation in the launch path, latency-critical code that
cannot take cudaMalloc's implicit synchronisation). Its split-K scratch is a
static array in the library's device image (16 MiB of partial tiles + 16 KiB
of counters). This file is collected last so that a stop-at-first-failure run
has already run every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

from metrics import compare

pytestmark = pytest.mark.gpu


def _inputs(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g).cuda(), torch.randn(K, N, generator=g).cuda()


@pytest.mark.parametrize("M,N,K,split_k", [(1024, 1024, 1024, 4), (1024, 1024, 1024, 0),
                                           (300, 500, 2000, 3), (128, 128, 4096, 0)])
def test_noalloc_matches_allocating_entry_point(felix, M, N, K, split_k):
    A, B = _inputs(M, N, K, seed=M + K)
    ref = torch.empty(M, N, device="cuda")
    felix.sgemm(A, B, ref, 0.75, 0.0, split_k=split_k if split_k else None)
    torch.cuda.synchronize()
    r = ref.cpu().numpy()
    for call in range(2):  # two calls in a row share (and must reset) the scratch
        out = torch.full((M, N), float("nan"), device="cuda")
        felix.sgemm_noalloc(A, B, out, 0.75, 0.0, split_k=split_k)
        torch.cuda.synchronize()
        m = compare(r, out.cpu().numpy())
        assert m["nan"] == 0 and m["rel_frob"] <= 1e-5, (call, m)


def test_noalloc_beta_accumulates(felix):
    A, B = _inputs(256, 384, 640, seed=1)
    C0 = torch.randn(256, 384, device="cuda")
    ref = C0.clone()
    felix.sgemm(A, B, ref, 1.0, 0.5, split_k=2)
    out = C0.clone()
    felix.sgemm_noalloc(A, B, out, 1.0, 0.5, split_k=2)
    torch.cuda.synchronize()
    assert compare(ref.cpu().numpy(), out.cpu().numpy())["rel_frob"] <= 1e-5


def test_noalloc_rejects_split_beyond_static_scratch(felix):
    A, B = _inputs(1024, 1024, 1024, seed=2)
    out = torch.empty(1024, 1024, device="cuda")
    with pytest.raises(felix.FelixError) as e:
        felix.sgemm_noalloc(A, B, out, split_k=8)  # 64 tiles x 8 = 512 partial tiles > 256
    assert e.value.code == felix.API_ERROR
    assert "static scratch" in str(e.value)
