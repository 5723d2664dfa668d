"""felix_sgemm_noalloc: the SGEMM entry point that allocates nothing.

It is meant for callers that cannot call cudaMalloc inside an operator call
(hosts that own all device memory through their own pool or budget, plugin
runtimes that forbid allocation in the launch path, latency-critical code that
cannot take cudaMalloc's implicit synchronisation). Its split-K scratch is a
static array in the library's device image (16 MiB of partial tiles + 16 KiB
of counters). Results are checked against the fp64 CPU oracle and against the
allocating entry point, on two calls in a row (the calls share the scratch).
This file is collected last so that a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process.
"""
import os
import subprocess
import sys

import pytest
import torch

import oracle
from metrics import compare

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _inputs(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g), torch.randn(K, N, generator=g)


@pytest.mark.parametrize("M,N,K,split_k", [(1024, 1024, 1024, 4), (1024, 1024, 1024, 0),
                                           (300, 500, 2000, 3), (128, 128, 4096, 0),
                                           (2048, 2048, 512, 0)])
def test_noalloc_matches_oracle_and_allocating_entry_point(felix, M, N, K, split_k):
    A, B = _inputs(M, N, K, seed=M + K)
    ref = oracle.sgemm(A.numpy(), B.numpy(), 0.75)
    dA, dB = A.cuda(), B.cuda()
    alloc = torch.empty(M, N, device="cuda")
    felix.sgemm(dA, dB, alloc, 0.75, 0.0, split_k=split_k if split_k else None)
    torch.cuda.synchronize()
    for call in range(2):  # two calls in a row share (and must reset) the scratch
        out = torch.full((M, N), float("nan"), device="cuda")
        felix.sgemm_noalloc(dA, dB, out, 0.75, 0.0, split_k=split_k)
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        m = compare(ref, o)
        assert m["nan"] == 0 and m["rel_frob"] <= 1e-5, (call, m)
        m2 = compare(alloc.cpu().numpy(), o)
        assert m2["rel_frob"] <= 1e-5, (call, m2)


def test_noalloc_beta_accumulates(felix):
    A, B = _inputs(256, 384, 640, seed=1)
    C0 = torch.randn(256, 384)
    ref = oracle.sgemm(A.numpy(), B.numpy(), 1.0, 0.5, C0.numpy())
    for call in range(2):
        out = C0.cuda()
        felix.sgemm_noalloc(A.cuda(), B.cuda(), out, 1.0, 0.5, split_k=2)
        torch.cuda.synchronize()
        assert compare(ref, out.cpu().numpy())["rel_frob"] <= 1e-5, call


def test_noalloc_rejects_split_beyond_static_scratch(felix):
    A, B = _inputs(1024, 1024, 1024, seed=2)
    out = torch.empty(1024, 1024, device="cuda")
    with pytest.raises(felix.FelixError) as e:
        felix.sgemm_noalloc(A.cuda(), B.cuda(), out, split_k=8)  # 64 tiles x 8 > 256
    assert e.value.code == felix.API_ERROR
    assert "static scratch" in str(e.value)
    # the limit applies to the requested split even where K would clamp it:
    # K = 32 has 2 k-blocks, but 64 tiles x 5 requested > 256
    A, B = _inputs(1024, 1024, 32, seed=3)
    with pytest.raises(felix.FelixError):
        felix.sgemm_noalloc(A.cuda(), B.cuda(), out, split_k=5)


_PROBE = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from sion_b200 import abi
torch.cuda.init()
def free_bytes():
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0]
shapes = [(1024, 1024, 1024, 4), (1024, 1024, 1024, 0), (300, 500, 2000, 3),
          (128, 128, 4096, 0), (2048, 2048, 512, 0), (4096, 4096, 256, 0)]
bufs = []
for M, N, K, s in shapes:
    bufs.append((torch.randn(M, K, device="cuda"), torch.randn(K, N, device="cuda"),
                 torch.empty(M, N, device="cuda"), s))
A, B, C, s = bufs[0]
abi.sgemm_noalloc(A, B, C, split_k=s)   # first call: per-device set-up
before = free_bytes()
for _ in range(3):
    for A, B, C, s in bufs:
        abi.sgemm_noalloc(A, B, C, split_k=s)
after = free_bytes()
print("FREE", before, after)
"""


def test_noalloc_allocates_nothing(tmp_path):
    # a fresh process: after the first call (per-device set-up), calls over
    # several shapes and split counts, automatic fallback included, leave the
    # device's free memory unchanged (a library workspace would take some)
    p = tmp_path / "probe.py"
    p.write_text(_PROBE)
    r = subprocess.run([sys.executable, str(p), ROOT], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("FREE")][0]
    _, before, after = line.split()
    assert int(before) == int(after), line
