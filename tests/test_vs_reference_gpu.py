"""Our kernels against the reference's own kernels (built unmodified for sm_100a
into oracle/_ref) on identical seeded inputs, both measured against the fp64
CPU oracle. The reference accumulates HGEMM and attention in fp16, so it is not
bit-comparable; the gate is that our error against the exact result is within
the north-star tolerance and no larger than the reference's own."""
import numpy as np
import pytest
import torch

import oracle
from oracle import reference as ref
from metrics import compare

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built")]


def test_sgemm_vs_reference_kernel(felix):
    g = torch.Generator().manual_seed(0)
    A = torch.randn(1024, 1024, generator=g)
    B = torch.randn(1024, 1024, generator=g)
    ours = torch.empty(1024, 1024, device="cuda")
    theirs = torch.empty(1024, 1024, device="cuda")
    felix.sgemm(A.cuda(), B.cuda(), ours)
    ref.sgemm(A.cuda(), B.cuda(), theirs)
    torch.cuda.synchronize()
    exact = oracle.sgemm(A.numpy(), B.numpy())
    mo, mr = compare(exact, ours.cpu().numpy()), compare(exact, theirs.cpu().numpy())
    print(f"\nsgemm 1024^3 rel_frob ours {mo['rel_frob']:.2e} reference {mr['rel_frob']:.2e}")
    assert mo["rel_frob"] <= 1e-5 and mr["rel_frob"] <= 1e-5
    assert compare(theirs.cpu().numpy(), ours.cpu().numpy())["rel_frob"] <= 1e-5


@pytest.mark.parametrize("nt", [True, False])
def test_hgemm_vs_reference_kernel(felix, nt):
    # reference test shape (tests/hgemm/hgemm_test.cpp:39-72): 2048^3; rows sampled for the oracle
    g = torch.Generator().manual_seed(1)
    M = N = K = 2048
    A = (torch.rand(M, K, generator=g) * 2 - 1).half()
    B = ((torch.rand(N, K, generator=g) if nt else torch.rand(K, N, generator=g)) * 2 - 1).half()
    ours = torch.empty(M, N, dtype=torch.half, device="cuda")
    theirs = torch.empty(M, N, dtype=torch.half, device="cuda")
    felix.hgemm(A.cuda(), B.cuda(), ours, b_layout=felix.B_NK if nt else felix.B_KN)
    ref.hgemm(A.cuda(), B.cuda(), theirs, nt=nt)
    torch.cuda.synchronize()
    rows = np.r_[0:4, 1000, 2044:2048]
    exact = oracle.hgemm(A[rows].numpy(), B.numpy(), nt)
    mo = compare(exact, ours.cpu().numpy()[rows].astype(np.float64))
    mr = compare(exact, theirs.cpu().numpy()[rows].astype(np.float64))
    print(f"\nhgemm 2048^3 nt={nt}: rel_frob ours {mo['rel_frob']:.2e} (max {mo['max_abs']:.3f}) "
          f"reference {mr['rel_frob']:.2e} (max {mr['max_abs']:.3f})")
    assert mo["rel_frob"] <= 1e-3
    assert mo["rel_frob"] <= mr["rel_frob"] and mo["max_abs"] <= mr["max_abs"]


def test_attention_vs_reference_kernel(felix):
    # reference test case (tests/flash_attention/fa_test.cpp:24-42): 16x16x1280x128
    g = torch.Generator().manual_seed(0)
    Q, K, V = [torch.randn(16, 16, 1280, 128, generator=g).half() for _ in range(3)]
    ours = torch.empty_like(Q, device="cuda")
    theirs = torch.empty_like(Q, device="cuda")
    felix.flash_attn_fwd(Q.cuda(), K.cuda(), V.cuda(), ours)
    ref.flash_attn(Q.cuda(), K.cuda(), V.cuda(), theirs)
    torch.cuda.synchronize()
    rows = np.r_[0:4, 640, 1276:1280]
    worst_o, worst_r = 0.0, 0.0
    for (b, h) in [(0, 0), (7, 9), (15, 15)]:
        sl = (slice(b, b + 1), slice(h, h + 1))
        exact, _ = oracle.attention(Q[sl].numpy(), K[sl].numpy(), V[sl].numpy(), rows=rows)
        mo = compare(exact, ours[sl].cpu().numpy()[:, :, rows].astype(np.float64))
        mr = compare(exact, theirs[sl].cpu().numpy()[:, :, rows].astype(np.float64))
        worst_o, worst_r = max(worst_o, mo["max_abs"]), max(worst_r, mr["max_abs"])
    print(f"\nattention 16x16x1280x128 max_abs ours {worst_o:.2e} reference {worst_r:.2e}")
    assert worst_o <= 1e-2 and worst_o <= worst_r
