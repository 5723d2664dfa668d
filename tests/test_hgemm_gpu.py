"""HGEMM (tcgen05) parity through the C ABI against the fp64 CPU oracle.
Gate: rel-Frobenius <= 1e-3 and |err| <= max(1e-2, 1 fp16 ulp(|ref|)) per
element (the output is fp16, whose rounding alone exceeds 1e-2 for |C| > 32)."""
import numpy as np
import pytest
import torch

import oracle
from metrics import assert_fp16_close, compare

pytestmark = pytest.mark.gpu


def _inputs(M, N, K, nt, seed, dist="uniform", std=1.0):
    g = torch.Generator().manual_seed(seed)
    draw = (lambda *s: torch.rand(*s, generator=g) * 2 - 1) if dist == "uniform" else \
        (lambda *s: torch.randn(*s, generator=g) * std)
    A = draw(M, K).half()
    B = draw(N, K).half() if nt else draw(K, N).half()
    C0 = draw(M, N).half()
    return A, B, C0


def _run(felix, M, N, K, nt=True, alpha=1.0, beta=0.0, seed=0, **kw):
    A, B, C0 = _inputs(M, N, K, nt, seed)
    dC = C0.clone().cuda()
    felix.hgemm(A.cuda(), B.cuda(), dC, alpha, beta, b_layout=felix.B_NK if nt else felix.B_KN,
                **kw)
    torch.cuda.synchronize()
    ref = oracle.hgemm(A.numpy(), B.numpy(), nt, alpha, beta, C0.numpy())
    return ref, dC.cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("nt", [True, False])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 256, 128), (512, 1024, 1024),
                                   (128, 128, 64)])
def test_hgemm_aligned(felix, nt, M, N, K):
    ref, out = _run(felix, M, N, K, nt=nt)
    assert_fp16_close(ref, out, ctx=f"{M}x{N}x{K} nt={nt}")


@pytest.mark.parametrize("nt", [True, False])
@pytest.mark.parametrize("M,N,K", [(200, 136, 72), (1, 8, 8), (129, 264, 200), (77, 512, 1032)])
def test_hgemm_ragged(felix, nt, M, N, K):
    ref, out = _run(felix, M, N, K, nt=nt)
    assert_fp16_close(ref, out, ctx=f"{M}x{N}x{K} nt={nt}")


@pytest.mark.parametrize("nt", [True, False])
def test_hgemm_alpha_beta(felix, nt):
    ref, out = _run(felix, 256, 512, 256, nt=nt, alpha=0.5, beta=-0.75)
    assert_fp16_close(ref, out, ctx="alpha/beta")


@pytest.mark.parametrize("block_n", [64, 128, 256])
@pytest.mark.parametrize("nt", [True, False])
def test_hgemm_stream_k_forced(felix, block_n, nt):
    # 5 x 4 tiles on 3 persistent CTAs: 18 whole tiles + 2 stream-K tiles
    M, N, K = 640, 4 * block_n, 1024
    ref, out = _run(felix, M, N, K, nt=nt, block_n=block_n, stream_k=2, max_ctas=3)
    assert_fp16_close(ref, out, ctx="stream-K")
    _, out2 = _run(felix, M, N, K, nt=nt, block_n=block_n, stream_k=2, max_ctas=3)
    np.testing.assert_array_equal(out, out2)  # deterministic fix-up


def test_hgemm_stream_k_all_partial(felix):
    # fewer tiles than CTAs: every tile is split over several CTAs
    ref, out = _run(felix, 256, 512, 4096, nt=True, block_n=256, stream_k=2, max_ctas=7)
    assert_fp16_close(ref, out, ctx="stream-K all partial")


def test_hgemm_skinny_config_sampled(felix):
    # config 3 shape: M=128, N=8192, K=16384, N(0, 0.02), exercises stream-K by default
    from sion_b200.workloads import HGEMM_SKINNY, gemm_inputs
    A, B = gemm_inputs(HGEMM_SKINNY)
    C = torch.empty(128, 8192, dtype=torch.half, device="cuda")
    felix.hgemm(A.cuda(), B.cuda(), C, b_layout=felix.B_NK)
    torch.cuda.synchronize()
    cols = np.arange(0, 8192, 37)
    ref = oracle.hgemm(A.numpy(), B[cols].numpy(), True)
    out = C.cpu().numpy()[:, cols].astype(np.float64)
    assert_fp16_close(ref, out, ctx="skinny sampled")


@pytest.mark.parametrize("nt", [True, False])
@pytest.mark.parametrize("M,N,K", [(128, 8192, 8192), (200, 4096, 4096)])
def test_hgemm_cluster_split_k(felix, nt, M, N, K):
    # few 128 x 128 tiles and a long K: each tile's K is split over a 2-CTA
    # cluster that reduces through DSMEM (the automatic plan); sampled columns
    # against the oracle, and bit-identical on a second call
    g = torch.Generator().manual_seed(M + N + K)
    A = ((torch.rand(M, K, generator=g) * 2 - 1) * 0.05).half()
    B = ((torch.rand(N, K, generator=g) * 2 - 1) * 0.05).half()
    Bd = B.cuda() if nt else B.t().contiguous().cuda()
    lay = felix.B_NK if nt else felix.B_KN
    C = torch.empty(M, N, dtype=torch.half, device="cuda")
    felix.hgemm(A.cuda(), Bd, C, b_layout=lay)
    torch.cuda.synchronize()
    out = C.cpu().numpy()
    cols = np.r_[0:40, N // 2 - 7:N // 2 + 9, N - 40:N]
    ref = oracle.hgemm(A.numpy(), B[cols].numpy(), True)
    assert_fp16_close(ref, out[:, cols].astype(np.float64), ctx="cluster split-K")
    felix.hgemm(A.cuda(), Bd, C, b_layout=lay)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out, C.cpu().numpy())


def _tile_samples(n, tile, salt):
    """One index in every `tile`-wide block of [0, n), at an offset that moves
    from block to block (so both 128-row halves of a CTA-pair tile are hit)."""
    return np.array([min(n - 1, t * tile + (t * salt + 3) % tile) for t in range(-(-n // tile))])


def _full_size_check(felix, cfg, row_tile, col_tile):
    """A full-size benchmark GEMM config through the C ABI (the automatic plan:
    CTA pairs, stream-K tail), checked three ways: sampled rows and sampled
    columns against the fp64 oracle (one of each in every output tile, so every
    stream-K / fix-up tile and both halves of every CTA pair are hit), and the
    whole output against cuBLAS with fp32 accumulation (torch.matmul) within
    max(1e-2, 2 fp16 ulp) per element."""
    from sion_b200.workloads import gemm_inputs
    A, B = gemm_inputs(cfg)
    dA, dB = A.cuda(), B.cuda()
    C = torch.empty(cfg.M, cfg.N, dtype=torch.half, device="cuda")
    felix.hgemm(dA, dB, C, b_layout=felix.B_NK)
    torch.cuda.synchronize()
    rows = _tile_samples(cfg.M, row_tile, 53)
    cols = _tile_samples(cfg.N, col_tile, 97)
    ref_r = oracle.hgemm(A[rows].numpy(), B.numpy(), True)
    assert_fp16_close(ref_r, C[torch.from_numpy(rows).cuda()].cpu().numpy().astype(np.float64),
                      ctx=f"{cfg.name} sampled rows")
    ref_c = oracle.hgemm(A.numpy(), B[cols].numpy(), True)
    out_c = C[:, torch.from_numpy(cols).cuda()].cpu().numpy().astype(np.float64)
    assert_fp16_close(ref_c, out_c, ctx=f"{cfg.name} sampled columns")
    prev = torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    try:
        R = torch.matmul(dA, dB.t())
    finally:
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = prev
    del dA, dB
    bad = 0
    for r0 in range(0, cfg.M, 2048):  # chunks keep the fp32 temporaries small
        r = R[r0:r0 + 2048].float()
        d = (C[r0:r0 + 2048].float() - r).abs()
        ulp = torch.exp2(torch.floor(torch.log2(r.abs().clamp(min=2.0 ** -14))) - 10)
        tol = torch.clamp(2.0 * ulp, min=1e-2)
        bad += int((d > tol).sum())
    assert bad == 0, f"{cfg.name}: {bad} elements differ from cuBLAS by more than 2 ulp"
    # a second call gives identical bits (deterministic stream-K fix-up)
    C2 = torch.empty_like(C)
    felix.hgemm(A.cuda(), B.cuda(), C2, b_layout=felix.B_NK)
    torch.cuda.synchronize()
    assert torch.equal(C, C2)


def test_hgemm_config2_full_size(felix):
    # benchmark config 2: 4096^3 nt, U(-1, 1), seed 1; every 128 x 128 tile sampled
    from sion_b200.workloads import HGEMM_4096
    _full_size_check(felix, HGEMM_4096, 128, 128)


def test_hgemm_config5_full_size(felix):
    # benchmark config 5: 16384^3 nt, U(-1, 1), seed 4; one row in every
    # 256-row pair tile and one column in every 256-column tile
    from sion_b200.workloads import HGEMM_16384
    _full_size_check(felix, HGEMM_16384, 256, 256)


def test_hgemm_k_zero(felix):
    C0 = torch.randn(64, 64).half().cuda()
    out = C0.clone()
    A = torch.empty(64, 0, dtype=torch.half, device="cuda")
    B = torch.empty(64, 0, dtype=torch.half, device="cuda")
    felix.hgemm(A, B, out, 1.0, 2.0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), (2 * C0.float()).half().cpu().numpy())


def test_hgemm_rejects_unaligned_k(felix):
    A = torch.zeros(128, 65, dtype=torch.half, device="cuda")
    B = torch.zeros(128, 65, dtype=torch.half, device="cuda")
    C = torch.zeros(128, 128, dtype=torch.half, device="cuda")
    with pytest.raises(felix.FelixError) as e:
        felix.hgemm(A, B, C)
    assert e.value.code == felix.API_ERROR


@pytest.mark.parametrize("nt", [True, False])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (512, 768, 1024), (300, 576, 192),
                                   (1024, 1024, 2048), (130, 320, 320)])
def test_hgemm_cta_pair(felix, nt, M, N, K):
    # 256 x 256 tiles on 2-CTA clusters (cta_group::2 MMAs issued by the leader),
    # stages of two 64-deep k-blocks (odd counts end in a zero-filled block)
    ref, out = _run(felix, M, N, K, nt=nt, cta_pair=2)
    assert_fp16_close(ref, out, ctx="CTA pair")


def test_hgemm_cta_pair_rejects_ragged_k(felix):
    A = torch.zeros(256, 200, dtype=torch.half, device="cuda")
    B = torch.zeros(256, 200, dtype=torch.half, device="cuda")
    C = torch.empty(256, 256, dtype=torch.half, device="cuda")
    with pytest.raises(felix.FelixError):
        felix.hgemm(A, B, C, b_layout=felix.B_NK, cta_pair=2)


@pytest.mark.parametrize("nt", [True, False])
def test_hgemm_cta_pair_stream_k(felix, nt):
    # incomplete last wave of pair tiles spread by k-iterations over few pairs,
    # deterministic fix-up
    M, N, K = 768, 1280, 2048
    ref, out = _run(felix, M, N, K, nt=nt, cta_pair=2, stream_k=2, max_ctas=6)
    assert_fp16_close(ref, out, ctx="CTA pair stream-K")
    _, out2 = _run(felix, M, N, K, nt=nt, cta_pair=2, stream_k=2, max_ctas=6)
    np.testing.assert_array_equal(out, out2)


def test_hgemm_cta_pair_alpha_beta(felix):
    ref, out = _run(felix, 384, 512, 256, nt=True, alpha=0.5, beta=-0.75, cta_pair=2)
    assert_fp16_close(ref, out, ctx="CTA pair alpha/beta")


@pytest.mark.parametrize("M,N,K", [(4096, 10240, 512), (4000, 10000, 1024)])
def test_hgemm_wide_pair_tiles(felix, M, N, K):
    # four or more waves of 256 x 512 "nt" pair tiles: two N = 256 MMAs per k
    # step into one TMEM accumulator, tiles handed out at run time; ragged M
    # and N clip at the tensor-map edges
    from sion_b200.workloads import GemmConfig
    cfg = GemmConfig(f"wide_{M}x{N}x{K}", M, N, K, "f16", "nk", "uniform", 1.0, M + N)
    _full_size_check(felix, cfg, 256, 512)


@pytest.mark.parametrize("M,N,K,nt,cta_pair", [(4608, 4608, 256, False, None),
                                               (5120, 5120, 128, True, 1)])
def test_hgemm_dynamic_tiles(felix, M, N, K, nt, cta_pair):
    # four or more waves of whole tiles: tile ids handed out at run time by a
    # global counter (CTA pairs with B stored K x N; single CTAs with pairs
    # turned off). Sampled rows/columns against the fp64 oracle, the whole
    # output against cuBLAS, bit-identical on a second call (the counter must
    # be back at zero, and the tile-to-CTA assignment must not matter).
    from metrics import fp16_ulp
    g = torch.Generator().manual_seed(M + K)
    A = (torch.rand(M, K, generator=g) * 2 - 1).half()
    B = (torch.rand(*((N, K) if nt else (K, N)), generator=g) * 2 - 1).half()
    dA, dB = A.cuda(), B.cuda()
    lay = felix.B_NK if nt else felix.B_KN
    outs = []
    for _ in range(2):
        C = torch.empty(M, N, dtype=torch.half, device="cuda")
        felix.hgemm(dA, dB, C, b_layout=lay, cta_pair=cta_pair)
        torch.cuda.synchronize()
        outs.append(C)
    assert torch.equal(outs[0], outs[1])
    C = outs[0]
    rows = _tile_samples(M, 256, 29)
    Bnk = B if nt else B.t().contiguous()
    ref = oracle.hgemm(A[rows].numpy(), Bnk.numpy(), True)
    assert_fp16_close(ref, C[torch.from_numpy(rows).cuda()].cpu().numpy().astype(np.float64),
                      ctx="dynamic tiles rows")
    R = torch.matmul(dA.float(), (dB.float().t() if nt else dB.float()))
    tol = torch.from_numpy(np.maximum(1e-2, 2 * fp16_ulp(R.cpu().numpy()))).cuda()
    assert int(((C.float() - R).abs() > tol).sum()) == 0
