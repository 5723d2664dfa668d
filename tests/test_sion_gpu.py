"""The sion:: LibTorch wrappers as the reference's callers use them
(src/sion/gemm/sgemm/sgemm.cpp:5-32, src/sion/gemm/hgemm/hgemm.cpp:4-83,
src/sion/gemm/gemm.cpp:10-31, src/sion/flash_attention/flash_attn.cpp:7-66),
through both ``sion_b200`` and the drop-in ``sion`` package name
(python/binding.cpp:6), checked against the fp64 CPU oracle.

beta != 0: the wrappers allocate C themselves, so C starts at zero (the
reference reads uninitialised memory there) and the result is alpha*A*B."""
import numpy as np
import pytest
import torch

import oracle
from metrics import assert_fp16_close, compare

pytestmark = pytest.mark.gpu


def _mods():
    import sion
    import sion_b200
    return [sion_b200, sion]


def _f32(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g), torch.randn(K, N, generator=g)


def _f16(M, N, K, seed, nt):
    g = torch.Generator().manual_seed(seed)
    A = (torch.rand(M, K, generator=g) * 2 - 1).half()
    B = (torch.rand(*((N, K) if nt else (K, N)), generator=g) * 2 - 1).half()
    return A, B


@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (0.4, 0.3), (-2.0, 1.0)])
@pytest.mark.parametrize("M,N,K", [(433, 477, 466), (1024, 1024, 1024), (7, 300, 33)])
def test_sgemm(M, N, K, alpha, beta):
    # 433 x 466 x 477, alpha 0.4, beta 0.3: the reference's python/sgemm_test.py case
    A, B = _f32(M, N, K, seed=M + N)
    ref = oracle.sgemm(A.numpy(), B.numpy(), alpha)  # C starts at zero
    for mod in _mods():
        C = mod.sgemm(A.cuda(), B.cuda(), alpha, beta)
        C2 = mod.sgemm(A.cuda(), B.cuda(), alpha=alpha, beta=beta)
        torch.cuda.synchronize()
        m = compare(ref, C.cpu().numpy())
        assert m["nan"] == 0 and m["rel_frob"] <= 1e-5, (mod.__name__, m)
        assert torch.equal(C, C2)


@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (0.5, 0.7)])
@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (200, 136, 72), (512, 1024, 2048)])
def test_hgemm_and_hgemm_nt(M, N, K, alpha, beta):
    for nt in (False, True):
        A, B = _f16(M, N, K, seed=M + K, nt=nt)
        ref = oracle.hgemm(A.numpy(), B.numpy(), nt, alpha)
        for mod in _mods():
            fn = mod.hgemm_nt if nt else mod.hgemm
            C = fn(A.cuda(), B.cuda(), alpha, beta)
            torch.cuda.synchronize()
            assert C.dtype == torch.half and tuple(C.shape) == (M, N)
            assert_fp16_close(ref, C.cpu().numpy().astype(np.float64),
                              ctx=f"{mod.__name__} nt={nt} {M}x{N}x{K}")


def test_gemm_dispatches_on_dtype():
    # sion::gemm: fp32 -> sgemm, fp16 -> hgemm (B stored K x N)
    A, B = _f32(130, 70, 90, seed=3)
    Ah, Bh = _f16(256, 192, 64, seed=4, nt=False)
    for mod in _mods():
        C = mod.gemm(A.cuda(), B.cuda(), 1.5, 0.0)
        Ch = mod.gemm(Ah.cuda(), Bh.cuda(), 1.0, 0.25)
        torch.cuda.synchronize()
        assert C.dtype == torch.float32 and Ch.dtype == torch.half
        assert compare(oracle.sgemm(A.numpy(), B.numpy(), 1.5), C.cpu().numpy())["rel_frob"] <= 1e-5
        assert_fp16_close(oracle.hgemm(Ah.numpy(), Bh.numpy(), False),
                          Ch.cpu().numpy().astype(np.float64), ctx="gemm fp16")
        assert torch.equal(Ch, mod.hgemm(Ah.cuda(), Bh.cuda(), 1.0, 0.25))


def test_gemm_validation_messages():
    # the reference's TORCH_CHECK texts (sgemm.cpp, hgemm.cpp, gemm.cpp)
    import sion
    A = torch.zeros(4, 4, device="cuda")
    with pytest.raises(RuntimeError, match="A must be CUDA tensor"):
        sion.sgemm(A.cpu(), A)
    with pytest.raises(RuntimeError, match="A must be float32"):
        sion.sgemm(A.half(), A)
    with pytest.raises(RuntimeError, match="B.size\\(0\\) must match A.size\\(1\\)"):
        sion.sgemm(A, torch.zeros(5, 4, device="cuda"))
    with pytest.raises(RuntimeError, match="A must be float16"):
        sion.hgemm(A, A.half())
    with pytest.raises(RuntimeError, match="B.size\\(1\\) must match A.size\\(1\\) for NT GEMM"):
        sion.hgemm_nt(A.half(), torch.zeros(4, 8, device="cuda").half())
    with pytest.raises(RuntimeError, match="A and B must have the same dtype"):
        sion.gemm(A, A.half())
    with pytest.raises(RuntimeError, match="Unsupported dtype for gemm"):
        sion.gemm(A.double(), A.double())


def test_gemm_non_contiguous_inputs_sgemm():
    # sion::sgemm makes its inputs contiguous (sgemm.cpp: .contiguous())
    import sion
    A, B = _f32(96, 64, 80, seed=5)
    At = A.t().contiguous().cuda().t()  # a transposed view of the same values
    C = sion.sgemm(At, B.cuda())
    torch.cuda.synchronize()
    assert compare(oracle.sgemm(A.numpy(), B.numpy()), C.cpu().numpy())["rel_frob"] <= 1e-5


@pytest.mark.parametrize("D", [64, 128])
def test_flash_attention_reference_script_case(D):
    # python/flash_attn_test.py: B=8, S=1280, H=8, D=128 (also D=64); oracle on
    # sampled rows of every head
    g = torch.Generator().manual_seed(D)
    Q, K, V = [torch.randn(8, 8, 1280, D, generator=g).half() for _ in range(3)]
    rows = np.r_[0, 63, 64, 640, 1279]
    Oref, Lref = oracle.attention(Q.numpy(), K.numpy(), V.numpy(), rows=rows)
    for mod in _mods():
        O = mod.flash_attention(Q.cuda(), K.cuda(), V.cuda())
        O2, L = mod.flash_attention_lse(Q.cuda(), K.cuda(), V.cuda())
        torch.cuda.synchronize()
        o = O.cpu().numpy()[:, :, rows].astype(np.float64)
        m = compare(Oref, o)
        assert m["max_abs"] <= 1e-2 and m["rel_frob"] <= 1e-3, (mod.__name__, m)
        assert torch.equal(O, O2)
        ml = compare(Lref, L.cpu().numpy()[:, :, rows])
        assert ml["max_rel"] <= 1e-3, ml


def test_flash_attention_validation():
    import sion
    Q = torch.zeros(1, 1, 64, 128, device="cuda").half()
    with pytest.raises(RuntimeError, match="All tensors must be half"):
        sion.flash_attention(Q.float(), Q, Q)
    with pytest.raises(RuntimeError, match="unsupported head dimension"):
        z = torch.zeros(1, 1, 64, 96, device="cuda").half()
        sion.flash_attention(z, z, z)
