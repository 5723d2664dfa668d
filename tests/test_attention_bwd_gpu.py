"""Flash-attention backward (tcgen05) through the C ABI against the fp64 oracle.
The forward output O and LSE come from our forward kernel, as in training.
Gate: relative Frobenius error of dQ, dK, dV <= 1e-2, and no worse than 2x the
error of torch's own fp16 SDPA backward on the same inputs (measured in the
same test), i.e. at the precision fp16 attention gradients have."""
import numpy as np
import pytest
import torch

import oracle
from metrics import compare

pytestmark = pytest.mark.gpu


def _inputs(B, H, S, D, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, S, D, generator=g).half() for _ in range(4)]


def _torch_fp16_grads(Q, K, V, dO, causal):
    q, k, v = [t.cuda().requires_grad_(True) for t in (Q, K, V)]
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal)
    o.backward(dO.cuda())
    return [t.grad.float().cpu().numpy().astype(np.float64) for t in (q, k, v)]


def _run(felix, B, H, S, D, seed=0, causal=False):
    Q, K, V, dO = _inputs(B, H, S, D, seed)
    dQ_, dK_, dV_ = [torch.empty(B, H, S, D, dtype=torch.half, device="cuda") for _ in range(3)]
    O = torch.empty(B, H, S, D, dtype=torch.half, device="cuda")
    L = torch.empty(B, H, S, device="cuda")
    q, k, v, g = [t.cuda() for t in (Q, K, V, dO)]
    felix.flash_attn_fwd(q, k, v, O, L, causal=causal)
    felix.flash_attn_bwd(q, k, v, O, g, L, dQ_, dK_, dV_, causal=causal)
    torch.cuda.synchronize()
    exact = oracle.attention_bwd(Q.numpy(), K.numpy(), V.numpy(), dO.numpy(), causal=causal)
    ours = [t.cpu().numpy().astype(np.float64) for t in (dQ_, dK_, dV_)]
    theirs = _torch_fp16_grads(Q, K, V, dO, causal)
    for name, e, o, t in zip(("dQ", "dK", "dV"), exact, ours, theirs):
        mo, mt = compare(e, o), compare(e, t)
        assert mo["nan"] == 0 and mo["inf"] == 0, (name, mo)
        if np.linalg.norm(e) < 1e-6:  # e.g. dQ with one key: exactly zero gradient
            assert mo["max_abs"] <= 1e-3, (name, mo)
            continue
        assert mo["rel_frob"] <= 1e-2, (name, S, D, causal, mo, mt["rel_frob"])
        assert mo["rel_frob"] <= 2 * mt["rel_frob"] + 1e-4, (name, S, D, causal, mo, mt)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("S", [128, 256, 384])
def test_attention_bwd_aligned(felix, S, D, causal):
    _run(felix, 1, 2, S, D, seed=S + D, causal=causal)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S", [1, 77, 200, 333])
def test_attention_bwd_ragged(felix, S, causal):
    _run(felix, 2, 1, S, 128, seed=S, causal=causal)


def test_attention_bwd_deterministic_shapes(felix):
    # dK, dV are written once per key block: bit-identical across runs
    Q, K, V, dO = [t.cuda() for t in _inputs(1, 2, 512, 128, 7)]
    O = torch.empty_like(Q)
    L = torch.empty(1, 2, 512, device="cuda")
    felix.flash_attn_fwd(Q, K, V, O, L)
    outs = []
    for _ in range(2):
        g = [torch.empty_like(Q) for _ in range(3)]
        felix.flash_attn_bwd(Q, K, V, O, dO, L, *g)
        outs.append(g)
    torch.cuda.synchronize()
    assert torch.equal(outs[0][1], outs[1][1]) and torch.equal(outs[0][2], outs[1][2])


@pytest.mark.parametrize("causal", [False, True])
def test_attention_autograd_through_sion(causal):
    """torch.autograd through sion_b200.flash_attention_autograd (sion:: ->
    felix:: -> C ABI) gives the oracle's gradients."""
    import sion_b200
    B, H, S, D = 1, 2, 200, 128
    Q, K, V, dO = _inputs(B, H, S, D, seed=7)
    q, k, v = [t.cuda().requires_grad_(True) for t in (Q, K, V)]
    o = sion_b200.flash_attention_autograd(q, k, v, causal)
    o.backward(dO.cuda())
    exact = oracle.attention_bwd(Q.numpy(), K.numpy(), V.numpy(), dO.numpy(), causal=causal)
    for name, e, t in zip(("dQ", "dK", "dV"), exact, (q.grad, k.grad, v.grad)):
        m = compare(e, t.float().cpu().numpy().astype(np.float64))
        assert m["rel_frob"] <= 1e-2, (name, m)


def test_attention_backward_rejects_bad_lse():
    import sion_b200
    q = torch.zeros(1, 1, 64, 64, dtype=torch.half, device="cuda")
    with pytest.raises(RuntimeError):
        sion_b200.flash_attention_backward(q, q, q, q, torch.zeros(1, 1, 32, device="cuda"), q)
