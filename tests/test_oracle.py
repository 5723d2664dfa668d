"""The CPU oracle pinned against the golden fixtures (torch addmm / SDPA in fp64,
the comparison functions of the reference's own tests)."""
import glob
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


@pytest.mark.parametrize("name", ["sgemm_67x45x33", "sgemm_128x128x128"])
def test_sgemm_oracle_matches_golden(name):
    g = _load(name)
    out = oracle.sgemm(g["A"], g["B"], float(g["alpha"]), float(g["beta"]), g["C0"])
    np.testing.assert_allclose(out, g["ref"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", ["hgemm_nt_128x256x64", "hgemm_nn_200x136x72"])
def test_hgemm_oracle_matches_golden(name):
    g = _load(name)
    out = oracle.hgemm(g["A"], g["B"], bool(g["nt"]), float(g["alpha"]), float(g["beta"]),
                       g["C0"])
    np.testing.assert_allclose(out, g["ref"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", ["attn_1x2x80x64", "attn_1x1x130x128"])
def test_attention_oracle_matches_golden(name):
    g = _load(name)
    O, L = oracle.attention(g["Q"], g["K"], g["V"])
    np.testing.assert_allclose(O, g["O"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(L, g["lse"], rtol=1e-12, atol=1e-12)


def test_attention_causal_oracle_matches_golden():
    g = _load("attn_causal_1x2x150x64")
    O, L = oracle.attention(g["Q"], g["K"], g["V"], causal=True)
    np.testing.assert_allclose(O, g["O"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(L, g["lse"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", ["attn_bwd_1x2x70x64", "attn_bwd_causal_1x1x90x128"])
def test_attention_bwd_oracle_matches_golden(name):
    g = _load(name)
    dQ, dK, dV = oracle.attention_bwd(g["Q"], g["K"], g["V"], g["dO"], causal=bool(g["causal"]))
    for got, want in ((dQ, g["dQ"]), (dK, g["dK"]), (dV, g["dV"])):
        np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-11)


def test_attention_oracle_row_subset():
    g = _load("attn_1x1x130x128")
    rows = np.array([0, 5, 129], np.int64)
    O, L = oracle.attention(g["Q"], g["K"], g["V"], rows=rows)
    np.testing.assert_allclose(O, g["O"][:, :, rows], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(L, g["lse"][:, :, rows], rtol=1e-12)


def test_half_conversions_exhaustive():
    bits = np.arange(65536, dtype=np.uint16)
    f = bits.view(np.float16)
    d = oracle.half_to_double(bits)
    finite = np.isfinite(f)
    np.testing.assert_array_equal(d[finite], f[finite].astype(np.float64))
    assert np.isnan(d[np.isnan(f)]).all()
    # round trip, and rounding of midpoints / random doubles agrees with numpy
    back = oracle.double_to_half(d[finite])
    np.testing.assert_array_equal(back, bits[finite])
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000) * 10.0 ** rng.integers(-8, 5, 200000),
                        (d[finite][:-1] + d[finite][1:]) / 2])
    x = x[np.abs(x) < 65504]
    np.testing.assert_array_equal(oracle.double_to_half(x), x.astype(np.float16).view(np.uint16))


def test_golden_fixtures_present():
    assert len(glob.glob(os.path.join(GOLD, "*.npz"))) == 9


def test_topk_oracle_matches_numpy_ordering():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 101)).astype(np.float32)
    x[0, :10] = np.float32(0.5)           # duplicates
    x[1, 3] = -0.0
    x[1, 4] = 0.0
    x[2, 7] = np.inf
    x[2, 8] = -np.inf
    for k in (1, 2, 50, 101):
        for largest in (True, False):
            got = oracle.topk(x, k, largest)
            srt = np.sort(x, axis=1)  # numpy sorts -0.0 == 0.0: compare values
            want = srt[:, -k] if largest else srt[:, k - 1]
            np.testing.assert_array_equal(got, want)
    # NaN is the largest key
    y = np.array([[1.0, np.nan, 3.0]], np.float32)
    assert np.isnan(oracle.topk(y, 1, True)[0]) and oracle.topk(y, 2, True)[0] == 3.0
    # -0.0 orders below +0.0 (bit-exact result)
    z = np.array([[0.0, -0.0]], np.float32)
    assert oracle.topk(z, 1, False).view(np.uint32)[0] == np.float32(-0.0).view(np.uint32)
