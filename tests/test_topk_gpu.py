"""k-th value per slice (felix_topk_select, the reference's sorting_radix_select)
through the C ABI against the CPU oracle: bit-exact."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


# Paths: <= 2048 values one warp per slice (keys in registers); aligned
# slices (n % 4 == 0) below 8K values staged in shared memory by bulk copies,
# from 8K values on read from HBM and again through the L2 (three passes,
# candidate lists); other slices up to 48K values staged by loads, larger
# ones read from global memory every pass; few slices of >= 1M values the
# grid-wide passes.


def _check(felix, x, k, largest):
    out = torch.empty(x.shape[0], device="cuda")
    felix.topk_select(torch.from_numpy(x).cuda(), out, k, largest)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32),
                                  oracle.topk(x, k, largest).view(np.uint32))


@pytest.mark.parametrize("largest", [True, False])
@pytest.mark.parametrize("ns,n,k", [(1, 1, 1), (7, 100, 1), (7, 100, 100), (300, 1000, 17),
                                    (33, 2048, 2048), (17, 2049, 1000), (19, 2052, 1),
                                    (40, 3001, 1500), (9, 32768, 16384), (5, 4096, 7),
                                    (6, 8188, 4000), (6, 8192, 1),
                                    (64, 49152, 1000), (3, 49153, 5), (2, 200000, 77777),
                                    (2, 200003, 100000)])
def test_topk_random(felix, ns, n, k, largest):
    rng = np.random.default_rng(ns * 7 + n)
    _check(felix, rng.standard_normal((ns, n)).astype(np.float32), k, largest)


@pytest.mark.parametrize("largest", [True, False])
@pytest.mark.parametrize("n", [5000, 12000])
def test_topk_special_values(felix, n, largest):
    # 5000: staged path; 12000: unstaged, whose raw-bit digit test must defer
    # to the converted keys where NaN bit patterns share the top digit
    rng = np.random.default_rng(5)
    x = rng.integers(-3, 4, size=(16, n)).astype(np.float32)  # heavy duplicates
    x[0, :100] = np.nan
    x[1, :50] = -0.0
    x[2, :50] = np.inf
    x[3, :50] = -np.inf
    x[4, :] = 0.0
    x[5, ::2] = -0.0
    x[6, :] = rng.standard_normal(n).astype(np.float32)
    x[6, ::3] = np.nan
    x[7, :] = -rng.random(n).astype(np.float32)
    x[7, :40] = -np.inf
    x[7, 40:60] = np.nan
    for k in (1, 2, 50, 101, 2500, n):
        _check(felix, x, k, largest)


@pytest.mark.parametrize("largest", [True, False])
def test_topk_few_huge_slices_grid_wide(felix, largest):
    # few slices of >= 1M values take the grid-wide path
    rng = np.random.default_rng(9)
    x = rng.standard_normal((2, 3_000_001)).astype(np.float32)
    x[1, :1000] = 7.0
    for k in (1, 1000, 1500000):
        _check(felix, x, k, largest)


def test_topk_argument_errors(felix):
    x = torch.zeros(2, 10, device="cuda")
    out = torch.empty(2, device="cuda")
    for k in (0, 11):
        with pytest.raises(felix.FelixError) as e:
            felix.topk_select(x, out, k)
        assert e.value.code == felix.API_ERROR


@pytest.mark.parametrize("largest", [True, False])
@pytest.mark.parametrize("n", [4096, 32768])
def test_topk_candidate_overflow_in_one_warp(felix, n, largest):
    # Aligned slices (staged below 8K values, re-read through the L2 from 8K
    # on) collect the keys whose top digit matches into one candidate region
    # per warp; here every such key sits in the 16-byte groups that warp 0
    # reads (group g goes to warp (g % 512) // 32), so that region overflows
    # while the slice as a whole has few candidates, and the last pass must
    # fall back to reading every key again.
    rng = np.random.default_rng(11)
    x = np.where(rng.random((3, n)) < 0.5, -100.0, 100.0).astype(np.float32)
    groups = np.arange(n) // 4
    warp0 = (groups % 512) // 32 == 0
    x[:, warp0] = (1.0 + rng.random((3, int(warp0.sum()))) * 0.5).astype(np.float32)
    m = int(warp0.sum())
    big = int((x[0] > 50).sum())
    for k in (big + 1, big + m // 2, big + m):
        _check(felix, x[:1], k, True)
    small = int((x[1] < -50).sum())
    _check(felix, x[1:2], small + 7, False)
    _check(felix, x, n // 2, largest)
