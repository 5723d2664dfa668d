"""bench.py's host-side pieces on the CPU: both arms describe a workload with
the same `config` dict (the driver compares them), the CPU host-path sample
measures something, and the suite covers every benchmark configuration."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402
from sion_b200 import workloads as W  # noqa: E402


def test_config_dict_is_shared_by_both_arms():
    for name, shard in [(bench.HEADLINE, True)] + list(bench.SUITE):
        cfg = W.CONFIGS[name]
        l2 = bench.runner_l2(cfg)
        for world in (1, 2, 8):
            a = bench.config_dict(cfg, world, shard, l2)
            b = bench.config_dict(cfg, world, shard, bench.runner_l2(cfg))
            assert a == b
            assert a["workload"] == name
            assert ("shards" in a["parallelism"]) == shard


def test_suite_covers_the_five_configurations():
    names = {bench.HEADLINE} | {n for n, _ in bench.SUITE}
    assert names == {W.SGEMM_1024.name, W.HGEMM_4096.name, W.HGEMM_SKINNY.name, W.FA_8192.name,
                     W.HGEMM_16384.name}
    # the headline and attention split over the ranks (strong scaling)
    assert dict(bench.SUITE)[W.FA_8192.name] is True


def test_cpu_sample_measures_the_host_path():
    gemm = W.GemmConfig("tiny", 64, 96, 80, "f32", "kn", "normal", 1.0, 0)
    v, threads, desc = bench.cpu_sample(gemm, budget_s=0.05)
    assert v > 0 and threads >= 1 and "torch.matmul" in desc
    attn = W.AttnConfig("tiny_attn", 1, 1, 256, 64, 0)
    v, threads, desc = bench.cpu_sample(attn, budget_s=0.05)
    assert v > 0 and "softmax" in desc
