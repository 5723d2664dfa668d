"""Multi-rank host logic of the sharded hot path (N-column GEMM shards, (b, h)
attention shards, all-gather reassembly) on world_size-2 gloo ranks, CPU only.
The compute function is a CPU stand-in; the GPU kernels are tested elsewhere."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sion_b200 import shard


def test_even_split_covers_exactly():
    for n in (1, 7, 256, 1000, 16384):
        for parts in (1, 2, 3, 8):
            for align in (1, 256):
                spans = [shard.even_split(n, parts, i, align) for i in range(parts)]
                assert spans[0][0] == 0 and spans[-1][1] == n
                for (a, b), (c, d) in zip(spans, spans[1:]):
                    assert b == c and a <= b
    with pytest.raises(ValueError):
        shard.even_split(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_gemm_nt(A, B):
    return (A.double() @ B.double().t()).to(torch.float32)


def _cpu_attention(Q, K, V):
    S, D = Q.shape[2], Q.shape[3]
    s = (Q.double() @ K.double().transpose(-1, -2)) / D ** 0.5
    return (torch.softmax(s, -1) @ V.double()).float(), torch.logsumexp(s, -1).float()


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        A = torch.randn(37, 24, generator=g)
        B = torch.randn(1000, 24, generator=g)  # N not a multiple of the 256 tile
        C = shard.sharded_hgemm_nt(A, B, rank, world, gather=True, compute=_cpu_gemm_nt)
        ok_gemm = torch.allclose(C, _cpu_gemm_nt(A, B), atol=1e-5)
        n0, n1, blk = shard.sharded_hgemm_nt(A, B, rank, world, compute=_cpu_gemm_nt)
        ok_block = torch.allclose(blk, _cpu_gemm_nt(A, B)[:, n0:n1], atol=1e-5)
        Q, K, V = [torch.randn(3, 5, 16, 8, generator=g) for _ in range(3)]
        O, L = shard.sharded_attention(Q, K, V, rank, world, gather=True, compute=_cpu_attention)
        Oref, Lref = _cpu_attention(Q, K, V)
        ok_attn = torch.allclose(O, Oref, atol=1e-5) and torch.allclose(L, Lref, atol=1e-5)
        results[rank] = (ok_gemm, ok_block, ok_attn)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_gather_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world,
                       start_method="spawn")
    assert sorted(results.keys()) == list(range(world))
    for r in range(world):
        assert results[r] == (True, True, True), (r, results[r])
