"""Independent sharding of the hot path across the GPUs of one node.

Every unit of work is independent, so there is no data-path collective:
  * GEMM: N is cut into contiguous column blocks, one per rank. With B stored
    N x K ("nt") a column block of C needs a contiguous row range of B; A is
    replicated. Rank r computes C[:, n0:n1].
  * Attention: the B*H (batch, head) pairs are cut into contiguous groups; a
    group is a contiguous slice of Q, K, V, O and LSE.
An optional all-gather (NCCL over NVLink on GPUs, gloo in the CPU tests)
reassembles the full C / O on every rank; it is the only collective and it is
outside the compute.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def even_split(n: int, parts: int, index: int, align: int = 1) -> tuple[int, int]:
    """[start, end) of part `index` when n units (in multiples of `align`) are cut
    into `parts` contiguous, near-equal blocks."""
    if parts <= 0 or not 0 <= index < parts:
        raise ValueError("bad shard index")
    units = (n + align - 1) // align
    s = units * index // parts
    e = units * (index + 1) // parts
    return min(n, s * align), min(n, e * align)


def gemm_column_shard(N: int, world: int, rank: int, align: int = 256) -> tuple[int, int]:
    """Column block of C owned by `rank` (aligned to the 256-wide HGEMM tile)."""
    return even_split(N, world, rank, align)


def attention_shard(batch: int, heads: int, world: int, rank: int) -> tuple[int, int]:
    """Range of flattened (b, h) indices owned by `rank`."""
    return even_split(batch * heads, world, rank)


def _default_hgemm_nt(A: torch.Tensor, B_nk: torch.Tensor) -> torch.Tensor:
    from . import abi
    C = torch.empty(A.shape[0], B_nk.shape[0], dtype=torch.half, device=A.device)
    abi.hgemm(A, B_nk, C, b_layout=abi.B_NK)
    return C


def sharded_hgemm_nt(A: torch.Tensor, B_nk: torch.Tensor, rank: int, world: int,
                     gather: bool = False, group=None,
                     compute: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] | None = None):
    """C = A @ B^T with B stored [N, K]. Each rank computes its column block; with
    gather=True every rank returns the full C (all-gather of equal-width padded
    blocks, then trimmed), else its (n0, n1, block)."""
    compute = compute or _default_hgemm_nt
    N = B_nk.shape[0]
    n0, n1 = gemm_column_shard(N, world, rank)
    block = compute(A, B_nk[n0:n1].contiguous()) if n1 > n0 else \
        torch.empty(A.shape[0], 0, dtype=A.dtype, device=A.device)
    if not gather:
        return n0, n1, block
    width = max(gemm_column_shard(N, world, r)[1] - gemm_column_shard(N, world, r)[0]
                for r in range(world))
    padded = torch.zeros(A.shape[0], width, dtype=block.dtype, device=block.device)
    padded[:, : n1 - n0] = block
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    cols = []
    for r in range(world):
        a, b = gemm_column_shard(N, world, r)
        cols.append(parts[r][:, : b - a])
    return torch.cat(cols, dim=1)


def _default_attention(Q, K, V):
    from . import abi
    O = torch.empty_like(Q)
    L = torch.empty(Q.shape[:3], dtype=torch.float32, device=Q.device)
    abi.flash_attn_fwd(Q, K, V, O, L)
    return O, L


def sharded_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, rank: int, world: int,
                      gather: bool = False, group=None, compute=None):
    """Flash attention over this rank's (b, h) group; with gather=True every rank
    returns the full (O, LSE), else (s, e, O_part, LSE_part) over flattened b*h."""
    compute = compute or _default_attention
    Bn, H, S, D = Q.shape
    s, e = attention_shard(Bn, H, world, rank)
    q = Q.reshape(Bn * H, 1, S, D)[s:e].reshape(1, e - s, S, D).contiguous()
    k = K.reshape(Bn * H, 1, S, D)[s:e].reshape(1, e - s, S, D).contiguous()
    v = V.reshape(Bn * H, 1, S, D)[s:e].reshape(1, e - s, S, D).contiguous()
    if e > s:
        O, L = compute(q, k, v)
    else:
        O = torch.empty(1, 0, S, D, dtype=Q.dtype, device=Q.device)
        L = torch.empty(1, 0, S, dtype=torch.float32, device=Q.device)
    if not gather:
        return s, e, O, L
    width = max(attention_shard(Bn, H, world, r)[1] - attention_shard(Bn, H, world, r)[0]
                for r in range(world))
    po = torch.zeros(width, S, D, dtype=O.dtype, device=O.device)
    pl = torch.zeros(width, S, dtype=L.dtype, device=L.device)
    po[: e - s] = O.reshape(e - s, S, D)
    pl[: e - s] = L.reshape(e - s, S)
    partsO = [torch.empty_like(po) for _ in range(world)]
    partsL = [torch.empty_like(pl) for _ in range(world)]
    dist.all_gather(partsO, po, group=group)
    dist.all_gather(partsL, pl, group=group)
    outO, outL = [], []
    for r in range(world):
        a, b = attention_shard(Bn, H, world, r)
        outO.append(partsO[r][: b - a])
        outL.append(partsL[r][: b - a])
    return torch.cat(outO).reshape(Bn, H, S, D), torch.cat(outL).reshape(Bn, H, S)
