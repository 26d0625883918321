"""KV-head sharding across GPUs (one process per GPU).

Rank r of N owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and, through the GQA
mapping q-head h -> kv-head h // (Hq/Hkv), the contiguous q-heads
[r*Hq/N, (r+1)*Hq/N).  Each rank keeps its own page pools for its heads
(same block tables on every rank), appends and decodes locally with no
communication, then the attention outputs [B][Hq/N][D] of all ranks are
all-gathered (NCCL over NVLink on GPUs) into [N][B][Hq/N][D] and viewed as
[B][Hq][D].
"""
from __future__ import annotations


def head_ranges(num_kv_heads: int, num_q_heads: int, world: int, rank: int):
    """((kv_lo, kv_hi), (q_lo, q_hi)) owned by `rank`."""
    if num_kv_heads % world or num_q_heads % num_kv_heads:
        raise ValueError("KV heads must divide over ranks and q-heads over KV heads")
    kv = num_kv_heads // world
    q = num_q_heads // world
    return (rank * kv, (rank + 1) * kv), (rank * q, (rank + 1) * q)


def gathered_to_heads(gathered):
    """[N][B][Hq/N][D] (all-gather order) -> [B][Hq][D]; works for torch
    tensors and numpy arrays."""
    n, b, hq_local, d = gathered.shape
    if hasattr(gathered, "permute"):
        return gathered.permute(1, 0, 2, 3).reshape(b, n * hq_local, d)
    return gathered.transpose(1, 0, 2, 3).reshape(b, n * hq_local, d)
