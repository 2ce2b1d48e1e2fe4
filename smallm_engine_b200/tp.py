"""Host side of tensor parallelism: which rows each rank owns, the NCCL id
handshake, and the max-over-ranks timing reduction.

The device-side split lives in ``csrc/model.cu`` (Model::load); ``tp_plan``
states the same split so callers and tests can reason about shards:

* query heads, KV heads and FFN rows are cut into ``tp_size`` equal
  contiguous blocks (column-parallel Q/K/V and gate/up);
* O and down are row-parallel: rank r reads the columns of its heads /
  FFN rows and its partial sum is all-reduced into the residual;
* the output projection is vocab-parallel, ceil(vocab / tp_size) rows per
  rank (the last rank may own fewer).

There is no such split in the reference, which is single-process
(src/model/qwen2_model.cpp owns the whole model).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

TP_SIZES = (1, 2, 4, 8)


@dataclass(frozen=True)
class Shard:
    """Half-open ranges [begin, end) of one rank's share."""
    heads: tuple[int, int]
    kv_heads: tuple[int, int]
    ffn_rows: tuple[int, int]
    vocab_rows: tuple[int, int]


def tp_plan(n_heads: int, n_kv_heads: int, ffn: int, vocab: int, tp_size: int, rank: int) -> Shard:
    """Rank `rank`'s share at degree `tp_size` (Model::load in csrc/model.cu);
    raises ValueError where the library returns SMALLM_ERR_INVALID."""
    if tp_size not in TP_SIZES:
        raise ValueError("tp_size must be 1, 2, 4 or 8")
    if not 0 <= rank < tp_size:
        raise ValueError("tp_rank out of range")
    if n_heads % tp_size or n_kv_heads % tp_size or ffn % tp_size:
        raise ValueError("tensor parallel degree does not divide the head / FFN counts")
    nh, nkv, nf = n_heads // tp_size, n_kv_heads // tp_size, ffn // tp_size
    nv = -(-vocab // tp_size)
    v0 = min(vocab, rank * nv)
    return Shard((rank * nh, (rank + 1) * nh), (rank * nkv, (rank + 1) * nkv), (rank * nf, (rank + 1) * nf),
                 (v0, min(vocab, v0 + nv)))


def new_nccl_id() -> bytes:
    """A fresh 128-byte ncclUniqueId from the library."""
    from ._lib import check, lib
    b = ctypes.create_string_buffer(128)
    check(lib().smallm_nccl_unique_id(b))
    return bytes(b.raw)


def share_nccl_id(rank: int, world_size: int, make=new_nccl_id) -> bytes | None:
    """Rank 0 makes the id and every rank receives it over the default
    torch.distributed group (any backend); None on a single rank."""
    if world_size == 1:
        return None
    import torch.distributed as dist
    buf = [make() if rank == 0 else None]
    dist.broadcast_object_list(buf, src=0)
    return buf[0]


def max_over_ranks(value: float, world_size: int, device: str | None = None) -> float:
    """The largest of the ranks' values (a multi-GPU time is the slowest
    rank's); the tensor lives on `device` (the NCCL backend needs the GPU)."""
    if world_size == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
