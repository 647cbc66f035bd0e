"""Tensor parallelism plumbing: one process per GPU, NCCL inside libshardlm_cuda.

The library owns the NCCL communicator (shd_tp_init) and does its own all-reduces of the packed
[2][M][h] partial shares after the row-parallel linears (o, down) and the max-reduction of argmax
keys. What runs here is the host side around it: the slice each rank holds (shd_tp_plan, a pure
host computation) and the exchange of the NCCL unique id over an already initialised
torch.distributed group (gloo or nccl), before any of the library's collectives exist.

The reference has no working tensor parallelism to mirror (its multi-GPU path is a layer
round-robin over host hops, and crates/v2/core/src/parallel.rs:89-98 refuses head counts that do
not divide); the plan here splits query heads evenly, replicates a kv head on every rank whose
query heads read it, splits the intermediate dimension in 16-row blocks and the vocabulary evenly.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import NL_APPROX, NL_GPU, ModelConfigC, ShardInfoC, check, lib

NCCL_UNIQUE_ID_BYTES = 128


@dataclass(frozen=True)
class ShardPlan:
    """One rank's slice: half-open ranges of query heads, kv heads, intermediate rows, vocab rows."""
    rank: int
    world: int
    q_heads: range
    kv_heads: range
    inter: range
    vocab: range


def tp_plan(shape, rank: int, world: int) -> ShardPlan:
    """shd_tp_plan for a ModelShape (no device needed)."""
    cfg = ModelConfigC(shape.hidden, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.head_dim,
                       shape.intermediate, shape.vocab, shape.rope_theta, shape.rms_eps, 1, 1,
                       NL_APPROX, NL_GPU, NL_APPROX, 0, rank, world)
    info = ShardInfoC()
    check(lib().shd_tp_plan(C.byref(cfg), C.byref(info)))
    r = lambda b, n: range(b, b + n)
    return ShardPlan(rank, world, r(info.q_head_begin, info.q_head_count),
                     r(info.kv_head_begin, info.kv_head_count), r(info.inter_begin, info.inter_count),
                     r(info.vocab_begin, info.vocab_count))


def share_unique_id(rank: int, device: torch.device | str = "cpu", make_id=None) -> bytes:
    """Rank 0 creates the NCCL unique id (shd_tp_unique_id), every rank receives it by a broadcast
    on the default torch.distributed group; `device` is where that group's tensors live ("cpu" for
    gloo, the rank's GPU for nccl). `make_id` replaces the id source (tests)."""
    import torch.distributed as dist

    buf = torch.zeros(NCCL_UNIQUE_ID_BYTES, dtype=torch.uint8, device=device)
    if rank == 0:
        if make_id is not None:
            raw = np.frombuffer(make_id(), np.uint8)
        else:
            host = np.zeros(NCCL_UNIQUE_ID_BYTES, np.uint8)
            check(lib().shd_tp_unique_id(host.ctypes.data))
            raw = host
        if raw.size != NCCL_UNIQUE_ID_BYTES:
            raise ValueError(f"unique id must be {NCCL_UNIQUE_ID_BYTES} bytes, got {raw.size}")
        buf.copy_(torch.from_numpy(raw.copy()))
    dist.broadcast(buf, 0)
    return bytes(buf.cpu().numpy().tobytes())


def init_tensor_parallel(ctx, rank: int, world: int) -> None:
    """Create the library's NCCL communicator for this rank (after torch.distributed is up)."""
    uid = share_unique_id(rank, device=torch.device("cuda", ctx.device))
    host = np.frombuffer(uid, np.uint8).copy()
    ctx.bind_stream()
    check(lib().shd_tp_init(ctx.ptr, rank, world, host.ctypes.data), ctx.ptr)
