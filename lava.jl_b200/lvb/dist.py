"""Multi-GPU plumbing for the path: one process per GPU, independent shards, an optional
NCCL all-gather of the outputs (torch.distributed over NVLink/NVSwitch).

Lava itself has no multi-device code. The units here are independent — GEMM output rows
(B replicated), attention (batch, kv-head) groups (a group's query heads never need another
group's K/V) — so each rank computes a contiguous range with no collective on the data path;
the all-gather exists only for a caller that wants the whole output on every GPU.
"""
from __future__ import annotations

import ctypes as C

from . import lib, check

GEMM_ROW_ALIGN = 128      # one MMA tile of rows: shards never split a tile


def shard_range(total: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """(begin, count) of rank's contiguous share (C ABI lvb_shard_range)."""
    b, n = C.c_int64(), C.c_int64()
    check(lib.lvb_shard_range(int(total), int(world), int(rank), int(align), C.byref(b), C.byref(n)))
    return b.value, n.value


def gemm_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    """Rows of A (and of C) owned by rank: tile-aligned contiguous block."""
    return shard_range(M, world, rank, GEMM_ROW_ALIGN)


def attention_units(B: int, Hkv: int, world: int, rank: int) -> list[tuple[int, int]]:
    """(batch, kv_head) groups owned by rank; each carries its Hq/Hkv query heads."""
    b0, n = shard_range(B * Hkv, world, rank, 1)
    return [divmod(u, Hkv) for u in range(b0, b0 + n)]


def allgather_rows(local, group=None):
    """Concatenate every rank's contiguous row block (row-major C shards of equal size)
    on every rank with one all_gather_into_tensor (NCCL on GPUs, gloo on CPU)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out
