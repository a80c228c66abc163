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


def allgather_rows(local, total: int | None = None, align: int = GEMM_ROW_ALIGN, group=None):
    """Concatenate every rank's contiguous row block of a row-major output on every rank with
    one all_gather_into_tensor (NCCL on GPUs, gloo on CPU).

    ``total``: the rows of the whole output when the shards come from
    ``shard_range(total, world, rank, align)`` (``gemm_rows``): their sizes may differ (the
    ragged last chunk, or one chunk more on the lower ranks), so each rank pads its block to
    the largest share, and the padding is dropped from the gathered result. Without ``total``
    every rank's block must have the same number of rows."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rest = tuple(local.shape[1:])
    if total is None:
        counts = [local.shape[0]] * world
    else:
        counts = [shard_range(total, world, r, align)[1] for r in range(world)]
        rank = dist.get_rank(group)
        if counts[rank] != local.shape[0]:
            raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its share of {total} "
                             f"is {counts[rank]}")
    width = max(counts) if counts else 0
    send = local.contiguous()
    if send.shape[0] != width:
        padded = torch.zeros((width,) + rest, dtype=local.dtype, device=local.device)
        padded[:send.shape[0]] = send
        send = padded
    out = torch.empty((world * width,) + rest, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, send, group=group)
    if all(c == width for c in counts):
        return out
    return torch.cat([out[r * width:r * width + counts[r]] for r in range(world)])


class Comm:
    """The C ABI's own NCCL communicator (lvb_comm_*), the all-gather a host without
    torch.distributed uses (the Julia package binds the same calls). One per process and GPU.

        uid = Comm.unique_id()            # on rank 0, then sent to the others
        comm = Comm(uid, world, rank)     # every rank, on its current device
        comm.allgather(send, recv)        # recv = the ranks' sends, concatenated in rank order
    """

    @staticmethod
    def unique_id() -> bytes:
        from . import lvb_comm_id
        uid = lvb_comm_id()
        check(lib.lvb_comm_unique_id(C.byref(uid)))
        return C.string_at(C.addressof(uid), 128)

    def __init__(self, uid: bytes, nranks: int, rank: int):
        from . import lvb_comm_id
        if len(uid) != 128:
            raise ValueError("a communicator id has 128 bytes")
        cid = lvb_comm_id()
        C.memmove(C.addressof(cid), uid, 128)
        h = C.c_void_p()
        check(lib.lvb_comm_init(C.byref(h), C.byref(cid), int(nranks), int(rank)))
        self._h = h
        self.nranks, self.rank = int(nranks), int(rank)

    def allgather(self, send, recv, stream=None) -> None:
        """recv (a device tensor of nranks · send.nbytes bytes) <- every rank's send, in rank
        order, enqueued on `stream` (default: torch's current stream)."""
        import torch
        nbytes = send.numel() * send.element_size()
        if recv.numel() * recv.element_size() != nbytes * self.nranks:
            raise ValueError("recv must hold nranks x send bytes")
        if not (send.is_contiguous() and recv.is_contiguous()):
            raise ValueError("send and recv must be contiguous")
        s = stream if stream is not None else torch.cuda.current_stream()
        check(lib.lvb_allgather(self._h, C.c_void_p(send.data_ptr()), C.c_void_p(recv.data_ptr()),
                                nbytes, C.c_void_p(s.cuda_stream)))

    def close(self) -> None:
        if self._h:
            check(lib.lvb_comm_destroy(self._h))
            self._h = None
