"""CPU tier: the multi-GPU host logic — shard planning (C ABI lvb_shard_range) and the
shard-then-gather flow — on world_size-2 gloo process groups. The per-shard compute here is
the CPU oracle standing in for each rank's GPU kernel; the GPU path itself runs in
bench.py under torchrun."""
import os
import socket

import numpy as np
import pytest


def test_shard_range_partitions(lvb):
    from lvb.dist import shard_range, gemm_rows, attention_units
    for total in (0, 1, 127, 128, 1000, 8192, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            for align in (1, 128):
                spans = [shard_range(total, world, r, align) for r in range(world)]
                pos = 0
                for b, n in spans:                 # contiguous, in rank order, covering all
                    assert b == pos and n >= 0
                    pos += n
                assert pos == total
                for b, n in spans:
                    assert n == 0 or b % align == 0   # non-empty shares start on a tile
                chunks = [-(-n // align) for _, n in spans]   # whole chunks per share
                assert max(chunks) - min(chunks) <= 1
    assert gemm_rows(8192 * 8, 8, 3) == (3 * 8192, 8192)
    assert attention_units(4, 32, 8, 0) == [(0, h) for h in range(16)]
    assert attention_units(8, 8, 8, 7) == [(7, h) for h in range(8)]
    with pytest.raises(lvb.LavaError):
        shard_range(10, 2, 2, 1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo), str(repo / "lava.jl_b200")]
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from lvb.dist import gemm_rows, allgather_rows, attention_units
        from oracle.gemm import gemm_ref
        from oracle.inputs import gemm_inputs
        from oracle.attention import attention_ref
        from oracle.inputs import attention_inputs
        # GEMM: every rank computes its tile-aligned row block of C = A·B, then all-gather.
        M, N, K = 512, 96, 64
        A, Bt = gemm_inputs(M, N, K, "Int8", seed=3)
        r0, rn = gemm_rows(M, world, rank)
        local = torch.from_numpy(gemm_ref(A[r0:r0 + rn], Bt.T, "Int32"))
        full = allgather_rows(local)
        ok_gemm = np.array_equal(full.numpy(), gemm_ref(A, Bt.T, "Int32"))
        # uneven shares (1000 rows: 512 + 488): padded to the largest share for the gather,
        # the padding dropped from the result
        M2 = 1000
        A2, Bt2 = gemm_inputs(M2, N, K, "Int8", seed=8)
        r0, rn = gemm_rows(M2, world, rank)
        local2 = torch.from_numpy(gemm_ref(A2[r0:r0 + rn], Bt2.T, "Int32"))
        full2 = allgather_rows(local2, total=M2)
        ok_gemm &= tuple(full2.shape) == (M2, N)
        ok_gemm &= np.array_equal(full2.numpy(), gemm_ref(A2, Bt2.T, "Int32"))
        # attention: (batch, kv-head) units, each with its group of query heads
        Q, Kt, V = attention_inputs(2, 4, 2, 64, 64, "Float16", seed=4)
        ref = attention_ref(Q, Kt, V, True, 0.125)
        g = 2
        ok_attn = True
        for (b, hk) in attention_units(2, 2, world, rank):
            hs = slice(hk * g, (hk + 1) * g)
            o = attention_ref(Q[b:b + 1, hs], Kt[b:b + 1, hk:hk + 1], V[b:b + 1, hk:hk + 1], True, 0.125)
            ok_attn &= np.allclose(o, ref[b:b + 1, hs], atol=1e-12)
        # max over ranks of a per-rank time, as bench.py reports it
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, bool(ok_gemm), bool(ok_attn), float(t.item())))
    finally:
        dist.destroy_process_group()


def test_two_rank_shard_and_gather_gloo(lvb):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    for rank, ok_gemm, ok_attn, tmax in res:
        assert ok_gemm and ok_attn and tmax == 2.0


def test_comm_host_side(lvb):
    """The C ABI's all-gather (lvb_comm_*) without a GPU: communicator ids (128 bytes, fresh
    each time) and the argument checks that come before any device work."""
    import ctypes as C
    from lvb.dist import Comm
    try:
        u1, u2 = Comm.unique_id(), Comm.unique_id()
    except lvb.LavaError as e:            # no NCCL on this machine: reported, not a crash
        assert e.status == 5
    else:
        assert len(u1) == len(u2) == 128 and u1 != u2
    for nranks, rank in [(2, 2), (2, -1), (0, 0)]:
        with pytest.raises(lvb.LavaError) as ei:
            Comm(bytes(128), nranks, rank)
        assert ei.value.status == 1
    with pytest.raises(ValueError):
        Comm(bytes(5), 1, 0)
    assert lvb.lib.lvb_allgather(None, None, None, 16, None) == 1
    assert lvb.lib.lvb_comm_destroy(None) == 0
    n, r = C.c_int32(), C.c_int32()
    assert lvb.lib.lvb_comm_size(None, C.byref(n), C.byref(r)) == 1
