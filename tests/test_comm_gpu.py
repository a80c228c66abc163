"""GPU tier, two GPUs: the C ABI's own all-gather (lvb_comm_* / lvb_allgather, NCCL over
NVLink) — each rank computes its row shard of an int8 GEMM (lvb_shard_range, 128-row
chunks), the shards are gathered on every rank, and the gathered C is bit-exact against
the oracle. Also: gathering in place (send = the rank's own slot of recv) and
an uneven last shard padded to the common size. Skipped on a box with fewer than 2 GPUs.

Ranks are spawned processes (one per GPU); rank 0 makes the communicator id and hands it
to the other through a pipe, as a host would through its own channel.
"""
import multiprocessing as mp
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]


def _rank(rank, world, uid_conn, out_conn, M, N, K):
    try:
        sys.path[:0] = [str(REPO), str(REPO / "lava.jl_b200")]
        import torch
        torch.cuda.set_device(rank)
        import lvb
        from lvb.dist import Comm, shard_range
        from oracle.gemm import gemm_ref
        from oracle.inputs import gemm_inputs

        if rank == 0:
            uid = Comm.unique_id()
            uid_conn.send(uid)
        else:
            uid = uid_conn.recv()
        comm = Comm(uid, world, rank)

        A, Bt = gemm_inputs(M, N, K, "Int8", seed=21)
        # Row shards of a row-major C; every shard padded to the largest so the gathered
        # buffer is [world][rows_max][N].
        shares = [shard_range(M, world, r, 128) for r in range(world)]
        rows_max = max(n for _, n in shares)
        b0, n = shares[rank]
        dA = torch.from_numpy(A[b0:b0 + n]).cuda()
        dB = torch.from_numpy(Bt).cuda().t()
        recv = torch.zeros(world * rows_max, N, dtype=torch.int32, device="cuda")
        mine = recv[rank * rows_max: rank * rows_max + n]
        if n:
            lvb.gemm(mine, dA, dB)
        comm.allgather(recv[rank * rows_max:(rank + 1) * rows_max], recv)   # in place
        torch.cuda.synchronize()
        assert lvb.device_status() == (0, 0, 0)
        got = recv.cpu().numpy()
        ref = gemm_ref(A, Bt.T, "Int32")
        full = np.concatenate([got[r * rows_max: r * rows_max + shares[r][1]] for r in range(world)])
        ok_inplace = np.array_equal(full, ref)

        # Out of place, a float tensor.
        x = torch.full((1000,), float(rank + 1), device="cuda")
        y = torch.empty(world * 1000, device="cuda")
        comm.allgather(x, y)
        torch.cuda.synchronize()
        ok_out = all(bool((y[r * 1000:(r + 1) * 1000] == r + 1).all()) for r in range(world))
        comm.close()
        out_conn.send(("ok", ok_inplace, ok_out))
    except Exception as e:  # noqa: BLE001
        out_conn.send(("error", repr(e), False))


def test_allgather_two_gpus(lvb, torch_cuda):
    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    uid_send, uid_recv = ctx.Pipe()
    outs = [ctx.Pipe(duplex=False) for _ in range(world)]      # (reader, writer)
    M, N, K = 1000, 384, 512        # shards of 512 and 488 rows
    procs = [ctx.Process(target=_rank, args=(0, world, uid_send, outs[0][1], M, N, K)),
             ctx.Process(target=_rank, args=(1, world, uid_recv, outs[1][1], M, N, K))]
    for p in procs:
        p.start()
    try:
        results = []
        for conn, _ in outs:
            if not conn.poll(240):
                raise AssertionError("a rank did not answer within 240 s")
            results.append(conn.recv())
        for p in procs:
            p.join(60)
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(10)
    for status, inplace, out in results:
        assert status == "ok", inplace
        assert inplace and out
