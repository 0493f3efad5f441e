"""CPU tests (gloo, two ranks) of the row-sharded pair's host-side algorithm:
the distributed transpose (the index maps of the pack and unpack kernels in
comm.cu, with point-to-point exchanges like the NCCL all-to-all) and the
outgoing product from row-sharded operands with an all-gathered b."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def pack(src, rows, n, nranks):
    """pack[s][j][i] = src[i][s*rows + j] (transpose_pack_kernel)."""
    out = np.empty((nranks, rows, rows) + src.shape[2:], src.dtype)
    for s_ in range(nranks):
        for j in range(rows):
            for i in range(rows):
                out[s_, j, i] = src[i, s_ * rows + j]
    return out


def unpack(recv, rows, n):
    """dst[j][r*rows + i] = recv[r][j][i] (transpose_unpack_kernel)."""
    dst = np.empty((rows, n) + recv.shape[3:], recv.dtype)
    for j in range(rows):
        for col in range(n):
            r, i = divmod(col, rows)
            dst[j, col] = recv[r, j, i]
    return dst


def exchange(packed, rank, nranks):
    recv = np.empty_like(packed)
    reqs = []
    for peer in range(nranks):
        if peer == rank:
            recv[peer] = packed[peer]
            continue
        send_t = torch.from_numpy(np.ascontiguousarray(packed[peer]))
        recv_t = torch.empty_like(send_t)
        reqs.append(dist.isend(send_t, peer))
        reqs.append((dist.irecv(recv_t, peer), recv_t, peer))
    for r in reqs:
        if isinstance(r, tuple):
            r[0].wait()
            recv[r[2]] = r[1].numpy()
        else:
            r.wait()
    return recv


def _worker(rank, nranks, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=nranks, timeout=datetime.timedelta(seconds=60))
    try:
        n, c = 8, 3
        rows = n // nranks
        full = np.random.default_rng(0).standard_normal((n, n, c)).astype(np.float32)
        mine = full[rank * rows:(rank + 1) * rows]
        # distributed transpose
        zt = unpack(exchange(pack(mine, rows, n, nranks), rank, nranks), rows, n)
        ok_t = np.array_equal(zt, full.transpose(1, 0, 2)[rank * rows:(rank + 1) * rows])
        # twice is the identity
        back = unpack(exchange(pack(zt, rows, n, nranks), rank, nranks), rows, n)
        ok_tt = np.array_equal(back, mine)
        # outgoing product x[i, j] = sum_k a[i, k] b[j, k] from row shards and an all-gathered b
        a = np.random.default_rng(1).standard_normal((n, n)).astype(np.float64)
        b = np.random.default_rng(2).standard_normal((n, n)).astype(np.float64)
        gathered = [torch.empty(rows, n, dtype=torch.float64) for _ in range(nranks)]
        dist.all_gather(gathered, torch.from_numpy(b[rank * rows:(rank + 1) * rows].copy()))
        b_full = torch.cat(gathered).numpy()
        x_rows = a[rank * rows:(rank + 1) * rows] @ b_full.T
        ok_out = np.array_equal(x_rows, (a @ b.T)[rank * rows:(rank + 1) * rows])
        result[rank] = int(ok_t and ok_tt and ok_out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("nranks", [2, 4])
def test_sharded_pair_algorithm_on_gloo(nranks):
    ctx = mp.get_context("spawn")
    result = ctx.Array("i", nranks)
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, nranks, port, result)) for r in range(nranks)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert list(result) == [1] * nranks
