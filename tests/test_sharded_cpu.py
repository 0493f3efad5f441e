"""CPU tests (gloo, two, four and eight ranks) of the row-sharded pair's host-side
algorithm for the triangle products: every rank projects its own pair rows in
R channel groups, an all-to-all hands every rank its channel group of all rows,
each rank contracts its channels over the whole N x N (the incoming product's k
running over the ranks' row blocks in order), and a second all-to-all returns
all channels of the rank's own rows.  The block layouts and exchanges are the
ones of triangle.cu / comm.cu, emulated with numpy and point-to-point gloo
messages; the results must equal the unsharded products exactly."""
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


def all_to_all(blocks, rank, nranks):
    """blocks[p] goes to rank p; returns recv with recv[p] = rank p's block for this rank."""
    recv = [None] * nranks
    pending = []
    for peer in range(nranks):
        if peer == rank:
            recv[peer] = blocks[peer].copy()
            continue
        send_t = torch.from_numpy(np.ascontiguousarray(blocks[peer]))
        recv_t = torch.empty_like(send_t)
        pending.append((dist.isend(send_t, peer), None, None))
        pending.append((dist.irecv(recv_t, peer), recv_t, peer))
    for req, buf, peer in pending:
        req.wait()
        if buf is not None:
            recv[peer] = buf.numpy()
    return recv


def _worker(rank, nranks, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=nranks, timeout=datetime.timedelta(seconds=60))
    try:
        n, c = 16, 8
        rows, hq = n // nranks, c // nranks
        mine = slice(rank * rows, (rank + 1) * rows)
        rng = np.random.default_rng(0)
        # gated projections of the whole pair, [pair row][pair column][channel]
        a = rng.standard_normal((n, n, c))
        b = rng.standard_normal((n, n, c))
        ok = True
        # ---- outgoing: x[i, j, h] = sum_k a[i, k, h] b[j, k, h] ----
        # projected local operands [group q][row][hq][k]
        a_loc = [a[mine, :, q * hq:(q + 1) * hq].transpose(0, 2, 1) for q in range(nranks)]
        b_loc = [b[mine, :, q * hq:(q + 1) * hq].transpose(0, 2, 1) for q in range(nranks)]
        a_all = np.concatenate(all_to_all(a_loc, rank, nranks))  # [n][hq][k]: every row, this rank's channels
        b_all = np.concatenate(all_to_all(b_loc, rank, nranks))
        x = np.einsum("ihk,jhk->hij", a_all, b_all)  # [hq][n][n]
        x_blocks = [x[:, p * rows:(p + 1) * rows] for p in range(nranks)]  # one block per destination rank
        x_rows = np.concatenate(all_to_all(x_blocks, rank, nranks))  # [c][rows][n]
        ok &= np.allclose(x_rows, np.einsum("ikh,jkh->hij", a, b)[:, mine], rtol=0, atol=1e-12)
        # ---- incoming: x[i, j, h] = sum_k a[k, j, h] b[k, i, h]; this rank holds rows k ----
        # projected local operands [group q][column][hq][local k]
        ai_loc = [a[mine, :, q * hq:(q + 1) * hq].transpose(1, 2, 0) for q in range(nranks)]
        bi_loc = [b[mine, :, q * hq:(q + 1) * hq].transpose(1, 2, 0) for q in range(nranks)]
        ai_all = np.stack(all_to_all(ai_loc, rank, nranks))  # [k block][n][hq][rows]
        bi_all = np.stack(all_to_all(bi_loc, rank, nranks))
        # k runs over the blocks in rank order, then inside each block
        ai_k = ai_all.transpose(1, 2, 0, 3).reshape(n, hq, n)
        bi_k = bi_all.transpose(1, 2, 0, 3).reshape(n, hq, n)
        xi = np.einsum("ihk,jhk->hij", bi_k, ai_k)
        xi_rows = np.concatenate(all_to_all([xi[:, p * rows:(p + 1) * rows] for p in range(nranks)], rank, nranks))
        ok &= np.allclose(xi_rows, np.einsum("kjh,kih->hij", a, b)[:, mine], rtol=0, atol=1e-12)
        result[rank] = int(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_channel_sharded_triangle_algorithm_on_gloo(nranks):
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
