"""Row-sharded triangle multiplication (channel-sharded contraction) and
outer-product mean on 2+ GPUs (one process per GPU, the library's NCCL
communicator): every rank's rows must be bit-identical to the single-GPU
result.  Skipped on boxes with fewer than two GPUs."""
import datetime
import os
import socket
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, nranks, port, result):
    sys.path.insert(0, str(ROOT / "alphafold2-webgpu_b200"))
    sys.path.insert(0, str(ROOT / "tests"))
    import numpy as np
    import torch
    import torch.distributed as dist

    import af2cuda
    from helpers import pack, triangle_case

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=nranks, timeout=datetime.timedelta(seconds=120))
    dev = af2cuda.Device(rank)
    ok = True
    try:
        uid = [af2cuda.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        af2cuda.comm_init(dev, uid[0], nranks, rank)
        # 64 rows per rank: the outgoing product copies the rank's own channel group;
        # whole 128-row tiles: it reads the group in place
        for n in sorted({64 * nranks, 256}):
            r0, r1 = af2cuda.rows_of(n, nranks, rank)
            z, mask, w = triangle_case(n, seed=7, mask_p=0.9, perturbed=True)
            mask[:, 17] = 0
            packed = torch.from_numpy(pack(w)).cuda()
            mask_d = torch.from_numpy(mask).cuda()
            torch.cuda.synchronize()
            for direction in (0, 1):
                full = torch.from_numpy(z).to("cuda", torch.bfloat16)
                rows = torch.from_numpy(z[r0:r1]).to("cuda", torch.bfloat16).contiguous()
                mask_rows = mask_d[r0:r1].contiguous()
                torch.cuda.synchronize()  # the library runs on its own stream
                af2cuda.encode_triangle_multiplication_tensors(dev, direction, full, mask_d, packed, residual=True)
                af2cuda.encode_triangle_multiplication_sharded_tensors(dev, direction, rows, mask_rows, packed, n,
                                                                       residual=True)
                dev.sync()
                ok &= bool(torch.equal(rows, full[r0:r1]))
        # f32 pair, written out of place, both directions
        zf = torch.from_numpy(z).cuda()
        zf_rows, mask_rows = zf[r0:r1].contiguous(), mask_d[r0:r1].contiguous()
        for direction in (0, 1):
            ref = torch.empty_like(zf)
            out_rows = torch.empty(r1 - r0, n, z.shape[2], device="cuda")
            torch.cuda.synchronize()
            af2cuda.encode_triangle_multiplication_tensors(dev, direction, zf, mask_d, packed, out=ref, residual=False)
            af2cuda.encode_triangle_multiplication_sharded_tensors(dev, direction, zf_rows, mask_rows, packed, n,
                                                                   out=out_rows, residual=False)
            dev.sync()
            ok &= bool(torch.equal(out_rows, ref[r0:r1]))
        # outer-product mean of a whole MSA into this rank's pair rows
        from test_opm_gpu import opm_case, opm_packed
        m, msa_mask, wo = opm_case(40, n, 64, cz=128, seed=4)
        msa = torch.from_numpy(m).to("cuda", torch.bfloat16)
        msa_mask_d = torch.from_numpy(msa_mask).cuda()
        pw = torch.from_numpy(opm_packed(wo)).cuda()
        pair_full = torch.from_numpy(z).to("cuda", torch.bfloat16)
        pair_rows = pair_full[r0:r1].clone()
        torch.cuda.synchronize()
        af2cuda.encode_outer_product_mean_tensors(dev, msa, msa_mask_d, pw, 32, 128, pair=pair_full, residual=True)
        msa_cols = msa[:, r0:r1].contiguous()  # this rank's residue columns
        af2cuda.encode_outer_product_mean_sharded_tensors(dev, msa_cols, msa_mask_d, pw, 32, 128, pair_rows,
                                                          residual=True)
        dev.sync()
        ok &= bool(torch.equal(pair_rows, pair_full[r0:r1]))
        af2cuda.comm_destroy(dev)
    finally:
        dev.close()
        dist.destroy_process_group()
    result[rank] = int(ok)


def test_sharded_pair_ops_are_bit_identical():
    import torch
    import torch.multiprocessing as mp
    count = torch.cuda.device_count()
    if count < 2:
        pytest.skip("needs two or more GPUs")
    nranks = 4 if count >= 4 else 2
    ctx = mp.get_context("spawn")
    result = ctx.Array("i", nranks)
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, nranks, port, result)) for r in range(nranks)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert list(result) == [1] * nranks


def _leave_worker(rank, nranks, port, result):
    """Two sharded steps with a short watchdog deadline; then the last rank leaves between
    steps (nothing of its own in flight), and the others find it on the host before the
    next step's launches, abort their communicators locally and keep using their GPUs."""
    sys.path.insert(0, str(ROOT / "alphafold2-webgpu_b200"))
    sys.path.insert(0, str(ROOT / "tests"))
    import torch
    import torch.distributed as dist

    import af2cuda
    from helpers import pack, triangle_case

    torch.cuda.set_device(rank)
    store = dist.TCPStore("127.0.0.1", port, nranks, rank == 0, timeout=datetime.timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=nranks, timeout=datetime.timedelta(seconds=60))
    dev = af2cuda.Device(rank)
    ok = True
    try:
        uid = [af2cuda.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        af2cuda.comm_init(dev, uid[0], nranks, rank)
        af2cuda.comm_set_timeout(dev, 20.0)
        mon = af2cuda.PeerMonitor(store, rank, nranks, timeout=10.0)
        n = 64 * nranks
        r0, r1 = af2cuda.rows_of(n, nranks, rank)
        z, mask, w = triangle_case(n, seed=3)
        packed = torch.from_numpy(pack(w)).cuda()
        rows = torch.from_numpy(z[r0:r1]).to("cuda", torch.bfloat16).contiguous()
        mask_rows = torch.from_numpy(mask[r0:r1]).cuda().contiguous()
        torch.cuda.synchronize()
        for step in range(3):
            if step == 2 and rank == nranks - 1:
                mon.leave()
                af2cuda.comm_abort(dev)
                break
            try:
                mon.step()
            except af2cuda.PeerLost as e:
                ok &= step == 2 and e.missing == [nranks - 1]
                af2cuda.comm_abort(dev)
                # the context still runs single-GPU work
                full = torch.from_numpy(z).to("cuda", torch.bfloat16)
                mask_d = torch.from_numpy(mask).cuda()
                torch.cuda.synchronize()
                af2cuda.encode_triangle_multiplication_tensors(dev, 0, full, mask_d, packed)
                dev.sync()
                ok &= bool(torch.isfinite(full.float()).all())
                try:  # the sharded form now reports that there is no communicator
                    af2cuda.encode_triangle_multiplication_sharded_tensors(dev, 0, rows, mask_rows, packed, n)
                    ok = False
                except (af2cuda.Af2Error, af2cuda.RangeError):
                    pass
                break
            af2cuda.encode_triangle_multiplication_sharded_tensors(dev, step % 2, rows, mask_rows, packed, n)
            dev.sync()  # the watchdog's wait
        else:
            ok = False
    finally:
        dev.close()
    result[rank] = int(ok)


def test_rank_leaving_between_steps_is_found_on_the_host():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two or more GPUs")
    nranks = 2
    ctx = mp.get_context("spawn")
    result = ctx.Array("i", nranks)
    port = _free_port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    old = os.environ.copy()
    os.environ.update(env)
    try:
        procs = [ctx.Process(target=_leave_worker, args=(r, nranks, port, result)) for r in range(nranks)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
    finally:
        os.environ.clear()
        os.environ.update(old)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert list(result) == [1] * nranks
