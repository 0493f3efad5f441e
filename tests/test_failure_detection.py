"""Failure detection of the sharded path, on the host only (no GPU is faulted).

- The library's watchdog loop (csrc/watchdog.h: the wait behind af2_sync and
  every host wait of a context with a communicator) against fake stream and
  communicator probes, built with g++ from tests/watchdog_check.cpp.
- af2cuda.PeerMonitor over gloo ranks on the CPU: a rank that leaves between
  steps (saying so, or by dying) is found on the host before the next step's
  launches, within the monitor's deadline.
"""
import datetime
import os
import shutil
import socket
import subprocess
import sys
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_watchdog_loop_against_fake_probes(tmp_path):
    exe = tmp_path / "watchdog_check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "alphafold2-webgpu_b200" / "csrc"),
                    str(ROOT / "tests" / "watchdog_check.cpp"), "-o", str(exe), "-pthread"], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, res.stdout + res.stderr
    assert res.stdout.strip() == "ok"


def _worker(rank, nranks, port, mode, result):
    sys.path.insert(0, str(ROOT / "alphafold2-webgpu_b200"))
    import torch
    import torch.distributed as dist

    from af2cuda.sharded import PeerLost, PeerMonitor
    store = dist.TCPStore("127.0.0.1", port, nranks, rank == 0, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=nranks,
                            timeout=datetime.timedelta(seconds=30))
    mon = PeerMonitor(store, rank, nranks, timeout=2.0)
    try:
        steps = 3
        for step in range(steps):
            if rank == nranks - 1 and step == 1 and mode != "all":
                # the last rank leaves between steps 0 and 1, with nothing in flight
                if mode == "leave":
                    mon.leave()
                    result.put((rank, "left", 0.0))
                    return
                result.put((rank, "died", 0.0))
                result.close()
                result.join_thread()
                os._exit(0)
            t0 = time.monotonic()
            try:
                mon.step()
            except PeerLost as e:
                result.put((rank, f"lost {e.missing} at {e.step}", time.monotonic() - t0))
                return
            t = torch.full((4,), float(rank + 1))
            dist.all_reduce(t)  # the step's collective, queued only after the check
            assert t[0].item() == nranks * (nranks + 1) / 2
        result.put((rank, "finished", 0.0))
    finally:
        if mode == "all":
            dist.destroy_process_group()


def _run(mode, nranks=2):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, nranks, port, mode, q)) for r in range(nranks)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(nranks):
        rank, what, waited = q.get(timeout=120)
        out[rank] = (what, waited)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_all_ranks_present_steps_pass():
    out = _run("all", nranks=3)
    assert all(what == "finished" for what, _ in out.values()), out


def test_rank_that_leaves_is_found_before_the_next_step():
    out = _run("leave", nranks=3)
    assert out[2][0] == "left"
    for r in (0, 1):
        what, waited = out[r]
        assert what == "lost [2] at 1", out
        assert waited < 1.5  # seen through the store at once, not at the 2 s deadline


def test_rank_that_dies_is_found_at_the_deadline():
    out = _run("die", nranks=2)
    assert out[1][0] == "died"
    what, waited = out[0]
    assert what == "lost [1] at 1", out
    assert 1.9 <= waited < 10
