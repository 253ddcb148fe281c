"""Failure detection of the expert-parallel path, without a GPU fault.

* the bounded waits on the communicator (csrc/ep_guard.hpp) against a
  scripted communicator and stream on a fake clock (tests/cpp/ep_guard_check.cpp);
* the host-side liveness check (k3xb.peers.PeerWatch) with real ranks as
  processes over a TCPStore: a rank that announces its departure between
  steps, and one that vanishes without a word, are both found on the host
  before the next launch, within the bound;
* the gloo restatement's exchange with a rank that raises before it: the
  surviving rank's collective ends with an error instead of waiting.
"""
import os
import shutil
import subprocess
import time

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_ep_guard_bounded_waits(tmp_path):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no C++ compiler")
    exe = tmp_path / "ep_guard_check"
    subprocess.run([cxx, "-std=c++20", "-O2", "-Wall", "-Wextra", "-Werror",
                    "-I", os.path.join(ROOT, "project-k3x_b200", "csrc"),
                    os.path.join(ROOT, "tests", "cpp", "ep_guard_check.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert out.stdout.startswith("ep guard ok"), out.stdout


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _watch_rank(rank, world, port, out_dir, mode, steps, timeout_s):
    from k3xb.peers import PeerLost, PeerWatch, make_store

    from datetime import timedelta
    store = make_store(rank, world, port=port, timeout_s=120)
    # every rank up before the bounded steps: a process that is still
    # importing torch is slow to start, not gone
    store.set(f"ready/{rank}", b"1")
    store.wait([f"ready/{g}" for g in range(world)], timedelta(seconds=120))
    watch = PeerWatch(store, rank, world, timeout_s=timeout_s)
    result = "ok"
    t0 = time.monotonic()
    try:
        for i in range(steps):
            if rank == world - 1 and i == 1 and mode != "healthy":
                if mode == "leave":
                    watch.leave()
                # "vanish": gone without a word (a crash between steps)
                open(os.path.join(out_dir, f"r{rank}.txt"), "w").write("left")
                if rank != 0:
                    os._exit(0)
            watch.step(i)
    except PeerLost as e:
        result = f"lost step={e.step} missing={e.missing} departed={e.departed}"
    elapsed = time.monotonic() - t0
    open(os.path.join(out_dir, f"r{rank}.txt"), "w").write(f"{result}\n{elapsed:.3f}")
    # the store's server (rank 0) outlives the other ranks' last use of it
    if mode == "healthy":
        store.set(f"done/{rank}", b"1")
        if rank == 0:
            store.wait([f"done/{g}" for g in range(world)], timedelta(seconds=120))
    elif rank == 0:
        time.sleep(0.2)


def _run_watch(tmp_path, mode, world=2, steps=3, timeout_s=2.0):
    port = _free_port()
    mp.start_processes(_watch_rank, args=(world, port, str(tmp_path), mode, steps, timeout_s), nprocs=world,
                       start_method="spawn")
    return [open(tmp_path / f"r{r}.txt").read().split("\n") for r in range(world)]


def test_peer_watch_healthy(tmp_path):
    res = _run_watch(tmp_path, "healthy", world=3)
    assert [r[0] for r in res] == ["ok"] * 3


def test_peer_watch_announced_departure(tmp_path):
    """Rank 1 leaves after step 0: rank 0's step 1 fails at once, naming it."""
    res = _run_watch(tmp_path, "leave", timeout_s=20.0)
    assert res[1] == ["left"]
    assert res[0][0] == "lost step=1 missing=[1] departed=[1]"
    assert float(res[0][1]) < 10.0   # well before the 20 s bound


def test_peer_watch_silent_departure(tmp_path):
    """Rank 1 vanishes after step 0: rank 0's step 1 fails at the bound."""
    res = _run_watch(tmp_path, "vanish", timeout_s=1.0)
    assert res[1] == ["left"]
    assert res[0][0] == "lost step=1 missing=[1] departed=[]"
    assert 1.0 <= float(res[0][1]) < 15.0


def test_peer_watch_arguments():
    from k3xb.peers import PeerWatch
    with pytest.raises(ValueError):
        PeerWatch(object(), 2, 2)
    with pytest.raises(ValueError):
        PeerWatch(object(), 0, 2, timeout_s=0)


def _gloo_rank(rank, world, port, out_dir):
    from datetime import timedelta

    import numpy as np
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:   # fails before the dispatch exchange (a host exception, no GPU involved)
        open(os.path.join(out_dir, "r1.txt"), "w").write("raised")
        os._exit(1)
    t0 = time.monotonic()
    send = torch.from_numpy(np.zeros((world, 4, 8), np.float32))
    parts = [torch.empty_like(send) for _ in range(world)]
    try:
        dist.all_gather(parts, send)
        result = "completed"
    except Exception as e:   # gloo reports the lost peer or the timeout
        result = "error " + type(e).__name__
    open(os.path.join(out_dir, "r0.txt"), "w").write(f"{result}\n{time.monotonic() - t0:.3f}")
    os._exit(0)


def test_gloo_exchange_with_a_failed_rank_ends(tmp_path):
    port = _free_port()
    spawn = mp.get_context("spawn")
    procs = [spawn.Process(target=_gloo_rank, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "the surviving rank did not return"
    r0 = open(tmp_path / "r0.txt").read().split("\n")
    assert open(tmp_path / "r1.txt").read() == "raised"
    assert r0[0].startswith("error"), r0
    assert float(r0[1]) < 60.0
