"""Failure detection of a sharded network, on CPU (no GPU is faulted, hung or
trapped).

* The bounded wait behind ``kl_net_set_comm_timeout`` (``csrc/watchdog.h``)
  runs against fake streams, a fake communicator and a fake clock: a drained
  queue returns at once; a communicator error or the deadline aborts the
  communicator exactly once and then waits for the queue to drain.
* ``dist.Heartbeat`` over a TCPStore with two spawned ranks: a rank that
  leaves between steps, or that goes silent, is named to the survivor before
  the survivor's next launch; healthy ranks pass every check.
"""

import shutil
import socket
import subprocess
import time
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def test_bounded_wait_cases(tmp_path):
    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("g++ not found")
    exe = tmp_path / "watchdog_harness"
    subprocess.run([gxx, "-std=c++17", "-O1", "-I", str(ROOT / "klearu_b200" / "csrc"),
                    str(ROOT / "tests" / "native" / "watchdog_harness.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    rows = {ln.split()[0]: tuple(int(v) for v in ln.split()[1:]) for ln in out if ln.strip()}
    # (result, aborts, drained, comm_error); result 0 done, 1 comm error, 2 timeout
    assert rows["done"] == (0, 0, 1, 0)
    assert rows["comm_error"] == (1, 1, 1, 5)
    assert rows["timeout"] == (2, 1, 1, 0)
    assert rows["stuck"] == (2, 1, 0, 0)           # still pending after the abort: reported, not waited on
    assert rows["error_first"] == (1, 1, 1, 5)     # an error wins over a drained queue


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, scenario, out):
    import torch.distributed as dist

    from klearu_b200.dist import Heartbeat, RankFailure

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=__import__("datetime").timedelta(seconds=30))
    hb = Heartbeat(store, rank, world, timeout_s=1.5)
    events = []
    try:
        for step in range(5):
            hb.check(step)
            time.sleep(0.01)  # the step
            if rank == 1 and step == 1 and scenario == "leave":
                hb.leave()  # announced before the last beat: no peer launches step 2
                hb.beat()
                events.append(f"step{step} left")
                break
            if rank == 1 and step == 2 and scenario == "silent":
                events.append("silent")  # stops after step 1's beat without a word
                break
            hb.beat()
            events.append(f"step{step}")
    except RankFailure as e:
        events.append(f"failure {e.ranks} {e.reason} {e.step}")
    out.put((rank, events))
    if rank == 0:
        time.sleep(0.5)  # the store's server lives in rank 0: let the peer finish with it


def _run_ranks(scenario):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, scenario, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    return got


def test_heartbeat_healthy_ranks():
    got = _run_ranks("healthy")
    assert got[0] == got[1] == [f"step{s}" for s in range(5)]


def test_heartbeat_rank_left_between_steps():
    t0 = time.monotonic()
    got = _run_ranks("leave")
    assert got[1] == ["step0", "step1 left"]
    assert got[0] == ["step0", "step1", "failure [1] left 2"]
    assert time.monotonic() - t0 < 60


def test_heartbeat_silent_rank():
    got = _run_ranks("silent")
    assert got[1] == ["step0", "step1", "silent"]
    # the survivor launched step 2 before the silence showed: on the GPU that
    # step's collectives are what kl_net_set_comm_timeout bounds
    assert got[0] == ["step0", "step1", "step2", "failure [1] silent 3"]


def test_heartbeat_single_rank_and_every(tmp_path):
    """One rank never waits; with every=2 only even steps are checked."""
    import torch.distributed as dist

    from klearu_b200.dist import Heartbeat, RankFailure

    store = dist.FileStore(str(tmp_path / "store"), 2)
    Heartbeat(store, 0, 1, timeout_s=0.1).check(5)  # world of one: nothing to wait for
    hb = Heartbeat(store, 0, 2, timeout_s=0.2, every=2)
    hb.check(0)  # step 0 needs no finished steps
    hb.beat()
    hb.check(1)  # odd step: not checked, the silent peer is not noticed yet
    hb.beat()
    t0 = time.monotonic()
    with pytest.raises(RankFailure) as e:
        hb.check(2)
    assert e.value.ranks == [1] and e.value.reason == "silent"
    assert time.monotonic() - t0 >= 0.2
