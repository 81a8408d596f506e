"""Failure detection on the host, with Gloo ranks on the CPU.

A 3-rank data-parallel training job runs through the real CLI loop
(``nano_megatron_b200.train.main``). Rank 2 fails before step 2 in one of
four ways (host-side injection; no GPU is involved): it announces that it
leaves and exits, it raises, it dies without a word, or it stops without a
word. The surviving ranks must stop with ``PeerLost`` before they launch step
2, within a bounded time, and say which rank was lost and how. Without the
peer watch, the survivors' next collective must end with an error within the
process-group timeout.

The harness waits with a deadline and classifies every rank: it reported a
result (finished, or which exception), it crashed (non-zero exit without a
report), it exited silently, or it hung (still alive at the deadline; killed).
"""

import os
import queue
import socket
import time

import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.distributed

WORLD = 3
BASE_ARGS = ["--dp=3", "--steps=4", "--num-microbatches=1", "--micro-batch-size=1",
             "--n-layer=1", "--n-head=2", "--n-embd=16", "--vocab-size=32", "--seq-len=8",
             "--dp-bucket-mb=0", "--pg-timeout=20"]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, argv, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(WORLD), LOCAL_RANK=str(rank), OMP_NUM_THREADS="1")
    from nano_megatron_b200 import train
    from nano_megatron_b200.utils.health import PeerLost
    t0 = time.monotonic()
    try:
        train.main(argv)
        results.put((rank, "finished", None, time.monotonic() - t0))
    except PeerLost as exc:
        results.put((rank, "PeerLost", (exc.rank, exc.kind, exc.detail), time.monotonic() - t0))
    except BaseException as exc:  # noqa: BLE001 - the harness classifies it
        results.put((rank, type(exc).__name__, str(exc)[:300], time.monotonic() - t0))
        raise SystemExit(1)


def run_job(extra, deadline_s=90.0):
    """Run the job; return {rank: outcome} with outcome (status, info, seconds)."""
    spawn = mp.get_context("spawn")
    results = spawn.Queue()
    port = _free_port()
    procs = [spawn.Process(target=_rank_main, args=(r, port, BASE_ARGS + extra, results))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    outcome = {}
    deadline = time.monotonic() + deadline_s
    others_done_at = None
    while time.monotonic() < deadline and any(p.is_alive() for p in procs):
        try:
            rank, status, info, secs = results.get(timeout=0.2)
            outcome[rank] = (status, info, secs)
        except queue.Empty:
            pass
        # every rank either reported or is gone, except possibly a hung one
        if all(r in outcome or not procs[r].is_alive() for r in range(WORLD)):
            break
        if len(outcome) == WORLD - 1 and others_done_at is None:
            others_done_at = time.monotonic()
        if others_done_at is not None and time.monotonic() > others_done_at + 5:
            break  # a rank still silent 5 s after all others reported is hung
    while True:
        try:
            rank, status, info, secs = results.get(timeout=0.5)
            outcome[rank] = (status, info, secs)
        except queue.Empty:
            break
    for r, p in enumerate(procs):
        p.join(timeout=2)
        if p.is_alive():
            p.kill()
            p.join()
            outcome.setdefault(r, ("hung", None, None))
        elif r not in outcome:
            outcome[r] = ("crashed" if p.exitcode else "exited silently", p.exitcode, None)
    return outcome


@pytest.mark.parametrize("mode, kind, detail, lost_status", [
    ("leave", "left", "left on request before step 2", "exited silently"),
    ("raise", "left", "RuntimeError: injected fault before step 2", "RuntimeError"),
    ("vanish", "silent", "no announcement", "crashed"),
    ("hang", "silent", "no announcement", "hung"),
])
def test_survivors_stop_before_the_next_step(mode, kind, detail, lost_status):
    outcome = run_job(["--peer-timeout=4", f"--inject-fault=2:2:{mode}"])
    assert outcome[2][0] == lost_status, outcome
    for r in (0, 1):
        status, info, secs = outcome[r]
        assert status == "PeerLost", outcome
        lost_rank, lost_kind, lost_detail = info
        # a survivor may first hear of the other survivor stopping; either way rank 2 is named
        assert (lost_rank == 2 and lost_kind == kind and detail in lost_detail) or \
               (lost_rank in (0, 1) and "rank 2" in lost_detail), outcome
        assert secs < 60, outcome


def test_without_the_watch_the_next_collective_fails_within_the_pg_timeout():
    outcome = run_job(["--peer-timeout=0", "--inject-fault=2:2:vanish"])
    assert outcome[2][0] == "crashed" and outcome[2][1] == 3, outcome
    for r in (0, 1):
        status, info, secs = outcome[r]
        assert status not in ("finished", "hung", "PeerLost"), outcome
        assert secs < 60, outcome


def test_clean_job_finishes_on_every_rank():
    outcome = run_job(["--peer-timeout=30"])
    assert all(outcome[r][0] == "finished" for r in range(WORLD)), outcome
