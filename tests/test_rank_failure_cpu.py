"""Failure detection of bench.py's multi-rank path, as gloo ranks on CPU (no GPU).

The path's one collective (gather_embeddings) is preceded by a host-side readiness
exchange (bench.rank_checkpoint) in the process group's store, and the group is
formed with a short timeout (bench.init_ranks). Each case makes the failure on the
host and checks that every surviving rank ends with an error within a bound well
under any hang:
* a rank raises before the all-gather and reports it (bench.main's handler does
  this): the peers stop at once, naming the failed rank and its error;
* a rank exits before the all-gather without reporting: the peers stop at the
  checkpoint's timeout;
* the rank hosting the store exits: the survivor stops (store unreachable or
  timeout), not hangs;
* a rank leaves between steps, after the checkpoint: the survivor's next all-gather
  ends with an error within the group's timeout.
"""
import os
import socket
import time

import pytest

import bench

TIMEOUT_S = 4.0  # checkpoint / process-group timeout in these tests


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, scenario, out_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world))
    bench.init_ranks("gloo", timeout_s=TIMEOUT_S)
    t0 = time.monotonic()
    try:
        if scenario == "raise" and rank == 1:
            try:
                raise ValueError("weights file unreadable")
            except ValueError as e:
                bench.report_rank_error(e)
                out_q.put((rank, "raised", str(e), 0.0))
                return
        if scenario == "exit" and rank == 1:
            os._exit(3)
        if scenario == "store_host_exit" and rank == 0:
            os._exit(3)
        bench.rank_checkpoint("setup", timeout_s=TIMEOUT_S)
        local = torch.full((4, 8), float(rank))
        gathered = torch.empty(world * 4, 8)
        bench.gather_embeddings(local, gathered, world)  # step 1: every rank is here
        if scenario == "leave_between_steps" and rank == 1:
            os._exit(0)
        bench.gather_embeddings(local, gathered, world)  # step 2
        out_q.put((rank, "ok", "", time.monotonic() - t0))
    except Exception as e:
        out_q.put((rank, type(e).__name__, str(e), time.monotonic() - t0))
    finally:
        if scenario == "ok":
            dist.destroy_process_group()


def _run(scenario, world=2, expect_reports=None):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, scenario, q))
             for r in range(world)]
    for p in procs:
        p.start()
    n = world if expect_reports is None else expect_reports
    res = {}
    for _ in range(n):
        r, kind, msg, dt = q.get(timeout=120)
        res[r] = (kind, msg, dt)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join()
    return res


def test_healthy_ranks_pass_the_checkpoint():
    res = _run("ok", world=3)
    assert {r: v[0] for r, v in res.items()} == {0: "ok", 1: "ok", 2: "ok"}


def test_rank_that_raises_stops_its_peers_at_once():
    res = _run("raise", world=3)
    assert res[1][0] == "raised"
    for r in (0, 2):
        kind, msg, dt = res[r]
        assert kind == "RankFailure", res[r]
        assert "rank 1 failed" in msg and "weights file unreadable" in msg
        assert dt < TIMEOUT_S, dt  # told by the store, not by the timeout


def test_rank_that_exits_silently_times_out_the_checkpoint():
    res = _run("exit", world=2, expect_reports=1)
    kind, msg, dt = res[0]
    assert kind == "RankFailure", res[0]
    assert "[1] did not reach 'setup'" in msg
    assert TIMEOUT_S * 0.9 <= dt < TIMEOUT_S + 10


def test_store_host_exit_does_not_hang_the_survivor():
    res = _run("store_host_exit", world=2, expect_reports=1)
    kind, msg, dt = res[1]
    assert kind == "RankFailure", res[1]
    assert dt < TIMEOUT_S + 30


def test_rank_leaving_between_steps_fails_the_next_gather():
    res = _run("leave_between_steps", world=2, expect_reports=1)
    kind, msg, dt = res[0]
    assert kind != "ok", res[0]
    assert dt < TIMEOUT_S + 30


def test_checkpoint_is_a_no_op_without_a_group():
    bench.rank_checkpoint("anything", timeout_s=0.0)
    bench.report_rank_error(RuntimeError("x"))


@pytest.mark.parametrize("tag", ["setup", "parity"])
def test_bench_checkpoints_precede_its_collectives(tag):
    """bench.py calls each checkpoint before the collective it guards."""
    src = open(bench.__file__).read()
    assert f'rank_checkpoint("{tag}")' in src
