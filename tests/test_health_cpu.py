"""Host-side failure detection on CPU ranks (gloo): a collective whose peer is
late raises ``CollectiveTimeout`` within its bound instead of blocking; an
on-time collective completes with the right result.  No GPU is involved."""
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, path, late_s):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    from h3b200.health import CollectiveTimeout, bounded_collective
    if rank == 1 and late_s:
        time.sleep(late_s)
    local = torch.full((4,), float(rank + 1))
    out = torch.empty(8)
    t0 = time.monotonic()
    outcome = "ok"
    try:
        bounded_collective(lambda: dist.all_gather_into_tensor(out, local, async_op=True), "test all-gather",
                           timeout_s=0.5)
    except CollectiveTimeout:
        outcome = "timeout"
    elapsed = time.monotonic() - t0
    dist.barrier()            # the late rank's all-gather completes before this (ops run in order)
    with open(f"{path}.{rank}", "w") as f:
        f.write(f"{outcome} {elapsed:.3f} {out.tolist() if outcome == 'ok' else ''}")
    dist.destroy_process_group()


def _run(tmp_path, late_s):
    path = str(tmp_path / "h")
    mp.start_processes(_worker, args=(_free_port(), path, late_s), nprocs=2, start_method="spawn")
    return [open(f"{path}.{r}").read().split(" ", 2) for r in range(2)]


def test_late_peer_raises_within_bound(tmp_path):
    res = _run(tmp_path, late_s=3.0)
    outcome, elapsed, _ = res[0]
    assert outcome == "timeout", "rank 0 should report the late peer"
    assert float(elapsed) < 2.0, f"rank 0 waited {elapsed} s, beyond its 0.5 s bound"


def test_on_time_collective_completes(tmp_path):
    res = _run(tmp_path, late_s=0.0)
    for outcome, _, values in res:
        assert outcome == "ok"
        assert values.strip() == str([1.0] * 4 + [2.0] * 4)


def _worker_gone(rank, port, path):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=30))
    from h3b200.health import CollectiveTimeout, bounded_collective, shutdown_group
    if rank == 1:             # a rank that never joins the collective and leaves
        time.sleep(1.0)
        os._exit(0)
    local = torch.ones(4)
    out = torch.empty(8)
    outcome = "ok"
    try:
        bounded_collective(lambda: dist.all_gather_into_tensor(out, local, async_op=True), "test all-gather",
                           timeout_s=0.5)
    except CollectiveTimeout:
        outcome = "timeout"
    t0 = time.monotonic()
    shutdown_group()          # the survivor tears the group down instead of waiting on it
    with open(f"{path}.0", "w") as f:
        f.write(f"{outcome} {time.monotonic() - t0:.3f} {dist.is_initialized()}")


def test_survivor_shuts_the_group_down(tmp_path):
    """A rank that never joins: the survivor's bounded wait raises, and
    ``shutdown_group`` then tears the process group down without blocking."""
    path = str(tmp_path / "g")
    mp.start_processes(_worker_gone, args=(_free_port(), path), nprocs=2, start_method="spawn")
    outcome, shut_s, initialized = open(f"{path}.0").read().split()
    assert outcome == "timeout"
    assert float(shut_s) < 20.0
    assert initialized == "False"
