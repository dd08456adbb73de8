"""Host-side failure detection for the multi-GPU step: bounded waits on
collectives and on the device, so a rank that is late or gone turns into an
error on the others instead of a hang.

The reference synchronises its rank threads with an unbounded spin barrier
(``SpinBarrier``, patches/InfiniLM.patch:303-324) and NCCL calls that wait as
long as the library lets them.  Here:

* ``bounded_collective`` starts a torch.distributed collective asynchronously
  and polls its completion (for NCCL: the communicator's completion event, the
  same state torch's watchdog checks with ``ncclCommGetAsyncError``) in a host
  loop with a deadline; past the deadline it raises ``CollectiveTimeout``
  naming the collective, and the caller shuts the group down.
* ``bounded_sync`` replaces a blocking stream synchronisation: it records an
  event and polls it with a deadline (``DeviceTimeout``), e.g. after replaying a
  CUDA graph that holds collectives or peer-exchange waits.

Device-side waits (the peer-exchange flags, the kernels' mbarriers) have their
own bounds and report through ``h3_device_error()``; these two cover the host.
"""
from __future__ import annotations

import time

import torch


class CollectiveTimeout(RuntimeError):
    """A collective did not complete within its deadline (a peer is late or gone)."""


class DeviceTimeout(RuntimeError):
    """Work queued on a stream did not complete within its deadline."""


def _poll(done, timeout_s: float, poll_s: float) -> bool:
    deadline = time.monotonic() + timeout_s
    while not done():
        if time.monotonic() > deadline:
            return False
        time.sleep(poll_s)
    return True


def bounded_collective(start, what: str, timeout_s: float = 60.0, poll_s: float = 0.0005):
    """Run ``start()`` -- a torch.distributed call made with ``async_op=True``
    that returns its work handle -- and wait for it at most ``timeout_s``."""
    work = start()
    if work is None:
        return None
    if not _poll(work.is_completed, timeout_s, poll_s):
        raise CollectiveTimeout(f"{what}: not complete after {timeout_s:.3g} s (a peer rank is late or gone)")
    work.wait()
    return work


def bounded_sync(stream: torch.cuda.Stream | None = None, timeout_s: float = 60.0, what: str = "stream",
                 poll_s: float = 0.0002) -> None:
    """Wait for the work queued so far on ``stream`` (default: current) for at
    most ``timeout_s``."""
    ev = torch.cuda.Event()
    ev.record(stream)
    if not _poll(ev.query, timeout_s, poll_s):
        raise DeviceTimeout(f"{what}: device work not complete after {timeout_s:.3g} s")


def shutdown_group(group=None) -> None:
    """Best-effort teardown of a process group after a timeout: abort it where the
    backend supports that (NCCL), else destroy it."""
    import torch.distributed as dist
    abort = getattr(dist.distributed_c10d, "_abort_process_group", None)
    try:
        if abort is not None and dist.get_backend(group) == "nccl":
            abort(group)
        else:
            dist.destroy_process_group(group)
    except Exception:  # noqa: BLE001 - teardown after a failure is best effort
        pass
