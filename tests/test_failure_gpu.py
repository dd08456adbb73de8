"""Failure detection on the GPU without a fault: a bounded device wait that
nothing satisfies gives up after its limit, the kernel ends, the host reads
H3_ERR_TIMEOUT, and the context keeps working."""
import pytest
import torch

pytestmark = pytest.mark.gpu

H3_ERR_TIMEOUT = 8


def test_bounded_wait_expires_and_reports():
    import h3b200
    lib = h3b200.load()
    assert lib.h3_device_error() == 0
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.h3_selftest_wait_timeout(20_000_000, stream) == 0      # 20 ms limit
    assert lib.h3_device_error() == H3_ERR_TIMEOUT
    assert lib.h3_device_error() == 0                                  # cleared by the read
    x = torch.randn(64, 256, dtype=torch.bfloat16, device="cuda")      # context still usable
    out = h3b200.h3_gated_residual(x, torch.zeros_like(x), x)
    assert torch.equal(out, x)


def test_selftest_rejects_unbounded_limit():
    import h3b200
    lib = h3b200.load()
    assert lib.h3_selftest_wait_timeout(0, None) != 0
    assert lib.h3_selftest_wait_timeout(5_000_000_000, None) != 0


def test_exchange_wait_for_a_silent_peer_times_out():
    """The Ulysses peer exchange on one GPU with a fake second rank that never
    signals: this rank's signal succeeds, its wait for rank 1 gives up after
    50 ms, the host reads H3_ERR_TIMEOUT and the context keeps working."""
    import ctypes
    import h3b200
    lib = h3b200.load()
    assert lib.h3_device_error() == 0
    ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
    assert lib.h3_ipc_alloc(4096, ctypes.byref(ptr), handle) == 0
    try:
        # both ranks' flag arrays are this one allocation: rank 0's signal lands in
        # flags[slot][0]; nothing ever writes flags[slot][1]
        peers = (ctypes.c_void_p * 2)(ptr.value, ptr.value)
        epoch = torch.zeros(4, dtype=torch.int64, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        ep = ctypes.c_void_p(epoch.data_ptr())
        assert lib.h3_exchange_signal(peers, ep, 1, 0, 2, stream) == 0
        assert lib.h3_exchange_wait(ptr, ep, 1, 0, 2, 50_000_000, stream) == 0
        assert lib.h3_device_error() == H3_ERR_TIMEOUT
        assert int(epoch[1]) == 1
        # a peer that did signal: write rank 1's flag by hand, the next wait passes
        flags = torch.zeros(4 * 8, dtype=torch.int64, device="cuda")
        flags[1 * 8 + 1] = 5
        assert lib.h3_exchange_wait(ctypes.c_void_p(flags.data_ptr()), ep, 1, 0, 2, 50_000_000, stream) == 0
        assert lib.h3_device_error() == 0
        # argument checks
        assert lib.h3_exchange_wait(ptr, ep, 1, 0, 2, 0, stream) != 0          # unbounded wait refused
        assert lib.h3_exchange_wait(ptr, ep, 4, 0, 2, 1000, stream) != 0       # slot out of range
        assert lib.h3_exchange_signal(peers, ep, 0, 2, 2, stream) != 0         # rank out of range
        x = torch.randn(64, 256, dtype=torch.bfloat16, device="cuda")
        assert torch.equal(h3b200.h3_gated_residual(x, torch.zeros_like(x), x), x)
    finally:
        torch.cuda.synchronize()
        assert lib.h3_ipc_free(ptr) == 0


def test_bounded_host_sync_reports_slow_device_work():
    """The host-side bound on a stream synchronisation: device work that outlasts
    the bound (here a self-test wait of 300 ms, which itself ends by its own
    limit) raises DeviceTimeout after ~50 ms instead of blocking the host; a
    generous bound then succeeds and the device reports the self-test's expiry."""
    import time

    import h3b200
    from h3b200.health import DeviceTimeout, bounded_sync
    lib = h3b200.load()
    assert lib.h3_device_error() == 0
    stream = torch.cuda.current_stream()
    assert lib.h3_selftest_wait_timeout(300_000_000, stream.cuda_stream) == 0
    t0 = time.monotonic()
    with pytest.raises(DeviceTimeout):
        bounded_sync(stream, timeout_s=0.05, what="self-test")
    assert time.monotonic() - t0 < 0.25
    bounded_sync(stream, timeout_s=10.0, what="self-test")
    assert lib.h3_device_error() == H3_ERR_TIMEOUT
