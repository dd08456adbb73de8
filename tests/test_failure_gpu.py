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
