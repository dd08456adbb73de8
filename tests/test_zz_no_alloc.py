"""The allocation-free entry point (``h3_linear_gated_residual_rms_modulate_noalloc``)
against the regular one that takes a caller-owned workspace.

Why it exists: some callers of this library cannot allocate device memory at the
point where they call it -- a host framework that owns every device allocation
through its own pool and hands out only the tensors it has planned, or a plugin
boundary whose host side has no device allocator at all.  For them the scratch
of the fused out-projection + RMSNorm/AdaLN (the per-tile sums of squares that
pass from the projection's epilogue to the norm pass) lives in a fixed array in
the library's device image instead of a workspace argument.

Checked through the C-ABI (ctypes), on two calls in a row with different inputs
(the array keeps the previous call's contents, so the second call must not see
them): outputs bitwise equal to the workspace entry point's (the same kernels
and the same arithmetic; tolerance 0).  Requests beyond the array's capacity are
refused with H3_ERR_TOO_LARGE.  Collected last so that a failure here comes
after every other test of a run that stops at the first failure.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
H3_ERR_TOO_LARGE = 10


def _case(m, n, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    r = lambda *s, std=1.0: (torch.randn(*s, generator=g, device=DEV) * std).bfloat16()  # noqa: E731
    return dict(x=r(m, k), w=r(n, k, std=0.02), residual=r(m, n), gate=r(n, std=0.5).expand(m, n),
                weight=(r(n, std=0.1).float() + 1).bfloat16(), scale=r(n, std=0.1).expand(m, n),
                shift=r(n, std=0.1).expand(m, n))


def _descs(c, residual_out, out):
    from h3b200 import _lib
    names = ("x", "w", "residual", "gate", "weight", "scale", "shift")
    return [_lib.desc(residual_out), _lib.desc(out)] + [_lib.desc(c[n]) for n in names]


def _run(entry, c, workspace=None):
    from h3b200 import _lib
    m, n = c["residual"].shape
    residual_out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    d = _descs(c, residual_out, out)
    args = [ctypes.byref(t) for t in d[:9]] + [ctypes.c_float(1e-6)]
    if workspace is not None:
        args.append(ctypes.byref(_lib.desc(workspace)))
    args.append(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    status = getattr(_lib.load(), entry)(*args)
    return status, residual_out, out


@pytest.mark.parametrize("m,n,k", [(2048, 5120, 1024), (777, 1792, 512)])
def test_noalloc_equals_workspace_entry_point_twice(m, n, k):
    import h3b200
    lib = h3b200.load()
    for call, seed in enumerate((1, 2)):
        c = _case(m, n, k, seed + m)
        ws = torch.empty(m, (n + 255) // 256, dtype=torch.float32, device=DEV)
        s_ref, r_ref, o_ref = _run("h3_linear_gated_residual_rms_modulate", c, ws)
        s_new, r_new, o_new = _run("h3_linear_gated_residual_rms_modulate_noalloc", c)
        torch.cuda.synchronize()
        assert s_ref == 0 and s_new == 0, (s_ref, s_new)
        assert torch.equal(r_new, r_ref), f"call {call + 1}: residual differs"
        assert torch.equal(o_new, o_ref), f"call {call + 1}: normalised output differs"
    assert lib.h3_device_error() == 0


def test_noalloc_refuses_requests_beyond_its_scratch():
    import h3b200
    lib = h3b200.load()
    from h3b200 import _lib
    # 16 tiles of 256 columns per row: the 1 Mi-float array holds 65536 such rows, one more is refused
    rows = (1 << 20) // 16 + 1
    out = torch.empty(rows, 4096, dtype=torch.bfloat16, device=DEV)
    x = torch.empty(rows, 64, dtype=torch.bfloat16, device=DEV)
    w = torch.empty(4096, 64, dtype=torch.bfloat16, device=DEV)
    vec = torch.empty(4096, dtype=torch.bfloat16, device=DEV)
    row = vec.expand(rows, 4096)
    args = [ctypes.byref(_lib.desc(t)) for t in (out, out, x, w, out, row, vec, row, row)]
    status = lib.h3_linear_gated_residual_rms_modulate_noalloc(*args, ctypes.c_float(1e-6),
                                                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == H3_ERR_TOO_LARGE
    assert lib.h3_status_string(status).decode().startswith("request exceeds")
    assert lib.h3_device_error() == 0
