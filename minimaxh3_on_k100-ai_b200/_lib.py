"""ctypes bridge to ``libh3b200.so`` (the C-ABI declared in include/h3_b200.h).

The library is loaded once.  If it is missing, every op raises: there is no
fallback implementation of any op.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libh3b200.so"

H3_OK = 0
_STATUS = {
    1: "null descriptor or data pointer",
    2: "bad shape",
    3: "bad dtype",
    4: "bad layout (strides/alignment)",
    5: "unsupported configuration",
    6: "CUDA launch error",
    7: "driver entry point unavailable",
    8: "bounded device wait timed out",
    9: "row index outside the indexed tensor",
    10: "request exceeds the library's static scratch capacity",
}
_DTYPES = {torch.bfloat16: 0, torch.float32: 1, torch.float64: 2, torch.int64: 3}


class H3Tensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("shape", ctypes.c_int64 * 4),
        ("strides", ctypes.c_int64 * 4),
        ("ndim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


P = ctypes.POINTER(H3Tensor)
_F = ctypes.c_float
_V = ctypes.c_void_p
_I = ctypes.c_int32

# name -> argtypes (every entry point returns int)
SIGNATURES = {
    "h3_abi_version": [],
    "h3_status_string": [ctypes.c_int],
    "h3_device_error": [],
    "h3_selftest_wait_timeout": [ctypes.c_uint64, _V],
    "h3_gemm_variant": [ctypes.c_int],
    "h3_adaln_projection": [P, P, P, P, _V],
    "h3_rms_norm": [P, P, P, _F, _V],
    "h3_swiglu": [P, P, P, _V],
    "h3_rms_modulate": [P, P, P, P, P, _F, _V],
    "h3_ln_modulate": [P, P, P, P, _F, _V],
    "h3_gated_residual": [P, P, P, P, _V],
    "h3_gated_residual_rms_modulate": [P, P, P, P, P, P, P, P, _F, _V],
    "h3_rope": [P, P, P, P, _V],
    "h3_qk_norm_rope": [P, P, P, P, P, _F, _V],
    "h3_rope_cache": [P, P, P, _V],
    "h3_rope_cache_sectioned": [P, P, P, _I, _I, _I, _V],
    "h3_timestep_embedding": [P, P, _F, _V],
    "h3_mha": [P, P, P, P, _F, _V],
    "h3_mha_scatter": [P, _I, P, P, P, _F, _V],
    "h3_linear": [P, P, P, _V],
    "h3_linear_swiglu": [P, P, P, _V],
    "h3_linear_gated_residual": [P, P, P, P, P, _V],
    "h3_linear_gated_residual_sq": [P, P, P, P, P, P, _V],
    "h3_rms_modulate_sq": [P, P, P, P, P, P, _F, _V],
    "h3_linear_gated_residual_segmented": [P, P, P, P, P, P, ctypes.POINTER(ctypes.c_int64), _I, _V],
    "h3_rms_modulate_segmented": [P, P, P, P, P, P, ctypes.POINTER(ctypes.c_int64), _I, _F, _V],
    "h3_linear_gated_residual_rms_modulate": [P, P, P, P, P, P, P, P, P, _F, P, _V],
    "h3_linear_gated_residual_rms_modulate_noalloc": [P, P, P, P, P, P, P, P, P, _F, _V],
    "h3_pack_gate_up": [P, P, _V],
    "h3_linear_qkv_norm_rope": [P, P, P, P, P, _I, P, P, P, P, _F, _V],
    "h3_linear_f32": [P, P, P, P, _V],
    "h3_gather_rows": [P, P, P, _V],
    "h3_index_copy_rows": [P, P, P, _V],
    "h3_silu": [P, P, _V],
    "h3_qk_norm_rope_multi": [P, _I, P, P, P, P, _F, _V],
    "h3_copy_blocks": [P, _I, P, _V],
    "h3_peer_reduce_rows": [P, P, _I, _V],
    "h3_ipc_alloc": [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p],
    "h3_ipc_open": [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)],
    "h3_ipc_close": [ctypes.c_void_p],
    "h3_ipc_free": [ctypes.c_void_p],
    "h3_exchange_signal": [ctypes.POINTER(ctypes.c_void_p), _V, _I, _I, _I, _V],
    "h3_exchange_wait": [_V, _V, _I, _I, _I, ctypes.c_uint64, _V],
}

_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build() "
                               "(nvcc, sm_100a). There is no fallback implementation.")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_char_p if name == "h3_status_string" else ctypes.c_int
        _lib = lib
    return _lib


def desc(t: torch.Tensor | None) -> H3Tensor | None:
    if t is None:
        return None
    if t.dim() > 4:
        raise ValueError(f"at most 4 dims supported, got {t.dim()}")
    d = H3Tensor()
    d.data = t.data_ptr()
    for i in range(t.dim()):
        d.shape[i] = t.shape[i]
        d.strides[i] = t.stride(i)
    d.ndim = t.dim()
    try:
        d.dtype = _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None
    return d


def ref(d: H3Tensor | None):
    return None if d is None else ctypes.byref(d)


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def check(status: int, op: str) -> None:
    if status == H3_OK:
        return
    msg = f"{op}: {_STATUS.get(status, f'status {status}')}"
    if status in (2, 3, 4):
        raise ValueError(msg)
    raise RuntimeError(msg)


# Number of C-ABI entry-point calls made (each launches exactly one kernel, or
# none for an empty input); bench.py reads it to count its kernel launches.
CALLS = {"n": 0}


def call(name: str, *args) -> None:
    lib = load()
    conv = [ctypes.byref(a) if isinstance(a, H3Tensor) else a for a in args]
    CALLS["n"] += 1
    check(getattr(lib, name)(*conv), name)


def check_device(where: str) -> None:
    """Synchronise the current device and raise if a bounded device-side wait gave
    up (a peer that never signalled, an mbarrier that never completed), a row index
    was out of range, or the device reported an error since the last check.  The
    kernels that hit such a condition return normally and leave their outputs
    incomplete, so every public entry point that hands results back checks here."""
    check(load().h3_device_error(), f"{where} (device status)")


def require_cuda(*tensors: torch.Tensor) -> None:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("H3 ops take CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same device")
    if dev is not None and dev.index != torch.cuda.current_device():
        raise ValueError(f"tensors on {dev} but the current device is cuda:{torch.cuda.current_device()}; "
                         "call under torch.cuda.device(...)")


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def library_path() -> str:
    return os.fspath(LIB_PATH)
