"""Gloo tests (world sizes 2 and 4) of the Ulysses exchange logic on CPU.

The same host code as the GPU path (``SequenceParallel.attention_from_qkv``)
runs on gloo ranks with the CPU oracle standing in for the three device ops.  Checks: the received blocks are exactly the global-order q/k/v of the
rank's heads (integer layout, bit-exact), and the per-rank outputs, gathered,
match single-rank attention over the whole sequence (sequence padding included).
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import h3_oracle as O

HEADS, D, SEQ, WORLD = 4, 128, 9, 2     # 9 tokens -> T = 5, one padded row (world 4: T = 3, three)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(heads=HEADS):
    torch.manual_seed(0)
    x = torch.randn(SEQ, heads * D).bfloat16()
    w_qkv = (torch.randn(3 * heads * D, heads * D) * 0.05).bfloat16()
    wq = (torch.randn(D) * 0.1 + 1).bfloat16()
    wk = (torch.randn(D) * 0.1 + 1).bfloat16()
    table = O.rotary_cache(O.grid_positions(1, 3, 3))
    return x, w_qkv, wq, wk, table[:, :48], table[:, 48:]


def _oracle_kernels():
    import h3b200.ulysses as U
    return U.Kernels(
        linear=lambda out, x, w: out.copy_(O.linear(x, w)),
        qk_norm_rope=lambda out, x, w, cos, sin, eps: out.copy_(O.qk_norm_rope(x, w, cos, sin, eps)),
        mha=lambda out, q, k, v, scale: out.copy_(O.attention_fp32(q, k, v, scale).bfloat16()))


def _single_rank_reference(heads=HEADS):
    x, w_qkv, wq, wk, cos, sin = _inputs(heads)
    parts = O.linear(x, w_qkv).view(SEQ, 3, heads, D)
    q = O.qk_norm_rope(parts[:, 0], wq, cos, sin, 1e-6)
    k = O.qk_norm_rope(parts[:, 1], wk, cos, sin, 1e-6)
    v = parts[:, 2]
    out = O.attention_fp32(q[None], k[None], v[None], D ** -0.5)[0].bfloat16()
    return q, k, v, out.reshape(SEQ, heads * D)


def _worker(rank, port, result_path, world, heads):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import h3b200.ulysses as U
    t, start, padded = U.local_rows(SEQ, world, rank)
    x, w_qkv, wq, wk, cos, sin = _inputs(heads)
    pad = torch.zeros(padded - SEQ, x.shape[1], dtype=x.dtype)
    x_p = torch.cat([x, pad])
    cos_p = torch.cat([cos, cos[:1].expand(padded - SEQ, -1)])     # padded rows reuse row 0
    sin_p = torch.cat([sin, sin[:1].expand(padded - SEQ, -1)])
    rows = slice(start, start + t)
    sp = U.SequenceParallel(world, rank, None, SEQ, t, heads, D, "cpu", kernels=_oracle_kernels(), groups=2)
    out = sp.attention(x_p[rows].contiguous(), w_qkv, wq, wk, cos_p[rows], sin_p[rows], 1e-6)
    torch.save({"out": out.clone(), "groups": sp.group_heads,
                "recv": [[r.clone() for r in grp] for grp in sp.recv]}, f"{result_path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,heads", [(2, 4), (4, 8)])
def test_ulysses_matches_single_rank(tmp_path, world, heads):
    port = _free_port()
    path = str(tmp_path / "res")
    mp.start_processes(_worker, args=(port, path, world, heads), nprocs=world, start_method="spawn")
    q, k, v, ref = _single_rank_reference(heads)
    t = (SEQ + world - 1) // world
    hl = heads // world
    outs = []
    for rank in range(world):
        res = torch.load(f"{path}.{rank}")
        outs.append(res["out"])
        # received blocks = this rank's heads of each group over the global token
        # order (bit-exact integer layout)
        off = 0
        for hs, grp in zip(res["groups"], res["recv"]):
            heads = slice(rank * hl + off, rank * hl + off + hs)
            for got, full in zip(grp, (q, k, v)):
                glob = got.reshape(world * t, hs, D)[:SEQ]
                assert torch.equal(glob, full[:, heads])
            off += hs
    gathered = torch.cat(outs)[:SEQ]
    assert O.max_abs_rel(gathered, ref) <= 1e-2


def _dropout_worker(rank, port, result_path):
    """Rank 1 leaves between steps (before the exchange); rank 0 must get an
    error from its collective within the process-group timeout, not hang."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=5))
    import h3b200.ulysses as U
    if rank == 1:
        dist.destroy_process_group()
        return
    t, start, padded = U.local_rows(SEQ, WORLD, rank)
    x, w_qkv, wq, wk, cos, sin = _inputs()
    sp = U.SequenceParallel(WORLD, rank, None, SEQ, t, HEADS, D, "cpu", kernels=_oracle_kernels())
    outcome = "no error"
    try:
        sp.attention(x[:t].contiguous(), w_qkv, wq, wk, cos[:t], sin[:t], 1e-6)
    except Exception as exc:  # noqa: BLE001 - any collective error is the expected outcome
        outcome = f"error: {type(exc).__name__}"
    with open(result_path, "w") as f:
        f.write(outcome)


def test_ulysses_dropped_rank_reports_error(tmp_path):
    port = _free_port()
    path = str(tmp_path / "dropout")
    ctx = mp.start_processes(_dropout_worker, args=(port, path), nprocs=WORLD, start_method="spawn",
                             join=False)
    deadline = 120
    import time
    t0 = time.time()
    while not ctx.join(timeout=5):
        assert time.time() - t0 < deadline, "a rank hung instead of reporting the dropped peer"
    with open(path) as f:
        assert f.read().startswith("error")
