"""Host logic of the multi-GPU sharding layer, on CPU with gloo (world_size 2).

The per-rank compute here is the CPU oracle (test infrastructure); what is under test is the
product's sharding: the head slices of ``qwen_tp_weights`` plus a SUM all-reduce must give
the unsharded block, and the stats -> MAX all-reduce -> apply protocol of the row-sharded
norm must give the single-device per-tensor scale.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from b200fp8 import sharding
from helpers import gen, randn
from oracle import blocks as ob
from oracle import norm as onorm
from oracle.attention import rope_tables


def test_split_range_and_plans():
    assert [sharding.split_range(10, 3, i) for i in range(3)] == [(0, 3), (3, 6), (6, 10)]
    assert sharding.plan_block_parallel(1, 4, 32, 8) == (1, 1)
    assert sharding.plan_block_parallel(4, 4, 32, 8) == (4, 1)
    assert sharding.plan_block_parallel(8, 4, 32, 8) == (4, 2)
    assert sharding.plan_block_parallel(8, 4, 32, 8, tp=8) == (1, 8)
    with pytest.raises(ValueError):
        sharding.plan_block_parallel(8, 4, 32, 8, tp=16)
    t = torch.arange(10).view(10, 1)
    parts = [sharding.shard_rows(t, r, 3, align=2) for r in range(3)]
    assert torch.equal(torch.cat(parts), t)
    assert all(p.shape[0] % 2 == 0 for p in parts[:-1])


def _qwen_weights(interleaved, hidden=256, heads=4, kv_heads=2, d=64, seq=32):
    g = gen(5)
    q8 = lambda shape: (randn(shape, g) * 0.05 / 0.05 * 448 / 4).clamp(-448, 448).to(
        torch.float8_e4m3fn)  # noqa: E731
    cos, sin = rope_tables(seq, d, 1e6)
    qrows = 2 * heads * d if interleaved else heads * d
    return ob.QwenWeights(
        q8((qrows, hidden)), 1 / 2048, None if interleaved else q8((heads * d, hidden)), 1 / 2048,
        q8((kv_heads * d, hidden)), 1 / 2048, q8((kv_heads * d, hidden)), 1 / 2048,
        q8((hidden, heads * d)), 1 / 4096, randn((hidden,), g, 0.02), randn((d,), g, 0.02),
        randn((d,), g, 0.02), cos, sin, heads, kv_heads, d, d, interleaved=interleaved)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, interleaved, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        batch, seq, hidden = 2, 32, 256
        w = _qwen_weights(interleaved)
        x = randn((batch * seq, hidden), gen(11))
        # heads-parallel block: local heads, residual only on the first rank
        local = sharding.qwen_tp_weights(w, rank, world)
        out = ob.qwen_block(x, local, batch=batch)
        part = out if rank == 0 else out - x
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
        full = ob.qwen_block(x, w, batch=batch)
        err_block = float((part - full).abs().max())
        # row-sharded norm: stats -> MAX all-reduce -> apply
        xs = randn((64, 512), gen(21)).to(torch.bfloat16)
        rs = randn((64, 512), gen(22)).to(torch.bfloat16)
        gamma = (1 + randn((512,), gen(23), 0.02)).to(torch.bfloat16)
        lo, hi = sharding.split_range(64, world, rank)
        _, y = onorm.residual_norm(xs[lo:hi], gamma, residual=rs[lo:hi], h_dtype=torch.bfloat16)
        y = y.to(torch.bfloat16).float()
        amax = y.abs().max().reshape(1)
        dist.all_reduce(amax, op=dist.ReduceOp.MAX)
        s = float(amax) / 448.0
        q_local = (y / s).to(torch.float8_e4m3fn).view(torch.uint8)
        qs = [torch.empty_like(q_local) for _ in range(world)]
        dist.all_gather(qs, q_local)
        q_ref, s_ref, _ = onorm.residual_rmsnorm_amax_quant(xs, rs, gamma)
        ok_norm = s == s_ref and torch.equal(torch.cat(qs), q_ref.view(torch.uint8))
        q.put((rank, err_block, ok_norm, local.heads, local.kv_heads))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("interleaved", [False, True])
def test_heads_parallel_qwen_and_row_sharded_norm_gloo(interleaved):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, interleaved, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, ok_norm, h, hk in results:
        assert (h, hk) == (2, 1)
        assert err < 1e-4, err
        assert ok_norm


def _fault_worker(rank, world, port, q):
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            # this rank fails on the host before the row-sharded norm's MAX all-reduce
            q.put((rank, "raised"))
            raise RuntimeError("injected host-side failure")
        amax = torch.tensor([1.0])
        t0 = time.time()
        try:
            dist.all_reduce(amax, op=dist.ReduceOp.MAX)
            q.put((rank, "completed"))
        except Exception as exc:  # the collective must fail, not hang
            q.put((rank, f"error after {time.time() - t0:.1f}s: {type(exc).__name__}"))
    except RuntimeError:
        pass
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_failed_rank_surfaces_as_collective_error_gloo():
    """A rank that dies before the amax all-reduce makes the surviving rank's collective
    fail within the process-group timeout (host-side failure detection; no GPU involved)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert results[1] == "raised"
    assert results[0].startswith("error after"), results[0]
    assert float(results[0].split()[2].rstrip("s:")) < 60
