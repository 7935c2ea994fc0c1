"""Multi-GPU sharding of the hot path: one process per GPU, torch.distributed over NCCL.

Work is split only where it shards naturally:

- GEMMs: along N (``shard_rows`` of B [N, K], its bias and per-column scales).  A is
  replicated, every rank writes its own column block, no communication.
- Residual + RMSNorm + per-tensor amax quantisation: rows.  Each rank runs pass 1 on its
  rows (h and the local amax), one MAX all-reduce of a single f32 gives the global amax,
  then each rank runs pass 2 with that scale (``RowShardedNorm``).
- GPT-2 block: batch (whole sequences per rank), no communication.
- Qwen gated-attention block: heads.  The q / gate / k / v projections are column-parallel
  (each rank owns heads [h0, h1) and their KV groups), the o-projection row-parallel; the
  rank that owns the first heads adds the residual, the partial outputs are summed by one
  all-reduce (``QwenBlockTP``).  ``plan_block_parallel`` combines batch and head groups
  (for example 4 sequences on 8 GPUs: 4 batch groups x 2-way heads).

Reference: the reference runs every task on one GPU (its evaluators, e.g.
tasks/model_qwen35_4b_full_attention_block_fp8/starter.py, have no multi-GPU path); the
head split follows the block's own per-head structure (GQA group g = h / (hq / hkv)).
"""
from __future__ import annotations

import math
from types import SimpleNamespace
from typing import Optional, Tuple

import torch

from . import blocks, ops


def split_range(n: int, parts: int, i: int) -> Tuple[int, int]:
    """[lo, hi) of part i when n items are split into contiguous, near-equal parts."""
    if parts <= 0 or not 0 <= i < parts:
        raise ValueError("bad split")
    return n * i // parts, n * (i + 1) // parts


def shard_rows(t: Optional[torch.Tensor], rank: int, world: int, align: int = 1):
    """Rows [lo, hi) of t for this rank (contiguous copy); row counts are multiples of
    ``align`` except possibly the last rank's."""
    if t is None:
        return None
    units = math.ceil(t.shape[0] / align)
    lo, hi = split_range(units, world, rank)
    return t[lo * align:min(hi * align, t.shape[0])].contiguous()


def plan_block_parallel(world: int, batch: int, heads: int, kv_heads: int,
                        tp: Optional[int] = None) -> Tuple[int, int]:
    """(dp, tp) with dp * tp == world: as many whole-sequence groups as the batch allows
    (no communication), the rest split by heads.  ``tp`` forces the head split."""
    if tp is None:
        dp = math.gcd(world, batch)
        tp = world // dp
    if world % tp or batch % (world // tp):
        raise ValueError(f"cannot split batch {batch} x {world} GPUs with tp={tp}")
    if kv_heads % tp or heads % tp:
        raise ValueError(f"tp={tp} must divide heads {heads} and kv heads {kv_heads}")
    return world // tp, tp


def tp_groups(world: int, tp: int):
    """Create (every rank must call this) the head-parallel process groups: ranks
    [d*tp, (d+1)*tp) form group d.  Returns (dp_index, tp_rank, this rank's group)."""
    import torch.distributed as dist
    rank = dist.get_rank()
    mine = None
    for d in range(world // tp):
        ranks = list(range(d * tp, (d + 1) * tp))
        g = dist.new_group(ranks) if tp > 1 else None
        if rank in ranks:
            mine = g
    return rank // tp, rank % tp, mine


class RowShardedNorm:
    """Residual + RMSNorm/LayerNorm + per-tensor amax e4m3 quantisation over row shards:
    pass 1 per rank, MAX all-reduce of the amax, pass 2 per rank.  Every rank ends with the
    same scale as a single-device run over all rows, and the same bits in its rows."""

    def __init__(self, group=None):
        self.group = group
        self._stats = None  # per-row (mean, rstd) handed from the stats to the apply phase

    def __call__(self, x, weight, *, residual=None, h_out=None, q_out=None, kind="rms",
                 bias=None, weight_offset=0.0, eps=1e-6, amax=None, scale_out=None):
        import torch.distributed as dist
        if h_out is None:
            raise ValueError("row-sharded pass 2 re-reads h: pass h_out")
        dev = x.device
        amax = torch.zeros(1, device=dev) if amax is None else amax
        scale_out = torch.empty(1, device=dev) if scale_out is None else scale_out
        if self._stats is None or self._stats.numel() < 2 * x.shape[0]:
            self._stats = torch.empty((2 * x.shape[0],), dtype=torch.float32, device=dev)
        common = dict(kind=kind, bias=bias, weight_offset=weight_offset, eps=eps,
                      residual=residual, h_out=h_out, q_out=q_out, amax=amax,
                      row_stats=self._stats)
        q_out, _ = ops.norm_quant(x, weight, phase="stats", **common)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
        common["q_out"] = q_out
        return ops.norm_quant(x, weight, phase="apply", scale_out=scale_out, **common)


def qwen_tp_weights(w, tp_rank: int, tp: int):
    """This rank's slice of a Qwen block's weights for a ``tp``-way head split: query heads
    [h0, h1) with their gate rows, KV heads [g0, g1) (the GQA groups those query heads
    read), o-projection input columns of heads [h0, h1).  Norm weights and RoPE tables are
    shared."""
    h, hk, d = w.heads, w.kv_heads, w.head_dim
    if h % tp or hk % tp:
        raise ValueError("tp must divide the query and KV head counts")
    if getattr(w, "mlp_down_w", None) is not None:
        raise ValueError("the heads-parallel block covers the attention block without MLP")
    h0, h1 = split_range(h, tp, tp_rank)
    g0, g1 = split_range(hk, tp, tp_rank)
    out = SimpleNamespace(**vars(w)) if not hasattr(w, "__dataclass_fields__") else \
        SimpleNamespace(**{k: getattr(w, k) for k in w.__dataclass_fields__})
    for k in ("post_norm_w", "mlp_gate_w", "mlp_up_w", "mlp_down_w"):
        if not hasattr(out, k):
            setattr(out, k, None)
    rows = lambda t, a, b: t[a * d:b * d].contiguous()  # noqa: E731
    if w.interleaved:  # [q_h | gate_h] pairs of rows per head
        out.q_w = w.q_w[2 * h0 * d:2 * h1 * d].contiguous()
    else:
        out.q_w = rows(w.q_w, h0, h1)
        out.gate_w = rows(w.gate_w, h0, h1)
    out.k_w = rows(w.k_w, g0, g1)
    out.v_w = rows(w.v_w, g0, g1)
    out.o_w = w.o_w[:, h0 * d:h1 * d].contiguous()
    out.heads, out.kv_heads = h1 - h0, g1 - g0
    return out


class QwenBlockTP:
    """Heads-parallel Qwen gated-attention block: column-parallel q / gate / k / v,
    row-parallel o-projection, one all-reduce (sum) of the [T, hidden] output over the
    head group.  The group's first rank adds the residual inside its o-projection
    epilogue.  ``replay`` runs the captured local block, then the all-reduce."""

    def __init__(self, w, *, batch: int, seq: int, group, tp_rank: int, tp: int,
                 residual_dtype=torch.bfloat16, out_dtype=torch.bfloat16, device="cuda"):
        self.group, self.tp_rank, self.tp = group, tp_rank, tp
        local = qwen_tp_weights(w, tp_rank, tp)
        self.blk = blocks.QwenBlock(local, batch=batch, seq=seq, residual_dtype=residual_dtype,
                                    out_dtype=out_dtype, device=device,
                                    add_residual=(tp_rank == 0))
        self.launches_per_forward = 7

    def flops(self) -> float:
        return self.blk.flops()

    def _reduce(self, out: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            import torch.distributed as dist
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
        return out

    def forward(self, hidden: torch.Tensor, hidden_scale: float = 1.0) -> torch.Tensor:
        return self._reduce(self.blk.forward(hidden, hidden_scale))

    def capture(self, hidden: torch.Tensor, hidden_scale: float = 1.0) -> torch.Tensor:
        return self.blk.capture(hidden, hidden_scale)

    @property
    def graph_input(self) -> torch.Tensor:
        return self.blk.graph_input

    def replay(self) -> torch.Tensor:
        return self._reduce(self.blk.replay())
