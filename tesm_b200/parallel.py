"""Tensor-parallel BitLinear over the ranks of a torch.distributed (NCCL) group.

The reference runs on one device; this is the column/row-parallel split of its FeedForward
(mixer_seq_simple.py:45-67) and of the mixer's out_proj (tesm.py:1261) for multi-GPU decode:

* gate/up (column-parallel): each rank owns a contiguous range of 128-row blocks of
  d_intermediate; the SwiGLU GEMM runs on its rows only.
* down_proj (row-parallel over the same d_intermediate range): the per-token int8 scale needs the
  max |h| over the full row, so the ranks all-reduce (MAX) their row maxima first and every rank
  quantises its columns with the global scale.  Its int32 partial accumulators are all-reduced
  (SUM) and scaled once: the codes, the accumulators and the float epilogue are those of a single
  device, so the output is bit-identical.
* out_proj (row-parallel over d_model): y is replicated, so every rank quantises the full row
  locally and keeps its column range; int32 partials are all-reduced (SUM).

Every ternary shard is packed with the scale of the full weight (the reference quantises each
BitLinear as a whole, tesm.py:211-215).  Prefill uses data parallelism instead (independent
sequences, no collective); tensor parallelism is for decode, where it divides the per-GPU weight
traffic by the number of ranks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import ops
from ._lib import TesmError


@dataclass
class TPGroup:
    rank: int
    world: int
    group: object = None  # torch.distributed ProcessGroup (None: the default group)


def shard_range(n: int, world: int, rank: int, unit: int = 1) -> Tuple[int, int]:
    """Contiguous [lo, hi) share of n items in whole units of `unit`, the first n_units % world
    ranks taking one extra unit."""
    if n % unit:
        raise ValueError(f"tensor-parallel split of {n} needs a multiple of {unit}")
    units = n // unit
    base, extra = divmod(units, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo * unit, hi * unit


def enable_tensor_parallel(model, group=None):
    """Shard every block's FeedForward and out_proj over the ranks of `group`.  All ranks must
    hold the same full weights (same seed or the same checkpoint)."""
    import torch.distributed as dist
    tp = TPGroup(dist.get_rank(group), dist.get_world_size(group), group)
    for block in model.backbone.layers:
        block.mlp.__dict__["_b200_tp"] = tp
        block.mixer.__dict__["_b200_tp"] = tp
    return tp


def get_tp(mod) -> Optional[TPGroup]:
    tp = mod.__dict__.get("_b200_tp")
    return tp if tp is not None and tp.world > 1 else None


def _all_reduce(t: torch.Tensor, op: str, tp: TPGroup):
    import torch.distributed as dist
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM, group=tp.group)
    return t


# ------------------------------------------------------------------ shards
def _no_imported(*lins):
    for lin in lins:
        if "_b200_int2" in lin.__dict__:
            raise TesmError("tesm_b200: tensor-parallel shards are cut from the latent weights; weights "
                            "imported from an INT2 export are supported on one GPU / data-parallel only")


def ffn_shards(ffn, tp: TPGroup, blk: int = 128):
    """(interleaved gate/up shard, down_proj column shard, (f0, f1)) of this rank, cached."""
    _no_imported(ffn.gate_proj, ffn.up_proj, ffn.down_proj)
    g, u, d = ffn.gate_proj.weight, ffn.up_proj.weight, ffn.down_proj.weight
    key = (g.data_ptr(), g._version, u.data_ptr(), u._version, d.data_ptr(), d._version, tp.rank, tp.world)
    hit = ffn.__dict__.get("_b200_tp_shards")
    if hit is not None and hit[0] == key:
        return hit[1]
    Fd, K = g.shape
    f0, f1 = shard_range(Fd, tp.world, tp.rank, blk)
    Fl = f1 - f0
    eps = ffn.gate_proj.bit_eps
    gs = ops.pack_shard(g.detach().contiguous(), eps, rows=(f0, f1))
    us = ops.pack_shard(u.detach().contiguous(), eps, rows=(f0, f1))
    dev = g.device
    # interleave [gate block | up block] per 128 rows, as ffn_packed does for the full weight
    f = torch.arange(Fl, device=dev)
    Kp = gs.tern.shape[1]
    packed = torch.empty(2 * Fl, gs.packed.shape[1], device=dev, dtype=torch.uint8)
    tern = torch.empty(2 * Fl, Kp, device=dev, dtype=torch.int8)
    deq = torch.empty(2 * Fl, device=dev, dtype=torch.float32)
    for i, s in enumerate((gs, us)):
        dst = (f // blk) * 2 * blk + i * blk + f % blk
        packed[dst] = s.packed
        tern[dst] = s.tern
        deq[dst] = s.deq.expand(Fl)
    gu = ops.PackedWeight(packed, tern, deq.clone(), deq, 2 * Fl, K, True)
    down = ops.pack_shard(d.detach().contiguous(), ffn.down_proj.bit_eps, cols=(f0, f1))
    shards = (gu, down, (f0, f1))
    ffn.__dict__["_b200_tp_shards"] = (key, shards)
    return shards


def out_proj_shard(mixer, tp: TPGroup):
    _no_imported(mixer.out_proj)
    w = mixer.out_proj.weight
    key = (w.data_ptr(), w._version, tp.rank, tp.world)
    hit = mixer.__dict__.get("_b200_tp_out")
    if hit is not None and hit[0] == key:
        return hit[1]
    K = w.shape[1]
    k0, k1 = shard_range(K, tp.world, tp.rank, 16)
    pw = ops.pack_shard(w.detach().contiguous(), mixer.out_proj.bit_eps, cols=(k0, k1))
    mixer.__dict__["_b200_tp_out"] = (key, (pw, (k0, k1)))
    return pw, (k0, k1)


# ------------------------------------------------------------------ forward pieces
def ffn_q_tp(ffn, q: ops.QuantAct, act_dtype, tp: TPGroup):
    """FeedForward.forward with gate/up column-parallel and down_proj row-parallel."""
    gu, down, (f0, f1) = ffn_shards(ffn, tp)
    Fl = f1 - f0
    if q.layout == ops.LAYOUT_ROWMAJOR:
        h = ops.gemm_swiglu(q, gu, act_dtype)
    else:
        g = ops.matmul_q(q, gu, act_dtype)
        h = torch.empty(q.M, Fl, device=g.device, dtype=act_dtype)
        ops.silu_mul(g, Fl, h, 128)
    amax = _all_reduce(ops.row_absmax(h), "max", tp)
    qd = ops.quant_act_amax(h, ffn.down_proj.bit_eps, amax)
    acc = torch.empty(q.M, down.N, device=h.device, dtype=torch.int32)
    ops.gemm_acc(qd.codes, qd.inv, down, q.M, acc)
    _all_reduce(acc, "sum", tp)
    return ops.acc_scale(acc, qd.inv, down, act_dtype)


def out_proj_tp(mixer, y2d: torch.Tensor, act_dtype, tp: TPGroup):
    """out_proj row-parallel over d_model: full-row quantisation (y is replicated), this rank's
    columns, int32 partials all-reduced."""
    pw, (k0, k1) = out_proj_shard(mixer, tp)
    M = y2d.shape[0]
    codes, inv, _ = ops.quant_act(y2d, mixer.out_proj.bit_eps, ops.LAYOUT_ROWMAJOR)
    acc = torch.empty(M, pw.N, device=y2d.device, dtype=torch.int32)
    ops.gemm_acc(codes[:, k0:k1], inv, pw, M, acc)
    _all_reduce(acc, "sum", tp)
    return ops.acc_scale(acc, inv, pw, act_dtype)
