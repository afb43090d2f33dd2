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


# ------------------------------------------------------------------ channel-parallel SISO mixer
# The widest configuration's whole SISO layer (tesm.py:1195-1261) over the ranks:
#   in_proj      column-parallel by segment: this rank's rows of local / gate (a d_model range)
#                and of value / decay / write (a d_state range); the q / k rows (ent_rank each)
#                are replicated, so every rank computes the same window scores.
#   scan, window on this rank's d_state channels only (both are per channel given q, k).
#   all-gather   tanh(ent), ent - s and the scan states (tokens x d_state): state_proj /
#                ent_proj need whole rows (per-token quantisation, K = d_state), and the next
#                layer's cross-layer q bias needs every channel's state.
#   combine      state_proj / ent_proj + output combine column-parallel on the d_model range.
#   out_proj     row-parallel on the same range: row maxima all-reduced (MAX), int32 partial
#                sums all-reduced (SUM), scaled once -- bit-identical to one device.
# Decode keeps the same split: this rank's channels of the fp64 state and of the window-state
# cache, the replicated key cache.  Every rank's share must be equal (d_model and d_state
# divisible by the world size in units of 16 / 8).

def enable_mixer_parallel(model, group=None):
    """enable_tensor_parallel plus the split of every mixer: SISO layers channel-parallel (see
    above), MIMO layers head-parallel (see mimo_prefill_tp)."""
    tp = enable_tensor_parallel(model, group)
    for block in model.backbone.layers:
        enable_mimo_head_parallel(block.mixer, tp) if _is_mimo(block.mixer) else _enable_siso(block.mixer, tp)
    return tp


def _is_mimo(mx):
    return hasattr(mx, "mimo_rank") and hasattr(mx, "n_heads")


def _enable_siso(mx, tp: TPGroup):
    if mx.d_model % (16 * tp.world) or mx.d_state % (8 * tp.world):
        raise TesmError(f"tesm_b200: channel-parallel mixer needs d_model % {16 * tp.world} == 0 and "
                        f"d_state % {8 * tp.world} == 0")
    mx.__dict__["_b200_tp"] = tp
    mx.__dict__["_b200_tp_mixer"] = True


def mixer_tp(mod) -> Optional[TPGroup]:
    tp = get_tp(mod)
    return tp if tp is not None and mod.__dict__.get("_b200_tp_mixer") else None


def mixer_shards(mixer, tp: TPGroup):
    """This rank's in_proj rows, decay bias, combine weight rows and out_proj columns, cached."""
    from . import layers
    _no_imported(mixer.in_proj, mixer.state_proj, mixer.ent_proj, mixer.out_proj)
    ws = [mixer.in_proj.weight, mixer.state_proj.weight, mixer.ent_proj.weight, mixer.out_proj.weight]
    key = tuple((w.data_ptr(), w._version) for w in ws) + (tp.rank, tp.world)
    hit = mixer.__dict__.get("_b200_tp_mix")
    if hit is not None and hit[0] == key:
        return hit[1]
    Dm, D, R = mixer.d_model, mixer.d_state, mixer.ent_rank
    dm0, dm1 = shard_range(Dm, tp.world, tp.rank, 16)
    d0, d1 = shard_range(D, tp.world, tp.rank, 8)
    dev = ws[0].device
    ar = lambda a, b: torch.arange(a, b, device=dev)  # noqa: E731
    rows = torch.cat([ar(dm0, dm1), Dm + ar(d0, d1), Dm + D + ar(d0, d1), Dm + 2 * D + ar(d0, d1),
                      Dm + 3 * D + ar(dm0, dm1), ar(2 * Dm + 3 * D, 2 * Dm + 3 * D + 2 * R)])
    w_in = ws[0].detach().contiguous()
    scale, deq = ops.weight_scale(w_in, mixer.in_proj.bit_eps)  # the full weight's scale
    in_pw = ops.pack_weight(w_in[rows].contiguous(), mixer.in_proj.bit_eps, scale=scale)
    in_pw.deq = deq
    tern, deq1, deq2, Dp = layers.combine_weight(mixer)
    out_pw = ops.pack_shard(ws[3].detach().contiguous(), mixer.out_proj.bit_eps, cols=(dm0, dm1))
    sh = dict(in_pw=in_pw, decay_bias=mixer.decay_bias.detach().float()[d0:d1].contiguous(),
              tern=tern[dm0:dm1].contiguous(), deq1=deq1, deq2=deq2, Dp=Dp, out_pw=out_pw,
              dm=(dm0, dm1), d=(d0, d1))
    mixer.__dict__["_b200_tp_mix"] = (key, sh)
    return sh


def _gather_cols(x: torch.Tensor, tp: TPGroup) -> torch.Tensor:
    """(M, n) per rank -> (M, world * n), rank r's columns at [r*n, (r+1)*n)."""
    import torch.distributed as dist
    x = x.contiguous()
    out = torch.empty(tp.world, *x.shape, device=x.device, dtype=x.dtype)
    dist.all_gather_into_tensor(out, x, group=tp.group)
    return out.permute(1, 0, 2).reshape(x.shape[0], -1)


def _combine_out(mixer, sh, proj_r, tanh_r, chg_r, M, act_dtype, tp: TPGroup):
    """All-gather tanh(ent) | ent - s, then the column-parallel combine and row-parallel out_proj."""
    D, Dp = mixer.d_state, sh["Dp"]
    D_r = tanh_r.shape[1]
    dm0, dm1 = sh["dm"]
    Dm_r = dm1 - dm0
    g = _gather_cols(torch.cat([tanh_r, chg_r], 1).view(M, 2, D_r).transpose(0, 1).reshape(2 * M, D_r), tp)
    tanh_full, chg_full = g[:M], g[M:]
    codes = torch.zeros(M, 2 * Dp, device=proj_r.device, dtype=torch.int8)
    c1, inv1, _ = ops.quant_act(tanh_full, mixer.state_proj.bit_eps, ops.LAYOUT_ROWMAJOR)
    c2, inv2, _ = ops.quant_act(chg_full, mixer.ent_proj.bit_eps, ops.LAYOUT_ROWMAJOR)
    codes[:, :D] = c1[:, :D]
    codes[:, Dp:Dp + D] = c2[:, :D]
    y_r = torch.empty(M, Dm_r, device=proj_r.device, dtype=act_dtype)
    ops.gemm_combine(codes, Dp, inv1, inv2, sh["tern"], sh["deq1"], sh["deq2"], proj_r, 0, Dm_r + 3 * D_r, M, Dm_r,
                     y_r)
    # out_proj row-parallel over this rank's y columns
    amax = _all_reduce(ops.row_absmax(y_r), "max", tp)
    qy = ops.quant_act_amax(y_r, mixer.out_proj.bit_eps, amax)
    pw = sh["out_pw"]
    acc = torch.empty(M, pw.N, device=y_r.device, dtype=torch.int32)
    ops.gemm_acc(qy.codes, qy.inv, pw, M, acc)
    _all_reduce(acc, "sum", tp)
    return ops.acc_scale(acc, qy.inv, pw, act_dtype)


def _shard_cache(cache, B, W, R, D_r, dev):
    tc = cache.get("_tp")
    if tc is None or tc["state"].shape != (B, D_r):
        tc = {"state": torch.zeros(B, D_r, device=dev, dtype=torch.float64),
              "kc": torch.zeros(B, W, R, device=dev, dtype=torch.float32),
              "vc": torch.zeros(B, W, D_r, device=dev, dtype=torch.float32)}
        cache["_tp"] = tc
    return tc


def siso_prefill_tp(mod, q: ops.QuantAct, shape, cross_layer_state, prev_state, cache, act_dtype, tp: TPGroup):
    """TESM_SISO.forward prefill (tesm.py:1175-1272) split over the ranks (see above).  A cache
    gets this rank's channels of the state and window states under cache["_tp"]."""
    from . import layers
    B, L = shape
    M = B * L
    sh = mixer_shards(mod, tp)
    Dm, D, R, W = mod.d_model, mod.d_state, mod.ent_rank, mod.entanglement_window
    (dm0, dm1), (d0, d1) = sh["dm"], sh["d"]
    Dm_r, D_r = dm1 - dm0, d1 - d0
    dev = q.codes.device
    proj = ops.matmul_q(q, sh["in_pw"], act_dtype)  # (M, 2 Dm_r + 3 D_r + 2 R)
    cross_bias = None
    if cross_layer_state is not None:
        cross_bias = layers.linear(mod.cross_layer_q_proj, cross_layer_state.reshape(M, D).float(), torch.float32)
    states = torch.empty(M, D_r, device=dev, dtype=torch.float32)
    fin32 = torch.empty(B, D_r, device=dev, dtype=torch.float32)
    fin64 = torch.empty(B, D_r, device=dev, dtype=torch.float64)
    h0 = prev_state.to(device=dev, dtype=torch.float64)[:, d0:d1].contiguous() if prev_state is not None else None
    ops.siso_scan(proj, B, L, Dm_r, D_r, R, sh["decay_bias"], h0, states, fin32, fin64, mod.state_scan_chunk_size)
    tanh_e = torch.empty(M, D_r, device=dev, dtype=act_dtype)
    chg = torch.empty(M, D_r, device=dev, dtype=act_dtype)
    thr, es, base = mod.entanglement_threshold, mod.entanglement_scale, mod.rope_base
    if W > 0:
        ops.siso_local_ent(proj, B, L, Dm_r, D_r, R, W, cross_bias, layers._param_cache(mod, "local_entanglement_bias"),
                           states, thr, es, base, tanh_e, chg)
    else:
        relb = ops.global_relbias(layers._param_cache(mod, "global_rel_pos_embed"), float(mod.global_rel_pos_scale),
                                  float(mod.global_rel_pos_bias), L)
        ops.siso_global_ent(proj, B, L, Dm_r, D_r, R, cross_bias, relb, states, thr, es, base, tanh_e, chg)
    if cache is not None and "state" in cache:
        layers._prepare_cache(cache, dev)
        tc = _shard_cache(cache, B, cache["ent_k_cache"].shape[1], R, D_r, dev)
        ops.cache_fill(proj, states, 1, B, L, Dm_r, 1, D_r, R, tc["kc"].shape[1], base, fin64, tc["state"], tc["kc"],
                       tc["vc"], cache["_ctl"])
        layers._set_prefilled(cache, L)
    out = _combine_out(mod, sh, proj, tanh_e, chg, M, act_dtype, tp)
    states_full = _gather_cols(states, tp)
    fin_full = _gather_cols(fin64, tp)
    mod.last_entanglement_map = None
    mod.last_entanglement_stats = None
    mod._last_cross_layer_state = states_full.view(B, L, D)
    mod._last_scan_state_f64 = fin_full
    return out.view(B, L, Dm), fin_full


def siso_decode_tp(mod, q: ops.QuantAct, B, cache, cross_layer_state, act_dtype, tp: TPGroup):
    """TESM_SISO._forward_incremental (tesm.py:1274-1400) split over the ranks."""
    from . import layers
    sh = mixer_shards(mod, tp)
    Dm, D, R = mod.d_model, mod.d_state, mod.ent_rank
    (dm0, dm1), (d0, d1) = sh["dm"], sh["d"]
    Dm_r, D_r = dm1 - dm0, d1 - d0
    dev = q.codes.device
    layers._prepare_cache(cache, dev)
    layers.snapshot_if_due(cache)
    W = cache["ent_k_cache"].shape[1]
    tc = _shard_cache(cache, B, W, R, D_r, dev)
    proj = ops.matmul_q(q, sh["in_pw"], act_dtype)
    cross_bias = None
    if cross_layer_state is not None:
        cross_bias = layers.linear(mod.cross_layer_q_proj, cross_layer_state.reshape(B, D).float(), torch.float32)
    tanh_e = torch.empty(B, D_r, device=dev, dtype=act_dtype)
    chg = torch.empty(B, D_r, device=dev, dtype=act_dtype)
    new_state = torch.empty(B, D_r, device=dev, dtype=torch.float32)
    ops.decode_step(proj, B, Dm_r, 1, D_r, R, W, sh["decay_bias"], layers._param_cache(mod, "local_entanglement_bias"),
                    cross_bias, tc["state"], tc["kc"], tc["vc"], cache["_ctl"], mod.entanglement_threshold,
                    mod.entanglement_scale, mod.rope_base, tanh_e, chg, new_state)
    layers._advance_host(cache, W)
    out = _combine_out(mod, sh, proj, tanh_e, chg, B, act_dtype, tp)
    mod._last_cross_layer_state = _gather_cols(new_state, tp)
    if cache.get("_b200_no_state_out"):
        return out.view(B, 1, Dm), None
    return out.view(B, 1, Dm), _gather_cols(tc["state"], tp)


# ------------------------------------------------------------------ head-parallel MIMO mixer
# TESMMIMO_Optimized (tesm_mimo.py:914-1062) over a group of ranks, each owning a contiguous
# range of heads (config 4 at 8 GPUs: batch x head units):
#   in_proj      this rank's value / decay / write / q / k rows of its heads; the local and gate
#                rows (d_model each) are replicated.
#   scan, window per head (tesm_mimo.py:969-1017), on this rank's heads only.
#   state_proj / ent_proj  row-parallel over the heads' channels (K = n_heads * d_state): row
#                maxima of tanh(ent) and ent - s all-reduced (MAX), int32 partials (SUM), scaled
#                once -- the single-device codes and accumulators.
#   combine, out_proj  replicated (every rank then holds the layer output).
# Decode keeps this rank's heads of the state and of both window caches.  Global entanglement
# mixes every head in one score (tesm_mimo.py:651-687) and is not split.

def enable_mimo_head_parallel(mixer, tp: TPGroup):
    """Split one MIMO mixer's heads over the ranks of ``tp`` (n_heads divisible by the world)."""
    if mixer.n_heads % tp.world:
        raise TesmError(f"tesm_b200: head-parallel MIMO needs n_heads % {tp.world} == 0")
    if mixer.entanglement_window <= 0 or mixer.local_entanglement_bias is None:
        raise TesmError("tesm_b200: head-parallel MIMO supports local entanglement only (global mixes all heads)")
    mixer.__dict__["_b200_tp"] = tp
    mixer.__dict__["_b200_tp_mixer"] = True
    return tp


def mimo_shards(mixer, tp: TPGroup):
    """This rank's in_proj rows, per-head parameters and state/ent_proj columns, cached."""
    _no_imported(mixer.in_proj, mixer.state_proj, mixer.ent_proj)
    ws = [mixer.in_proj.weight, mixer.state_proj.weight, mixer.ent_proj.weight]
    ps = [mixer.decay_bias, mixer.mimo_x, mixer.mimo_o, mixer.local_entanglement_bias]
    key = tuple((t.data_ptr(), t._version) for t in ws + ps) + (tp.rank, tp.world)
    hit = mixer.__dict__.get("_b200_tp_mimo")
    if hit is not None and hit[0] == key:
        return hit[1]
    Dm, D, R, H = mixer.d_model, mixer.d_state, mixer.ent_rank, mixer.n_heads
    C, Rc = H * D, H * R
    h0, h1 = shard_range(H, tp.world, tp.rank)
    dev = ws[0].device
    ar = lambda a, b: torch.arange(a, b, device=dev)  # noqa: E731
    rows = torch.cat([ar(0, Dm), Dm + ar(h0 * D, h1 * D), Dm + C + ar(h0 * D, h1 * D), Dm + 2 * C + ar(h0 * D, h1 * D),
                      Dm + 3 * C + ar(0, Dm), 2 * Dm + 3 * C + ar(h0 * R, h1 * R),
                      2 * Dm + 3 * C + Rc + ar(h0 * R, h1 * R)])
    w_in = ws[0].detach().contiguous()
    scale, deq = ops.weight_scale(w_in, mixer.in_proj.bit_eps)
    in_pw = ops.pack_weight(w_in[rows].contiguous(), mixer.in_proj.bit_eps, scale=scale)
    in_pw.deq = deq
    f = lambda t: t.detach().float()[h0:h1].contiguous()  # noqa: E731
    sh = dict(in_pw=in_pw, h=(h0, h1), decay_bias=f(ps[0]), mimo_x=f(ps[1]), mimo_o=f(ps[2]), bias=f(ps[3]),
              sp_pw=ops.pack_shard(ws[1].detach().contiguous(), mixer.state_proj.bit_eps, cols=(h0 * D, h1 * D)),
              ep_pw=ops.pack_shard(ws[2].detach().contiguous(), mixer.ent_proj.bit_eps, cols=(h0 * D, h1 * D)))
    mixer.__dict__["_b200_tp_mimo"] = (key, sh)
    return sh


def _row_parallel_acc(x_r, pw, eps, tp: TPGroup):
    """int32 accumulators of a BitLinear whose input columns are split over the ranks (global row
    maxima, local codes, partials summed) and the per-row 1/s."""
    amax = _all_reduce(ops.row_absmax(x_r), "max", tp)
    q = ops.quant_act_amax(x_r, eps, amax)
    acc = torch.empty(x_r.shape[0], pw.N, device=x_r.device, dtype=torch.int32)
    ops.gemm_acc(q.codes, q.inv, pw, x_r.shape[0], acc)
    _all_reduce(acc, "sum", tp)
    return acc, q.inv


def _mimo_tail(mod, sh, proj_r, tanh_r, chg_r, M, act_dtype, tp: TPGroup):
    """state_proj / ent_proj row-parallel over the rank's heads, then the combine epilogue of
    the one-device dual-accumulator GEMM on the summed accumulators (bit-identical to it)."""
    from . import layers
    acc1, inv1 = _row_parallel_acc(tanh_r, sh["sp_pw"], mod.state_proj.bit_eps, tp)
    acc2, inv2 = _row_parallel_acc(chg_r, sh["ep_pw"], mod.ent_proj.bit_eps, tp)
    h0, h1 = sh["h"]
    Dm = mod.d_model
    y = torch.empty(M, Dm, device=proj_r.device, dtype=act_dtype)
    ops.combine_acc(acc1, acc2, inv1, inv2, sh["sp_pw"].deq, sh["ep_pw"].deq, proj_r, 0,
                    Dm + 3 * (h1 - h0) * mod.d_state, y)
    return layers.linear(mod.out_proj, y, act_dtype)


def _mimo_shard_cache(cache, B, W, H_r, R, D, dev):
    tc = cache.get("_tp")
    if tc is None or tc["state"].shape != (B, H_r, D):
        tc = {"state": torch.zeros(B, H_r, D, device=dev, dtype=torch.float64),
              "kc": torch.zeros(B, W, H_r, R, device=dev, dtype=torch.float32),
              "vc": torch.zeros(B, W, H_r, D, device=dev, dtype=torch.float32)}
        cache["_tp"] = tc
    return tc


def mimo_prefill_tp(mod, q: ops.QuantAct, shape, cache, act_dtype, tp: TPGroup):
    """TESMMIMO_Optimized.forward prefill split over the heads (see above)."""
    from . import layers
    B, L = shape
    M = B * L
    sh = mimo_shards(mod, tp)
    Dm, D, R, RM, W = mod.d_model, mod.d_state, mod.ent_rank, mod.mimo_rank, mod.entanglement_window
    h0, h1 = sh["h"]
    H_r = h1 - h0
    C_r = H_r * D
    dev = q.codes.device
    proj = ops.matmul_q(q, sh["in_pw"], act_dtype)
    states = torch.empty(M, RM, C_r, device=dev, dtype=torch.float32)
    fin32 = torch.empty(B, C_r, device=dev, dtype=torch.float32)
    fin64 = torch.empty(B, C_r, device=dev, dtype=torch.float64)
    ops.mimo_scan(proj, B, L, Dm, H_r, D, R, RM, sh["decay_bias"], sh["mimo_x"], states, fin32, fin64)
    tanh_e = torch.empty(M, C_r, device=dev, dtype=act_dtype)
    chg = torch.empty(M, C_r, device=dev, dtype=act_dtype)
    ops.mimo_local_ent(proj, B, L, Dm, H_r, D, R, RM, W, sh["bias"], sh["mimo_o"], states,
                       mod.entanglement_threshold, mod.entanglement_scale, mod.rope_base, True, tanh_e, chg)
    if cache is not None and "state" in cache:
        layers._prepare_cache(cache, dev)
        tc = _mimo_shard_cache(cache, B, cache["ent_k_cache"].shape[1], H_r, R, D, dev)
        ops.cache_fill(proj, states, RM, B, L, Dm, H_r, D, R, tc["kc"].shape[1], mod.rope_base, fin64, tc["state"],
                       tc["kc"], tc["vc"], cache["_ctl"])
        layers._set_prefilled(cache, L)
    out = _mimo_tail(mod, sh, proj, tanh_e, chg, M, act_dtype, tp)
    last = states.view(B, L, RM, C_r)[:, -1, 0].contiguous()
    mod.last_entanglement_map = None
    mod._last_cross_layer_state = _gather_cols(last, tp).view(B, mod.n_heads, D)
    final = _gather_cols(fin64, tp).view(B, mod.n_heads, D)
    mod._last_scan_state_f64 = final
    return out.view(B, L, Dm), final


def mimo_decode_tp(mod, q: ops.QuantAct, B, cache, cross_layer_state, act_dtype, tp: TPGroup):
    """TESMMIMO_Optimized._forward_incremental (tesm_mimo.py:753-912) split over the heads."""
    from . import layers
    sh = mimo_shards(mod, tp)
    Dm, D, R = mod.d_model, mod.d_state, mod.ent_rank
    h0, h1 = sh["h"]
    H_r = h1 - h0
    dev = q.codes.device
    layers._prepare_cache(cache, dev)
    layers.snapshot_if_due(cache)
    W = cache["ent_k_cache"].shape[1]
    tc = _mimo_shard_cache(cache, B, W, H_r, R, D, dev)
    proj = ops.matmul_q(q, sh["in_pw"], act_dtype)
    cross_bias = None
    if cross_layer_state is not None:
        cs = cross_layer_state
        if cs.dim() != 3:
            raise TesmError("tesm_b200: MIMO decode expects a (B, n_heads, d_state) cross-layer state")
        cross_bias = layers.linear(mod.cross_layer_q_proj, cs[:, h0:h1].reshape(B * H_r, D).float(), torch.float32)
    tanh_e = torch.empty(B, H_r * D, device=dev, dtype=act_dtype)
    chg = torch.empty(B, H_r * D, device=dev, dtype=act_dtype)
    new_state = torch.empty(B, H_r * D, device=dev, dtype=torch.float32)
    ops.decode_step(proj, B, Dm, H_r, D, R, W, sh["decay_bias"], sh["bias"], cross_bias, tc["state"], tc["kc"],
                    tc["vc"], cache["_ctl"], mod.entanglement_threshold, mod.entanglement_scale, mod.rope_base,
                    tanh_e, chg, new_state)
    layers._advance_host(cache, W)
    out = _mimo_tail(mod, sh, proj, tanh_e, chg, B, act_dtype, tp)
    mod._last_cross_layer_state = _gather_cols(new_state, tp).view(B, mod.n_heads, D)
    if cache.get("_b200_no_state_out"):
        return out.view(B, 1, Dm), None
    return out.view(B, 1, Dm), _gather_cols(tc["state"].view(B, -1), tp).view(B, mod.n_heads, D)
