"""Tensor-parallel decomposition on CPU (gloo, world size 2): the shard ranges, and the claim the
GPU path relies on — row maxima all-reduced with MAX give every rank the single-device int8 codes
of its columns, and int32 partial products all-reduced with SUM give the single-device
accumulators exactly — checked with the oracle's quantiser and integer GEMM."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from tesm_b200.parallel import shard_range


@pytest.mark.parametrize("n,world,unit", [(11008, 8, 128), (4096, 8, 16), (768, 2, 128), (1000, 3, 8), (256, 4, 16)])
def test_shard_range_partition(n, world, unit):
    spans = [shard_range(n, world, r, unit) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in spans]
    assert all(s % unit == 0 for s in sizes)
    assert max(sizes) - min(sizes) <= unit


def test_shard_range_rejects_ragged():
    with pytest.raises(ValueError):
        shard_range(1000, 2, 0, 128)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(5)
    M, F, Dm = 12, 384, 64
    h = (rng.standard_normal((M, F)) * rng.uniform(0.1, 3.0, (M, 1))).astype(np.float32)
    w = (rng.standard_normal((Dm, F)) * 0.02).astype(np.float32)
    t, _, deq = O.ternary_weight(w, 1e-5)  # scale of the full weight
    f0, f1 = shard_range(F, world, rank, 128)
    # this rank: local row maxima -> MAX over ranks -> codes of its columns with the global scale
    amax = torch.from_numpy(np.abs(h[:, f0:f1]).max(1))
    dist.all_reduce(amax, op=dist.ReduceOp.MAX)
    codes_full, s_full = O.quant_act(h, 1e-5)
    codes_tp, s_tp = O.quant_act(h[:, f0:f1], 1e-5, amax=amax.numpy())
    acc = torch.from_numpy(O.int_gemm(codes_tp, t[:, f0:f1]).astype(np.int64))
    dist.all_reduce(acc, op=dist.ReduceOp.SUM)
    ok = (np.array_equal(s_tp, s_full) and np.array_equal(codes_tp, codes_full[:, f0:f1])
          and np.array_equal(acc.numpy(), O.int_gemm(codes_full, t).astype(np.int64)))
    with open(os.path.join(out_dir, f"r{rank}"), "w") as f:
        f.write("1" if ok else "0")
    dist.destroy_process_group()


def test_row_parallel_decomposition_exact(tmp_path):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    assert [open(tmp_path / f"r{r}").read() for r in range(2)] == ["1", "1"]


def _mixer_worker(rank, world, port, out_dir):
    """The channel-parallel SISO layer on the oracle: this rank's in_proj rows (local / gate on a
    d_model range, value / decay / write on a d_state range, q / k replicated), scan and window
    on its channels, all-gather, column-parallel combine, row-parallel out_proj -- against the
    oracle's whole layer (tesm.py:1195-1261), exactly."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(9)
    B, L, Dm, D, R, W = 2, 40, 64, 32, 16, 8
    eps, thr, es = 1e-5, 0.1, 0.2
    x = rng.standard_normal((B, L, Dm)).astype(np.float32)
    P = {"in_proj.weight": (rng.standard_normal((2 * Dm + 3 * D + 2 * R, Dm)) * 0.05).astype(np.float32),
         "state_proj.weight": (rng.standard_normal((Dm, D)) * 0.05).astype(np.float32),
         "ent_proj.weight": (rng.standard_normal((Dm, D)) * 0.05).astype(np.float32),
         "out_proj.weight": (rng.standard_normal((Dm, Dm)) * 0.05).astype(np.float32),
         "decay_bias": np.full(D, 3.0, np.float32) + rng.standard_normal(D).astype(np.float32) * 0.3,
         "local_entanglement_bias": (rng.standard_normal(W) * 0.3).astype(np.float32)}
    cfg = dict(d_model=Dm, d_state=D, ent_rank=R, entanglement_window=W, entanglement_threshold=thr,
               entanglement_scale=es, bit_eps=eps, rope_base=1e4, state_scan_chunk_size=16)
    y_ref, _, st_ref = O.siso_forward(P, cfg, x)
    dm0, dm1 = shard_range(Dm, world, rank, 16)
    d0, d1 = shard_range(D, world, rank, 8)
    # in_proj rows of this rank, quantised with the full weight's ternary codes and scale
    t_in, _, deq_in = O.ternary_weight(P["in_proj.weight"], eps)
    rows = np.concatenate([np.arange(dm0, dm1), Dm + np.arange(d0, d1), Dm + D + np.arange(d0, d1),
                           Dm + 2 * D + np.arange(d0, d1), Dm + 3 * D + np.arange(dm0, dm1),
                           2 * Dm + 3 * D + np.arange(2 * R)])
    c, s = O.quant_act(x, eps)
    proj = (O.int_gemm(c, t_in[rows]).astype(np.float64) * (1.0 / s.astype(np.float64))[..., None]
            * np.float64(deq_in)).astype(np.float32)
    Dm_r, D_r = dm1 - dm0, d1 - d0
    local, value, decay, write, gate, q, k = np.split(proj, np.cumsum([Dm_r, D_r, D_r, D_r, Dm_r, R])[:], axis=-1)
    a = O.sigmoid(decay + P["decay_bias"][d0:d1])
    u = (O.sigmoid(write) * np.tanh(value).astype(np.float32)).astype(np.float32)
    st64, _ = O.scan_chunked_f64(a, u)
    st = st64.astype(np.float32)
    avg = O.local_ent(O.rope(q), O.rope(k), st, P["local_entanglement_bias"], thr)
    ent = (st + np.float32(es) * (avg - st)).astype(np.float32)

    def gather(v):
        t = torch.from_numpy(np.ascontiguousarray(v))
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return torch.cat(parts, -1).numpy()

    tanh_full = gather(np.tanh(ent).astype(np.float32))
    chg_full = gather((ent - st).astype(np.float32))
    st_full = gather(st)
    t_s, _, deq_s = O.ternary_weight(P["state_proj.weight"], eps)
    t_e, _, deq_e = O.ternary_weight(P["ent_proj.weight"], eps)
    c1, s1 = O.quant_act(tanh_full, eps)
    c2, s2 = O.quant_act(chg_full, eps)
    sp = (O.int_gemm(c1, t_s[dm0:dm1]) * (1.0 / s1.astype(np.float64))[..., None] * np.float64(deq_s)).astype(np.float32)
    ep = (O.int_gemm(c2, t_e[dm0:dm1]) * (1.0 / s2.astype(np.float64))[..., None] * np.float64(deq_e)).astype(np.float32)
    y_r = (local + O.sigmoid(gate) * sp + ep).astype(np.float32)
    # out_proj row-parallel: MAX of row maxima, codes of this rank's columns, SUM of int32 partials
    amax = torch.from_numpy(np.abs(y_r).max(-1))
    dist.all_reduce(amax, op=dist.ReduceOp.MAX)
    cy, sy = O.quant_act(y_r, eps, amax=amax.numpy())
    t_o, _, deq_o = O.ternary_weight(P["out_proj.weight"], eps)
    acc = torch.from_numpy(O.int_gemm(cy, t_o[:, dm0:dm1]).astype(np.int64))
    dist.all_reduce(acc, op=dist.ReduceOp.SUM)
    out = (acc.numpy().astype(np.float64) * (1.0 / sy.astype(np.float64))[..., None]
           * np.float64(deq_o)).astype(np.float32)
    ok = np.array_equal(st_full, st_ref) and np.allclose(out, y_ref, rtol=0, atol=1e-6 * np.abs(y_ref).max())
    with open(os.path.join(out_dir, f"m{rank}"), "w") as f:
        f.write("1" if ok else f"0 {np.abs(st_full - st_ref).max()} {np.abs(out - y_ref).max()}")
    dist.destroy_process_group()


def test_channel_parallel_mixer_decomposition(tmp_path):
    mp.spawn(_mixer_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    assert [open(tmp_path / f"m{r}").read() for r in range(2)] == ["1", "1"]


def _mimo_head_worker(rank, world, port, out_dir):
    """The head-parallel MIMO layer tail on the oracle (config 4's (b, h) split): each rank owns
    a range of heads, state_proj / ent_proj run row-parallel over those heads' channels (MAX of
    row maxima, SUM of int32 partials), then the combine and out_proj -- against the oracle's
    whole layer (tesm_mimo.py:914-1062), exactly."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(13)
    B, L, Dm, H, D, R, RM, W = 2, 24, 48, 4, 8, 8, 2, 4
    C = H * D
    eps = 1e-5
    x = rng.standard_normal((B, L, Dm)).astype(np.float32)
    P = {"in_proj.weight": (rng.standard_normal((2 * Dm + 3 * C + 2 * H * R, Dm)) * 0.05).astype(np.float32),
         "state_proj.weight": (rng.standard_normal((Dm, C)) * 0.05).astype(np.float32),
         "ent_proj.weight": (rng.standard_normal((Dm, C)) * 0.05).astype(np.float32),
         "out_proj.weight": (rng.standard_normal((Dm, Dm)) * 0.05).astype(np.float32),
         "decay_bias": (np.full((H, D), 2.0) + rng.standard_normal((H, D)) * 0.3).astype(np.float32),
         "mimo_x": (1.0 / RM + rng.standard_normal((H, RM, D)) * 0.05).astype(np.float32),
         "mimo_o": (1.0 / RM + rng.standard_normal((H, RM, D)) * 0.05).astype(np.float32),
         "local_entanglement_bias": (rng.standard_normal((H, W)) * 0.3).astype(np.float32)}
    cfg = dict(d_model=Dm, d_state=D, ent_rank=R, n_heads=H, mimo_rank=RM, entanglement_window=W,
               entanglement_threshold=0.1, entanglement_scale=0.2, bit_eps=eps, rope_base=1e4)
    out_ref, _, _, det = O.mimo_forward(P, cfg, x, details=True)
    h0, h1 = shard_range(H, world, rank, 1)
    c0, c1 = h0 * D, h1 * D

    def row_parallel(xfull, w):
        xr = np.ascontiguousarray(xfull[..., c0:c1])
        amax = torch.from_numpy(np.abs(xr).max(-1))
        dist.all_reduce(amax, op=dist.ReduceOp.MAX)
        c, s = O.quant_act(xr, eps, amax=amax.numpy())
        t, _, deq = O.ternary_weight(w, eps)
        acc = torch.from_numpy(O.int_gemm(c, t[:, c0:c1]).astype(np.int64))
        dist.all_reduce(acc, op=dist.ReduceOp.SUM)
        return (acc.numpy().astype(np.float64) * (1.0 / s.astype(np.float64))[..., None]
                * np.float64(deq.reshape(-1)[0])).astype(np.float32)

    sp = row_parallel(np.tanh(det["ent"].reshape(B, L, C)), P["state_proj.weight"])
    ep = row_parallel(det["chg"].reshape(B, L, C), P["ent_proj.weight"])
    proj = O.bitlinear(x, P["in_proj.weight"], eps)
    local, gate = proj[..., :Dm], O.sigmoid(proj[..., Dm + 3 * C:2 * Dm + 3 * C])
    y = (local + gate * sp + ep).astype(np.float32)
    out = O.bitlinear(y, P["out_proj.weight"], eps)
    ok = np.array_equal(out, out_ref)
    with open(os.path.join(out_dir, f"h{rank}"), "w") as f:
        f.write("1" if ok else f"0 {np.abs(out - out_ref).max()}")
    dist.destroy_process_group()


def test_head_parallel_mimo_tail_decomposition(tmp_path):
    mp.spawn(_mimo_head_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    assert [open(tmp_path / f"h{r}").read() for r in range(2)] == ["1", "1"]
