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
