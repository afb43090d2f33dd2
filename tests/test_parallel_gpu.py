"""Tensor-parallel BitLinear (FeedForward column/row split, out_proj row split) and the split
mixers (SISO channel-parallel, MIMO head-parallel) against one device, on 2 GPUs: prefill and
decode logits must be bit-identical (int8 codes from the all-reduced row maxima, exact int32
partial sums, same float epilogue).  Skipped with fewer than 2 GPUs."""
import json
import os
import socket
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("batch,seqlen,mimo", [(4, 40, False), (96, 24, False), (4, 40, True), (96, 24, True)])
def test_tensor_parallel_bit_identical(batch, seqlen, mimo):
    import torch.multiprocessing as mp
    import tp_worker
    cfg = dict(n_layer=2, d_model=256, d_state=64, ent_rank=16, entanglement_window=8, vocab_size=512,
               d_intermediate=768, max_seq_len=128)
    if mimo:
        cfg.update(use_mimo=True, n_heads=4, d_state=32)
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "tp.json")
        mp.spawn(tp_worker.run, args=(2, _free_port(), out, cfg, batch, seqlen), nprocs=2, join=True)
        res = json.load(open(out))
    assert res["bit_identical"], res
