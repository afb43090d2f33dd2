"""Paged decode-state snapshots on the GPU: decoding with the pages gives the same outputs,
each page holds the states of its position, and least recently used pages move to the host."""
import pytest
import torch

from helpers import build_siso, max_rel, randn

pytestmark = pytest.mark.gpu


def test_paged_decode(lib):
    kw = dict(d_model=64, d_state=32, ent_rank=16, entanglement_window=8, max_seq_len=2048)
    m = build_siso(kw).cuda()
    B, L, steps = 2, 16, 12
    x = randn((B, L, 64), 1).cuda()
    xs = [randn((B, 1, 64), 10 + s).cuda() for s in range(steps)]
    outs = {}
    for paged in (False, True):
        c = m.allocate_inference_cache(B, 2048, use_paged_cache=paged, page_size=8, max_gpu_pages=1)
        ip = {"state_cache": c}
        seen = {}
        with torch.no_grad():
            m(x, inference_params=ip)
            ys = []
            for s in range(steps):
                seen[int(c["seq_pos"])] = c["state"].clone()
                ys.append(m(xs[s], inference_params=ip)[0])
        torch.cuda.synchronize()
        outs[paged] = torch.cat(ys, 1).cpu()
        if paged:
            pc = c["paged_cache"]
            assert sorted(pc.pages) == [2, 3]  # positions 16 and 24 (page size 8)
            assert pc.gpu_page_count == 1 and not pc.pages[2].is_on_gpu  # max_gpu_pages=1: LRU offloaded
            for pos in (16, 24):
                pc.active_state = None
                got = pc.load_state(pos)
                assert torch.equal(got["state"].cpu(), seen[pos].cpu())
    assert max_rel(outs[True].numpy(), outs[False].numpy()) == 0.0
