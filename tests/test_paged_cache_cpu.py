"""Paged decode-state snapshots (tesm_ssm/utils/paged_cache.py) on the host: the reference's
own PagedStateCache checks (tests/test_torch_only.py:406-437) and the allocation flag."""
import torch

from tesm_b200.paged_cache import PagedStateCache, snapshot_if_due
from helpers import build_siso, build_mimo


def _cpu_cache(**kw):
    d = dict(batch_size=1, d_state=16, ent_rank=8, window=4, page_size=512, device=torch.device("cpu"))
    d.update(kw)
    return PagedStateCache(**d)


def _states(v=0.0, b=1, d=16, r=8, w=4):
    return {"state": torch.full((b, d), v, dtype=torch.float64), "ent_k_cache": torch.full((b, w, r), v),
            "ent_v_cache": torch.full((b, w, d), v)}


def test_save_load_stats_clear():
    c = _cpu_cache()
    assert c.page_size == 512
    c.save_state(0, _states(1.5))
    assert c.load_state(0)["state"][0, 0] == 1.5
    c.save_state(1024, _states(2.5))
    c.active_state = None  # force a real page read
    got = c.load_state(1030)
    assert got["seq_pos"] == 6 and float(got["state"][0, 3]) == 2.5
    assert c.load_state(512 * 7) is None
    st = c.get_memory_stats()
    assert st["total_pages"] == 2 and "gpu_pages" in st
    c.clear()
    assert c.gpu_page_count == 0 and not c.pages


def test_alloc_flag_and_snapshot_position():
    kw = dict(d_model=32, d_state=16, ent_rank=8, entanglement_window=4, max_seq_len=4096)
    m = build_siso(kw)
    c = m.allocate_inference_cache(2, 4096, use_paged_cache=True, page_size=8)
    assert c["use_paged"] and isinstance(c["paged_cache"], PagedStateCache)
    assert not m.allocate_inference_cache(2, 512, use_paged_cache=True)["use_paged"]  # only above 1024
    for pos, due in [(0, False), (7, False), (8, True), (16, True)]:
        c["seq_pos"] = pos
        c["state"].fill_(pos)
        snapshot_if_due(c)
        assert (c["paged_cache"].get_page_for_position(pos) in c["paged_cache"].pages) == due or pos == 7
    assert float(c["paged_cache"].pages[2].state[0, 0]) == 16.0
    # MIMO caches hold (batch, heads, d_state): a page copies them into its flat buffers
    mm = build_mimo(dict(d_model=32, n_heads=2, d_state=8, ent_rank=4, entanglement_window=4, max_seq_len=4096))
    cm = mm.allocate_inference_cache(1, 4096, use_paged_cache=True, page_size=4)
    cm["seq_pos"] = 4
    cm["state"].fill_(3.0)
    snapshot_if_due(cm)
    assert cm["paged_cache"].pages[1].state.shape == (1, 16) and float(cm["paged_cache"].pages[1].state.sum()) == 48.0
