"""Paged decode-state snapshots (mirror of tesm_ssm/utils/paged_cache.py:17-248).

With ``allocate_inference_cache(..., use_paged_cache=True)`` and ``max_seqlen > 1024``
(tesm.py:636-657, tesm_mimo.py:702-721) a layer's cache carries a ``PagedStateCache``: every
``page_size`` decode positions the incremental step first stores the recurrent state and the
two window caches into the page of that position (tesm.py:1308-1316, tesm_mimo.py:812-819).
Pages live on the GPU up to ``max_gpu_pages``; beyond that the least recently used page other
than the active one moves to pinned host memory, and ``load_state`` brings a page back.  The
snapshots do not feed the decode computation.

Differences from the reference, kept on purpose: a page copies states of any layout into its
flat (batch, d_state) buffers (the MIMO cache holds (batch, heads, d_state), which the
reference's ``copy_`` rejects); a newly created page is never the one evicted to make room for
itself; offloaded pages use pinned host memory.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass
from typing import Dict, Optional

import torch


@dataclass
class StatePage:
    """States of one page: positions [start_pos, end_pos)."""
    page_id: int
    start_pos: int
    end_pos: int
    state: torch.Tensor        # (batch, d_state) float64
    ent_k_cache: torch.Tensor  # (batch, window, ent_rank) float32
    ent_v_cache: torch.Tensor  # (batch, window, d_state) float32
    device: torch.device
    is_on_gpu: bool = True
    last_access: int = 0


def _to_host(t: torch.Tensor) -> torch.Tensor:
    pin = t.is_cuda and torch.cuda.is_available()
    out = torch.empty(t.shape, dtype=t.dtype, device="cpu", pin_memory=pin)
    out.copy_(t)  # synchronous: the page is readable on the host right away
    return out


class PagedStateCache:
    def __init__(self, batch_size: int, d_state: int, ent_rank: int, window: int, page_size: int = 512,
                 max_gpu_pages: int = 100, device: Optional[torch.device] = None):
        self.batch_size = batch_size
        self.d_state = d_state
        self.ent_rank = ent_rank
        self.window = window
        self.page_size = page_size
        self.max_gpu_pages = max_gpu_pages
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.pages: Dict[int, StatePage] = OrderedDict()
        self.gpu_page_count = 0
        self.access_counter = 0
        self.active_state: Optional[Dict] = None
        self.active_page_id: Optional[int] = None

    def _create_empty_page(self, page_id: int, start_pos: int, device: torch.device) -> StatePage:
        b, w = self.batch_size, self.window
        return StatePage(page_id=page_id, start_pos=start_pos, end_pos=start_pos + self.page_size,
                         state=torch.zeros(b, self.d_state, device=device, dtype=torch.float64),
                         ent_k_cache=torch.zeros(b, w, self.ent_rank, device=device, dtype=torch.float32),
                         ent_v_cache=torch.zeros(b, w, self.d_state, device=device, dtype=torch.float32),
                         device=device, is_on_gpu=device.type == "cuda")

    def _tick(self, page: StatePage):
        page.last_access = self.access_counter
        self.access_counter += 1

    def _evict_lru_page(self) -> bool:
        """Move the least recently used GPU page (never the active one, never the last) to the
        host; False when there is nothing to move."""
        if self.gpu_page_count <= 1:
            return False
        victims = [p for p in self.pages.values() if p.is_on_gpu and p.page_id != self.active_page_id]
        if not victims:
            return False
        page = min(victims, key=lambda p: p.last_access)
        page.state, page.ent_k_cache, page.ent_v_cache = (_to_host(page.state), _to_host(page.ent_k_cache),
                                                          _to_host(page.ent_v_cache))
        page.is_on_gpu = False
        page.device = torch.device("cpu")
        self.gpu_page_count -= 1
        return True

    def _load_page_to_gpu(self, page_id: int):
        page = self.pages.get(page_id)
        if page is None:
            return
        if not page.is_on_gpu and self.device.type == "cuda":
            while self.gpu_page_count >= self.max_gpu_pages and self._evict_lru_page():
                pass
            page.state = page.state.to(self.device, non_blocking=True)
            page.ent_k_cache = page.ent_k_cache.to(self.device, non_blocking=True)
            page.ent_v_cache = page.ent_v_cache.to(self.device, non_blocking=True)
            page.is_on_gpu = True
            page.device = self.device
            self.gpu_page_count += 1
            self.pages.move_to_end(page_id)
        self._tick(page)

    def get_page_for_position(self, pos: int) -> int:
        return pos // self.page_size

    def save_state(self, pos: int, state_dict: Dict):
        """Store ``state``, ``ent_k_cache`` and ``ent_v_cache`` into the page of ``pos``."""
        page_id = self.get_page_for_position(pos)
        if page_id not in self.pages:
            page = self._create_empty_page(page_id, page_id * self.page_size, self.device)
            self.pages[page_id] = page
            if page.is_on_gpu:
                self.gpu_page_count += 1
            self.active_page_id = page_id
            while self.gpu_page_count > self.max_gpu_pages and self._evict_lru_page():
                pass
        page = self.pages[page_id]
        if not page.is_on_gpu:
            self._load_page_to_gpu(page_id)
        for name in ("state", "ent_k_cache", "ent_v_cache"):
            dst = getattr(page, name)
            dst.copy_(state_dict[name].reshape(dst.shape))
        self._tick(page)
        self.active_state = dict(state_dict)
        self.active_page_id = page_id

    def load_state(self, pos: int) -> Optional[Dict]:
        """States stored for the page of ``pos`` (None if never saved); ``seq_pos`` is the
        position relative to the page start."""
        page_id = self.get_page_for_position(pos)
        if page_id == self.active_page_id and self.active_state is not None:
            return self.active_state
        if page_id not in self.pages:
            return None
        self._load_page_to_gpu(page_id)
        page = self.pages[page_id]
        self.active_state = {"state": page.state, "ent_k_cache": page.ent_k_cache, "ent_v_cache": page.ent_v_cache,
                             "seq_pos": pos - page.start_pos}
        self.active_page_id = page_id
        return self.active_state

    def get_memory_stats(self) -> Dict:
        per_page = (self.batch_size * self.d_state * 8 + self.batch_size * self.window * self.ent_rank * 4 +
                    self.batch_size * self.window * self.d_state * 4)
        gpu = sum(1 for p in self.pages.values() if p.is_on_gpu)
        return {"gpu_pages": self.gpu_page_count, "cpu_pages": len(self.pages) - self.gpu_page_count,
                "total_pages": len(self.pages), "gpu_memory_mb": gpu * per_page / 2 ** 20,
                "cpu_memory_mb": (len(self.pages) - gpu) * per_page / 2 ** 20}

    def clear(self):
        self.pages.clear()
        self.gpu_page_count = 0
        self.active_state = None
        self.active_page_id = None


def snapshot_if_due(cache: Dict):
    """The decode-step hook (tesm.py:1308-1316): at positions that are a positive multiple of
    the page size, store the cache's states before this step updates them.  Never recorded into
    a CUDA graph being captured (graph-replayed decode steps call it from the host loop)."""
    paged = cache.get("paged_cache") if cache.get("use_paged", False) else None
    if paged is None:
        return
    if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
        return
    pos = int(cache["seq_pos"])
    if pos > 0 and pos % paged.page_size == 0:
        paged.save_state(pos, {"state": cache["state"], "ent_k_cache": cache["ent_k_cache"],
                               "ent_v_cache": cache["ent_v_cache"]})
