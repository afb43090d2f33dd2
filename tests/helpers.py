"""Shared test helpers: seeded inputs, state-dict hashing, comparators."""
from __future__ import annotations

import hashlib
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def randn(shape, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


def sd_hash(module):
    h = hashlib.sha256()
    for k, v in module.state_dict().items():
        h.update(k.encode())
        h.update(v.detach().cpu().contiguous().numpy().tobytes())
    return h.hexdigest()


def params_np(module):
    return {k: v.detach().cpu().float().numpy() if v.dtype != torch.float64 else v.detach().cpu().numpy()
            for k, v in module.state_dict().items()}


def max_rel(out, ref):
    """max|out-ref| / max|ref| over the tensor (the tolerance metric used throughout)."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(out - ref).max() / (den if den > 0 else 1.0))


def build_siso(kw, backend="b200"):
    from tesm_b200.modules import TESM_SISO
    torch.manual_seed(0)
    return TESM_SISO(kernel_backend=backend, **kw).eval()


def build_mimo(kw, backend="b200"):
    from tesm_b200.modules import TESMMIMO_Optimized
    torch.manual_seed(0)
    return TESMMIMO_Optimized(kernel_backend=backend, **kw).eval()


def build_model(cfg_kw, backend="b200"):
    from tesm_b200.models import TESMConfig, TESMLMHeadModel
    torch.manual_seed(0)
    return TESMLMHeadModel(TESMConfig(kernel_backend=backend, **cfg_kw)).eval()


def siso_cfg(m):
    return dict(d_model=m.d_model, d_state=m.d_state, ent_rank=m.ent_rank,
                entanglement_window=m.entanglement_window, entanglement_threshold=m.entanglement_threshold,
                entanglement_scale=m.entanglement_scale, bit_eps=m.in_proj.bit_eps, rope_base=m.rope_base,
                state_scan_chunk_size=m.state_scan_chunk_size)


def mimo_cfg(m):
    c = siso_cfg(m)
    c.update(n_heads=m.n_heads, mimo_rank=m.mimo_rank)
    return c


def model_cfg(cfg):
    return dict(n_layer=cfg.n_layer, d_model=cfg.d_model, d_state=cfg.d_state, ent_rank=cfg.ent_rank,
                entanglement_window=cfg.entanglement_window, entanglement_threshold=cfg.entanglement_threshold,
                entanglement_scale=cfg.entanglement_scale, bit_eps=cfg.bit_eps, rope_base=cfg.rope_base,
                state_scan_chunk_size=cfg.state_scan_chunk_size, use_mimo=cfg.use_mimo, n_heads=cfg.n_heads,
                mimo_rank=4, norm_epsilon=cfg.norm_epsilon)
