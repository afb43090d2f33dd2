"""Pin the numpy oracle to golden vectors produced by the reference itself (CPU only).

Also checks that the b200 mirror modules rebuild the reference's exact parameters
from the same seed (state_dict SHA-256 recorded by tests/golden/gen_golden.py), so
GPU parity tests can recreate the weights on machines without the reference.
"""
import numpy as np
import pytest
import torch

import cases
import oracle as O
from helpers import (build_mimo, build_model, build_siso, golden, max_rel, mimo_cfg, model_cfg, params_np,
                     randn, sd_hash, siso_cfg)


@pytest.mark.parametrize("c", cases.BITLINEAR, ids=lambda c: c["name"])
def test_bitlinear_golden(c):
    g = golden("bitlinear_" + c["name"])
    w = (randn((c["N"], c["K"]), 3) * c["wstd"]).to(getattr(torch, c["dtype"])).float().numpy()
    x = randn(c["xshape"], 1, getattr(torch, c["dtype"])).float().numpy()
    t, scale, deq = O.ternary_weight(w, 1e-5, c["dtype"])
    assert np.array_equal(t, g["t"]), "ternary codes differ from the reference"
    assert scale == g["scale"]
    codes, s = O.quant_act(x, 1e-5, c["dtype"])
    assert np.array_equal(codes, g["codes"]), "int8 activation codes differ from the reference"
    assert np.array_equal(s.reshape(-1), g["sx"].reshape(-1))
    acc = O.int_gemm(codes.reshape(-1, c["K"]), t)
    assert np.array_equal(acc, g["acc"]), "int32 accumulators differ"
    tp, sp, _ = O.ternary_weight(w, 1e-8)
    assert np.array_equal(O.pack_int2(tp), g["packed"]), "packed INT2 bytes differ from pack_int2_to_uint8"
    assert np.array_equal(O.unpack_int2(g["packed"], c["K"]), tp)
    y = O.bitlinear(x, w, 1e-5, c["dtype"])
    tol = 2e-2 if c["dtype"] == "bfloat16" else 1e-5
    assert max_rel(y, g["y"]) <= tol


@pytest.mark.parametrize("c", cases.SISO, ids=lambda c: c["name"])
def test_siso_golden(c):
    g = golden("siso_" + c["name"])
    m = build_siso(c["kw"])
    assert sd_hash(m) == str(g["sd_sha256"]), "mirror init does not reproduce the reference parameters"
    P = params_np(m)
    cfg = siso_cfg(m)
    B, L = c["B"], c["L"]
    x = randn((B, L, m.d_model), 1).numpy()
    cross = randn((B, L, m.d_state), 2).numpy() if c.get("cross") else None
    prev = randn((B, m.d_state), 4).double().numpy() if c.get("prev") else None
    cache = O.alloc_cache(cfg, B) if c.get("decode") else None
    y, fin, states = O.siso_forward(P, cfg, x, cross, prev, cache)
    assert max_rel(y, g["y"]) <= 1e-3
    assert max_rel(fin, g["final"]) <= 1e-6
    assert max_rel(states, g["states"]) <= 1e-5
    for s in range(c.get("decode", 0)):
        xt = randn((B, 1, m.d_model), 10 + s).numpy()
        ct = randn((B, m.d_state), 20 + s).numpy() if c.get("cross") else None
        yt, st, _ = O.siso_decode(P, cfg, xt, cache, ct)
        assert max_rel(yt, g[f"dec{s}_y"]) <= 1e-3, f"decode step {s}"
        assert max_rel(st, g[f"dec{s}_state"]) <= 1e-6
    if cache is not None:
        assert cache["cache_idx"] == int(g["cache_idx"]) and cache["seq_pos"] == int(g["cache_pos"])
        assert max_rel(cache["ent_k_cache"], g["cache_k"]) <= 1e-5
        assert max_rel(cache["ent_v_cache"], g["cache_v"]) <= 1e-5


@pytest.mark.parametrize("c", cases.MIMO, ids=lambda c: c["name"])
def test_mimo_golden(c):
    g = golden("mimo_" + c["name"])
    m = build_mimo(c["kw"])
    assert sd_hash(m) == str(g["sd_sha256"])
    P = params_np(m)
    cfg = mimo_cfg(m)
    B, L = c["B"], c["L"]
    x = randn((B, L, m.d_model), 1).numpy()
    cache = O.alloc_cache(cfg, B, mimo=True) if c.get("decode") else None
    y, fin, cross = O.mimo_forward(P, cfg, x, cache)
    assert max_rel(y, g["y"]) <= 1e-3
    assert max_rel(fin, g["final"]) <= 1e-5
    assert max_rel(cross, g["cross"]) <= 1e-5
    for s in range(c.get("decode", 0)):
        xt = randn((B, 1, m.d_model), 10 + s).numpy()
        ct = randn((B, m.n_heads, m.d_state), 20 + s).numpy() if c.get("cross") else None
        yt, st, _ = O.mimo_decode(P, cfg, xt, cache, ct)
        assert max_rel(yt, g[f"dec{s}_y"]) <= 1e-3, f"decode step {s}"
        assert max_rel(st, g[f"dec{s}_state"]) <= 1e-6


@pytest.mark.parametrize("c", cases.MODEL, ids=lambda c: c["name"])
def test_model_golden(c):
    g = golden("model_" + c["name"])
    m = build_model(c["cfg"])
    assert sd_hash(m) == str(g["sd_sha256"])
    P = params_np(m)
    cfg = model_cfg(m.tesm_config)
    ids = g["ids"]
    logits = O.model_forward(P, cfg, ids)
    assert max_rel(logits, g["logits"]) <= 1e-3
    cache = O.model_alloc_cache(cfg, c["B"])
    lg = O.model_forward(P, cfg, ids, cache)
    assert max_rel(lg, g["prefill_logits"]) <= 1e-3
    for s in range(c["decode"]):
        lg = O.model_forward(P, cfg, g[f"dec{s}_ids"], cache)
        assert max_rel(lg, g[f"dec{s}_logits"]) <= 1e-3, f"decode step {s}"


# ------------------------------------------------------------------ scan clamp and RoPE frequencies
def _scan_clamped_recurrence(a, u, cs=16):
    """The recurrence the SISO scan kernels run (fp64 here): h_t = a_t h_{t-1} + u_t min(1, P_t/1e-12),
    P_t the product of max(a, 1e-12) since the last multiple of cs.  It restates the reference's
    chunk formula h_t = A_t (h_c + sum u_s / max(A_s, 1e-12)) (tesm.py:1085-1088)."""
    a = np.maximum(np.asarray(a, np.float64), 1e-12)
    u = np.asarray(u, np.float64)
    B, L, D = a.shape
    cs = min(cs, L)
    h = np.zeros((B, D))
    P = np.ones((B, D))
    out = np.empty_like(u)
    for t in range(L):
        if t % cs == 0:
            P = np.ones((B, D))
        P = P * a[:, t]
        h = a[:, t] * h + u[:, t] * np.minimum(1.0, P / 1e-12)
        out[:, t] = h
    return out


@pytest.mark.parametrize("which", ["small", "usual"])
def test_scan_chunk_clamp_golden(which):
    """The oracle's chunked scan and the kernels' clamped recurrence both match the reference's
    _parallel_state_scan, including decays small enough to hit its 1e-12 clamp."""
    g = golden("scan_rope")
    a, u = g[f"scan_{which}_a"], g[f"scan_{which}_u"]
    ref, fin = O.scan_chunked_f64(a, u)
    assert max_rel(ref, g[f"scan_{which}_states"]) <= 1e-6
    assert max_rel(fin, g[f"scan_{which}_final"]) <= 1e-6
    assert max_rel(_scan_clamped_recurrence(a, u), g[f"scan_{which}_states"]) <= 1e-6
    if which == "small":  # the clamp changes the result: the plain recurrence does not match
        plain = _scan_clamped_recurrence(a, u, cs=10 ** 9)
        a64 = np.maximum(a.astype(np.float64), 1e-12)
        h = np.zeros(a.shape[::2])
        for t in range(a.shape[1]):
            h = a64[:, t] * h + u[:, t]
            plain[:, t] = h
        assert max_rel(plain, g[f"scan_{which}_states"]) > 1e-2


def test_rope_inv_freq_matches_reference_expression():
    """1 / base^(2i/D) as the reference's fp32 torch expression gives it (tesm.py:787-789),
    bit for bit, for every even width up to 64; the kernels compute it the same way (the
    power in fp64 rounded once to fp32, then an fp32 reciprocal)."""
    from oracle import tesm_oracle
    for D in range(2, 65, 2):
        idx = torch.arange(D // 2, dtype=torch.float32)
        ref = (1.0 / (10000.0 ** (2.0 * idx / D))).numpy()
        assert np.array_equal(tesm_oracle._inv_freq(D, 10000.0), ref), D


@pytest.mark.parametrize("R", [64, 48])
def test_rope_far_positions_golden(R):
    g = golden("scan_rope")
    y = O.rope(g[f"rope{R}_x"], pos_offset=8000)
    assert max_rel(y, g[f"rope{R}_y"]) <= 2e-6
