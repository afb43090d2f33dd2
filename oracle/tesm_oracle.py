"""numpy restatement of the reference TESM torch backend (checker only).

TEST INFRASTRUCTURE.  Nothing in the shipped package imports this module; the
CUDA path never routes through it.  Every function names the reference lines
(WANGLILIN360/tesm, paths relative to the project root) whose arithmetic it
restates.  Arrays are numpy; float32 unless stated.  ``dtype`` arguments take
"float32" or "bfloat16" and mean the torch dtype the reference would compute in
(bfloat16 values are carried as float32 arrays rounded to bf16).
"""
from __future__ import annotations

import math
import time

import numpy as np

F32 = np.float32
F64 = np.float64

__all__ = [
    "bf16_round", "cast", "ternary_weight", "pack_int2", "unpack_int2",
    "quant_act", "quant_tie_margin", "int_gemm", "bitlinear", "rope", "rope_mimo",
    "scan_chunked_f64", "scan_seq", "ternary", "local_ent", "local_ent_mimo",
    "global_rel_bias", "global_ent", "siso_forward", "siso_decode",
    "mimo_forward", "mimo_decode", "alloc_cache", "rmsnorm", "ffn",
    "model_forward", "model_alloc_cache", "sigmoid", "memo_weights",
]


# ---------------------------------------------------------------- numerics
def bf16_round(x):
    """Round float32 values to the nearest bfloat16 (ties to even), as torch does."""
    a = np.ascontiguousarray(np.asarray(x, dtype=F32))
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) & 0xFFFF0000
    out = u.astype(np.uint32).view(F32).copy()
    out[nan] = np.nan
    return out


def cast(x, dtype):
    x = np.asarray(x, dtype=F32)
    return bf16_round(x) if dtype == "bfloat16" else x


def sigmoid(x):
    x = np.asarray(x, dtype=F32)
    return (F32(1.0) / (F32(1.0) + np.exp(-x))).astype(F32)


# ---------------------------------------------------------------- BitLinear
def ternary_weight(w, eps=1e-5, dtype="float32", per_row=False):
    """Ternary codes of ``BitLinear.quantized_weight`` (tesm_ssm/modules/tesm.py:211-215).

    scale = 1 / max(mean|W|, eps) in the weight dtype; t = clamp(round(W*scale), -1, 1)
    (round half to even); the dequantised weight is t / scale == t * fl(1/scale).
    ``per_row`` restates the per-row absmean variant (tesm.py:261,270), used only by
    the standalone BitLinear microbench.
    Returns (t int8 (N,K), scale float32 scalar or (N,), deq float32 scalar or (N,)).
    """
    w = cast(w, dtype)
    a = np.abs(w.astype(F64))
    m = a.mean(axis=1) if per_row else a.mean()
    m = cast(np.maximum(np.asarray(m, dtype=F32), F32(eps)), dtype)
    scale = cast(F32(1.0) / m, dtype)
    prod = cast(w * (scale[:, None] if per_row else scale), dtype)
    t = np.clip(np.rint(prod), -1, 1).astype(np.int8)
    deq = cast(F32(1.0) / scale, dtype)
    return t, np.asarray(scale, dtype=F32), np.asarray(deq, dtype=F32)


def pack_int2(t):
    """Pack ternary codes four per byte (tesm_ssm/utils/int2_quantization.py:21-60).

    code = t + 1 (-1->0b00, 0->0b01, +1->0b10); byte = v0 | v1<<2 | v2<<4 | v3<<6 with
    v0 the lowest column; K padded to a multiple of 4 with code 1.
    """
    t = np.asarray(t, dtype=np.int8)
    n, k = t.shape
    enc = (t.astype(np.int16) + 1).astype(np.uint8)
    if k % 4:
        enc = np.concatenate([enc, np.ones((n, 4 - k % 4), np.uint8)], axis=1)
    enc = enc.reshape(n, -1, 4)
    return (enc[:, :, 0] | (enc[:, :, 1] << 2) | (enc[:, :, 2] << 4) | (enc[:, :, 3] << 6)).astype(np.uint8)


def unpack_int2(packed, k=None):
    """Inverse of :func:`pack_int2` (int2_quantization.py:63-93) returning int8 codes."""
    p = np.asarray(packed, dtype=np.uint8)
    v = np.stack([(p >> (2 * i)) & 3 for i in range(4)], axis=2).astype(np.int8) - 1
    v = v.reshape(p.shape[0], -1)
    return v if k is None else v[:, :k]


def quant_act(x, eps=1e-5, dtype="float32", amax=None):
    """int8 codes of ``BitLinear.quantized_input`` (tesm.py:206-209).

    s = 127 / max(max|x|, eps) in the input dtype -- torch evaluates ``127 / t`` as
    ``t.reciprocal() * 127`` (two roundings); c = clamp(round(x*s), -128, 127).
    ``amax`` (optional, per row) replaces max|x|: the quantisation of a column slice of a wider
    row with the full row's maximum (tensor-parallel shards).
    Returns (codes int8 (..., K), s float32 (...,)).
    """
    x = cast(x, dtype)
    ax = np.abs(x).max(axis=-1) if amax is None else np.asarray(amax, dtype=F32)
    mx = cast(np.maximum(ax, F32(eps)).astype(F32), dtype)
    s = cast(cast(F32(1.0) / mx, dtype) * F32(127.0), dtype)
    prod = cast(x * s[..., None], dtype)
    c = np.clip(np.rint(prod), -128, 127).astype(np.int8)
    return c, s.astype(F32)


def quant_tie_margin(x, eps=1e-5, dtype="float32"):
    """Per-row distance of x*s to the nearest rounding tie (k + 0.5) in the int8 activation
    quantisation of :func:`quant_act`.  A row whose margin is below the fp32 error of x*s
    (~1e-5) can legitimately round one element to a neighbouring code."""
    x = cast(x, dtype)
    mx = cast(np.maximum(np.abs(x).max(axis=-1), F32(eps)).astype(F32), dtype)
    s = cast(cast(F32(1.0) / mx, dtype) * F32(127.0), dtype)
    p = np.abs(cast(x * s[..., None], dtype)).astype(np.float64)
    return np.abs(p - np.floor(p) - 0.5).min(axis=-1)


def int_gemm(codes, t):
    """Exact integer product sum_k c[m,k] * t[n,k] (the int32 accumulator)."""
    # a floating-point GEMM is exact here: |c*t| <= 128, so every partial sum is an integer
    # below K*128; fp32 holds those exactly while K*128 < 2^24, fp64 beyond
    K = codes.shape[-1]
    ft = np.float32 if K * 128 < 2 ** 24 else np.float64
    c = np.asarray(codes, dtype=ft).reshape(-1, K)
    acc = c @ np.asarray(t, dtype=ft).T
    assert np.abs(acc).max(initial=0) < 2 ** 31
    return np.rint(acc).astype(np.int32).reshape(*codes.shape[:-1], t.shape[0])


_WEIGHT_MEMO = None


def memo_weights(enable=True):
    """Cache ternary weights by array identity, like the reference's eval-mode cache
    (tesm.py:226-236); used when timing the oracle as a CPU baseline."""
    global _WEIGHT_MEMO
    _WEIGHT_MEMO = {} if enable else None


def _ternary_cached(w, eps, dtype, per_row):
    if _WEIGHT_MEMO is None:
        return ternary_weight(w, eps, dtype, per_row)
    key = (id(w), eps, dtype, per_row)
    hit = _WEIGHT_MEMO.get(key)
    if hit is None:
        hit = ternary_weight(w, eps, dtype, per_row)
        _WEIGHT_MEMO[key] = hit
    return hit


def bitlinear(x, w, eps=1e-5, dtype="float32", per_row=False, return_acc=False):
    """``BitLinear.forward`` torch rung (tesm.py:287-290 -> F.linear at :275-276).

    y = F.linear(c/s, t*deq) evaluated in float64 and rounded to ``dtype``.
    """
    x = np.asarray(x, dtype=F32)
    t, _, deq = _ternary_cached(w, eps, dtype, per_row)
    c, s = quant_act(x, eps, dtype)
    acc = int_gemm(c, t)
    y = acc.astype(F64) * (1.0 / s.astype(F64))[..., None]
    y = y * (deq.astype(F64) if per_row else F64(deq.reshape(-1)[0]))
    y = cast(y.astype(F32), dtype)
    return (y, acc) if return_acc else y


def bitlinear_codes(codes, inv, w, eps=1e-5, dtype="float32"):
    """:func:`bitlinear` from given int8 activation codes and per-row 1/s (the dequantisation
    of ``BitLinear.quantized_input``, tesm.py:206-209) instead of quantising an input: lets a
    test hand the oracle the exact codes a device kernel quantised, so that rounding ties in
    the quantiser's input cannot make the two sides diverge."""
    t, _, deq = _ternary_cached(w, eps, dtype, False)
    K = t.shape[1]
    acc = int_gemm(np.asarray(codes)[..., :K], t)
    y = acc.astype(F64) * np.asarray(inv, F64)[..., None] * F64(deq.reshape(-1)[0])
    return cast(y.astype(F32), dtype)


def bitlinear_f32out(x, w, eps=1e-5, dtype="float32"):
    """:func:`bitlinear` with the input quantised and the weight ternarised in ``dtype`` but
    the output kept in fp32 (a consumer that fuses the next operation, such as the output
    combine, rounds once after it)."""
    x = np.asarray(x, dtype=F32)
    t, _, deq = _ternary_cached(w, eps, dtype, False)
    c, s = quant_act(x, eps, dtype)
    acc = int_gemm(c, t)
    return (acc.astype(F64) * (1.0 / s.astype(F64))[..., None] * F64(deq.reshape(-1)[0])).astype(F32)


# ---------------------------------------------------------------- layer pieces
def _inv_freq(dim, base):
    """``1.0 / (rope_base ** (2.0 * dim_idx / D))`` in fp32 (tesm.py:787-789): the power rounded
    to fp32 once (evaluated in fp64, i.e. correctly rounded), then an fp32 reciprocal.  This is
    what torch's CPU pow yields for every even D <= 64 (tests/test_oracle_golden.py checks it);
    numpy's own fp32 power differs from it by 1-2 ulp at several indices, which RoPE multiplies
    by the position."""
    ex = (F32(2.0) * np.arange(dim // 2, dtype=F32) / F32(dim)).astype(F32)
    pw = np.power(np.float64(F32(base)), ex.astype(np.float64)).astype(F32)
    return (F32(1.0) / pw).astype(F32)


def rope(x, pos_offset=0, base=10000.0):
    """``TESM_SISO._apply_rope`` (tesm.py:783-793): half-split rotation on (B, L, R)."""
    x = np.asarray(x, dtype=F32)
    L, R = x.shape[-2], x.shape[-1]
    half = R // 2
    pos = np.arange(pos_offset, pos_offset + L, dtype=F32)
    theta = (pos[:, None] * _inv_freq(R, base)[None, :]).astype(F32)
    c, s = np.cos(theta).astype(F32), np.sin(theta).astype(F32)
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1).astype(F32)


def rope_mimo(x, pos_offset=0, base=10000.0):
    """``TESMMIMO_Optimized._apply_rope`` (tesm_mimo.py:210-220) on (B, L, H, R)."""
    x = np.asarray(x, dtype=F32)
    L, R = x.shape[1], x.shape[-1]
    half = R // 2
    pos = np.arange(pos_offset, pos_offset + L, dtype=F32)
    theta = (pos[:, None] * _inv_freq(R, base)[None, :]).astype(F32)
    c, s = np.cos(theta)[:, None, :].astype(F32), np.sin(theta)[:, None, :].astype(F32)
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1).astype(F32)


def scan_chunked_f64(decay, update, h0=None, chunk=16):
    """``TESM_SISO._parallel_state_scan`` torch rung (tesm.py:1091-1164, :1065-1089).

    float64 chunks: A = cumprod(max(a,1e-12)); h = A * (h0 + cumsum(u / max(A,1e-12))).
    Returns (states float64 (B,L,D), final float64 (B,D)).
    """
    a = np.maximum(np.asarray(decay, dtype=F64), 1e-12)
    u = np.asarray(update, dtype=F64)
    B, L, D = a.shape
    h = np.zeros((B, D), F64) if h0 is None else np.asarray(h0, dtype=F64)
    chunk = min(max(chunk, 1), L)
    out = np.empty((B, L, D), F64)
    for c in range(0, L, chunk):
        e = min(c + chunk, L)
        A = np.cumprod(a[:, c:e], axis=1)
        out[:, c:e] = A * (h[:, None, :] + np.cumsum(u[:, c:e] / np.maximum(A, 1e-12), axis=1))
        h = out[:, e - 1]
    return out, h.copy()


def scan_seq(decay, update):
    """``_parallel_state_scan_pytorch_mimo`` (tesm_mimo.py:375-392): h = a*h + u in float32."""
    a = np.asarray(decay, dtype=F32)
    u = np.asarray(update, dtype=F32)
    out = np.empty_like(u)
    h = np.zeros(u[:, 0].shape, F32)
    for t in range(u.shape[1]):
        h = (a[:, t] * h).astype(F32) + u[:, t]
        out[:, t] = h
    return out


def ternary(scores, thr):
    """Eval-mode ``ternary_entanglement`` (tesm.py:695-714): +1 / -1 / 0 by threshold."""
    return np.where(scores > thr, F32(1), np.where(scores < -thr, F32(-1), F32(0))).astype(F32)


def local_ent(q, k, v, bias, thr, return_scores=False):
    """SISO local entanglement torch rung (tesm.py:922-952).

    For lag o in [0, min(W, L)): j = t - o (valid iff j >= 0); score = q_t.k_j / sqrt(R)
    + bias[W-1-o] (``local_entanglement_bias[-window:]`` aligned to the newest position);
    avg_t = sum tern * v_j / max(sum|tern|, 1).
    """
    q = np.asarray(q, F32); k = np.asarray(k, F32); v = np.asarray(v, F32)
    B, L, R = q.shape
    W = bias.shape[-1]
    win = min(W, L)
    inv = F32(1.0 / math.sqrt(R))
    num = np.zeros(v.shape, F64)
    norm = np.zeros((B, L), F64)
    sc_all = np.zeros((B, L, win), F32)
    for o in range(win):
        sc = np.zeros((B, L), F32)
        sc[:, o:] = (np.einsum("blr,blr->bl", q[:, o:], k[:, :L - o]) * inv).astype(F32) + F32(bias[W - 1 - o])
        valid = np.arange(L) >= o
        tern = ternary(sc, thr) * valid[None, :]
        sc_all[:, :, o] = np.where(valid[None, :], sc, np.nan)
        num[:, o:] += tern[:, o:, None] * v[:, :L - o]
        norm += np.abs(tern)
    out = (num / np.maximum(norm, 1.0)[..., None]).astype(F32)
    return (out, sc_all) if return_scores else out


def local_ent_mimo(q, k, v, bias, thr, return_scores=False):
    """MIMO local entanglement torch rung (tesm_mimo.py:525-588), low-temperature branch.

    Lag o uses bias[h, W-1-o].  Quirk kept: for t < W-1 only lags o in [W-1-t, t] take
    part (``window_len = min(W, t+1)`` loop with the ``hist_t < 0`` skip).
    q, k (B,L,H,R); v (B,L,H,D); bias (H,W).
    """
    q = np.asarray(q, F32); k = np.asarray(k, F32); v = np.asarray(v, F32)
    B, L, H, R = q.shape
    W = bias.shape[-1]
    inv = F32(1.0 / math.sqrt(R))
    num = np.zeros(v.shape, F64)
    norm = np.zeros((B, L, H), F64)
    sc_all = np.full((B, L, H, W), np.nan, F32)
    t = np.arange(L)
    for o in range(W):
        if o >= L:
            break
        valid = (t >= o) & (o >= (W - 1 - t))
        sc = np.zeros((B, L, H), F32)
        sc[:, o:] = (np.einsum("blhr,blhr->blh", q[:, o:], k[:, :L - o]) * inv).astype(F32) + bias[None, None, :, W - 1 - o]
        tern = ternary(sc, thr) * valid[None, :, None]
        sc_all[..., o] = np.where(valid[None, :, None], sc, np.nan)
        num[:, o:] += tern[:, o:, :, None] * v[:, :L - o]
        norm += np.abs(tern)
    out = (num / np.maximum(norm, 1.0)[..., None]).astype(F32)
    return (out, sc_all) if return_scores else out


def global_rel_bias(L, embed, scale, bias0):
    """Relative-position bias of global entanglement (tesm.py:970-982), float32.

    rel_bias[i, j] = scale * sum_k e_k (sin + cos)((i-j) * k*pi/1000) + bias0; it depends
    on i - j only, returned as a vector over d = i - j in [-(L-1), L-1] (index d + L - 1).
    """
    d = np.arange(-(L - 1), L, dtype=F32)
    fb = (np.arange(1, len(embed) + 1, dtype=F32) * F32(math.pi) / F32(1000.0)).astype(F32)
    ang = (d[:, None] * fb[None, :]).astype(F32)
    e = np.asarray(embed, F32)
    rb = (np.sin(ang) * e).sum(-1, dtype=F32) + (np.cos(ang) * e).sum(-1, dtype=F32)
    return (rb * F32(scale) + F32(bias0)).astype(F32)


def global_ent(q, k, v, relb_vec, thr, R=None, return_scores=False):
    """Causal global entanglement torch rung (tesm.py:1031-1043).

    scores = q k^T / sqrt(R) + rel_bias; ternary; causal mask; (tern / norm) @ v.
    """
    q = np.asarray(q, F32); k = np.asarray(k, F32); v = np.asarray(v, F32)
    B, L, Rq = q.shape
    R = Rq if R is None else R
    i = np.arange(L)
    rb = relb_vec[(i[:, None] - i[None, :]) + L - 1]
    sc = (np.einsum("bir,bjr->bij", q, k) / F32(math.sqrt(R))).astype(F32) + rb[None]
    tern = ternary(sc, thr) * (i[:, None] >= i[None, :])[None]
    norm = np.maximum(np.abs(tern).sum(-1, keepdims=True), 1.0)
    out = np.einsum("bij,bjd->bid", (tern / norm).astype(F64), v.astype(F64)).astype(F32)
    return (out, sc) if return_scores else out


# ---------------------------------------------------------------- SISO layer
def _split(proj, sizes):
    idx = np.cumsum(sizes)[:-1]
    return np.split(proj, idx, axis=-1)


def alloc_cache(cfg, batch, mimo=False):
    """``allocate_inference_cache`` (tesm.py:620-670; tesm_mimo.py:689-731), non-paged."""
    W = max(cfg["entanglement_window"], 1)
    if mimo:
        H = cfg["n_heads"]
        return {"state": np.zeros((batch, H, cfg["d_state"]), F64), "seq_pos": 0,
                "ent_k_cache": np.zeros((batch, W, H, cfg["ent_rank"]), F32),
                "ent_v_cache": np.zeros((batch, W, H, cfg["d_state"]), F32), "cache_idx": 0}
    return {"state": np.zeros((batch, cfg["d_state"]), F64), "seq_pos": 0,
            "ent_k_cache": np.zeros((batch, W, cfg["ent_rank"]), F32),
            "ent_v_cache": np.zeros((batch, W, cfg["d_state"]), F32), "cache_idx": 0}


def siso_forward(P, cfg, u, cross=None, prev_state=None, cache=None, details=False, in_codes=None, dtype="float32"):
    """``TESM_SISO.forward`` prefill in eval mode (tesm.py:1175-1272), float32 module.

    P: parameter dict with the reference's names; cfg: d_model, d_state, ent_rank,
    entanglement_window, entanglement_threshold, entanglement_scale, bit_eps, rope_base,
    state_scan_chunk_size.  Returns (y, final_state_f64, states) [+ details dict].

    ``dtype="bfloat16"`` gives the layer bf16 activations the way a bf16 module would run
    its BitLinears (tesm.py:206-215 in bf16: weight scale, products and codes rounded to
    bf16; outputs rounded to bf16) while the scan and the entanglement stay in fp32 on the
    bf16 projections; the output combine rounds once.  (The reference's own SISO layer
    cannot run in bf16, tesm.py:944, so this mode exists to check bf16 device paths.)
    """
    Dm, D, R = cfg["d_model"], cfg["d_state"], cfg["ent_rank"]
    eps = cfg.get("bit_eps", 1e-5)
    thr, es = cfg["entanglement_threshold"], cfg["entanglement_scale"]
    W = cfg["entanglement_window"]
    u = np.asarray(u, F32)
    B, L, _ = u.shape
    if in_codes is None:
        proj = bitlinear(u, P["in_proj.weight"], eps, dtype)
    else:  # test hook: in_proj from given (codes, 1/s), see bitlinear_codes
        proj = bitlinear_codes(in_codes[0], in_codes[1], P["in_proj.weight"], eps, dtype).reshape(B, L, -1)
    local, value, decay, write, gate, q, k = _split(proj, [Dm, D, D, D, Dm, R, R])
    value = np.tanh(value).astype(F32)
    decay = sigmoid(decay + P["decay_bias"])
    write = sigmoid(write)
    gate = sigmoid(gate)
    base = cfg.get("rope_base", 10000.0)
    q = rope(q, 0, base)
    k = rope(k, 0, base)
    if cross is not None:
        q = (q + bitlinear(cross, P["cross_layer_q_proj.weight"], eps)).astype(F32)
    update = (write * value).astype(F32)
    st64, final = scan_chunked_f64(decay, update, prev_state, cfg.get("state_scan_chunk_size", 16))
    states = st64.astype(F32)
    if W > 0:
        avg, scores = local_ent(q, k, states, P["local_entanglement_bias"], thr, return_scores=True)
    else:
        rb = global_rel_bias(L, P["global_rel_pos_embed"], P["global_rel_pos_scale"][0], P["global_rel_pos_bias"][0])
        avg, scores = global_ent(q, k, states, rb, thr, R, return_scores=True)
    ent = (states + F32(es) * (avg - states)).astype(F32)
    chg = (ent - states).astype(F32)
    if cache is not None:
        Wc = cache["ent_k_cache"].shape[1]
        cache["state"] = final.copy()
        cache["seq_pos"] = L
        if L >= Wc:
            cache["ent_k_cache"] = k[:, -Wc:].copy()
            cache["ent_v_cache"] = states[:, -Wc:].copy()
        else:
            cache["ent_k_cache"][:, -L:] = k
            cache["ent_v_cache"][:, -L:] = states
        cache["cache_idx"] = 0
    if dtype == "float32":
        sp = bitlinear(np.tanh(ent).astype(F32), P["state_proj.weight"], eps)
        ep = bitlinear(chg, P["ent_proj.weight"], eps)
        y = (local + gate * sp + ep).astype(F32)
    else:
        sp = bitlinear_f32out(np.tanh(ent).astype(F32), P["state_proj.weight"], eps, dtype)
        ep = bitlinear_f32out(chg, P["ent_proj.weight"], eps, dtype)
        y = cast((local + gate * sp + ep).astype(F32), dtype)
    out = bitlinear(y, P["out_proj.weight"], eps, dtype)
    if details:
        tie = np.minimum(np.minimum(quant_tie_margin(np.tanh(ent), eps, dtype), quant_tie_margin(chg, eps, dtype)),
                         quant_tie_margin(y, eps, dtype))
        return out, final, states, dict(proj=proj, q=q, k=k, states=states, avg=avg, ent=ent, chg=chg,
                                        y=y, scores=scores, decay=decay, update=update, tie_margin=tie)
    return out, final, states


def _decode_window(cache, k_vec, v_new, q_vec, bias, thr, R, mimo):
    """Ring-buffer write + ordered window of ``_forward_incremental``.

    tesm.py:1326-1381 (SISO) / tesm_mimo.py:838-894 (MIMO): write at cache_idx, advance
    cache_idx; if the window is full the gather order is slots (idx, idx+1, ...) % W with
    bias[w] (the newest entry first -- the reference's own ordering); otherwise slots
    [0, valid) with bias[W-valid+w] and zero-padding.
    """
    Kc, Vc = cache["ent_k_cache"], cache["ent_v_cache"]
    W = Kc.shape[1]
    idx = cache["cache_idx"]
    Kc[:, idx] = k_vec
    Vc[:, idx] = v_new
    cache["cache_idx"] = (idx + 1) % W
    valid = min(cache["seq_pos"] + 1, W)
    if valid >= W:
        slots = [(idx + w) % W for w in range(W)]
        bidx = list(range(W))
    else:
        slots = list(range(valid))
        bidx = [W - valid + w for w in range(valid)]
    inv = F32(1.0 / math.sqrt(R))
    num = np.zeros(v_new.shape, F64)
    norm = np.zeros(v_new.shape[:-1], F64)
    scs = []
    for s, bi in zip(slots, bidx):
        if mimo:
            sc = (np.einsum("bhr,bhr->bh", q_vec, Kc[:, s]) * inv).astype(F32) + bias[None, :, bi]
        else:
            sc = (np.einsum("br,br->b", q_vec, Kc[:, s]) * inv).astype(F32) + F32(bias[bi])
        scs.append(sc)
        t = ternary(sc, thr)
        num += t[..., None] * Vc[:, s]
        norm += np.abs(t)
    avg = (num / np.maximum(norm, 1.0)[..., None]).astype(F32)
    return avg, np.stack(scs, -1)


def siso_decode(P, cfg, u, cache, cross=None, details=False, in_codes=None, dtype="float32"):
    """``TESM_SISO._forward_incremental`` (tesm.py:1274-1400), one token, float32 module."""
    Dm, D, R = cfg["d_model"], cfg["d_state"], cfg["ent_rank"]
    eps = cfg.get("bit_eps", 1e-5)
    thr, es = cfg["entanglement_threshold"], cfg["entanglement_scale"]
    u = np.asarray(u, F32)
    if in_codes is None:
        proj = bitlinear(u, P["in_proj.weight"], eps, dtype)
    else:
        proj = bitlinear_codes(in_codes[0], in_codes[1], P["in_proj.weight"], eps, dtype).reshape(u.shape[0], 1, -1)
    local, value, decay, write, gate, q, k = _split(proj, [Dm, D, D, D, Dm, R, R])
    value = np.tanh(value).astype(F32)
    decay = sigmoid(decay + P["decay_bias"])
    write = sigmoid(write)
    gate = sigmoid(gate)
    pos = cache["seq_pos"]
    base = cfg.get("rope_base", 10000.0)
    q = rope(q, pos, base)[:, 0]
    k = rope(k, pos, base)[:, 0]
    if cross is not None:
        q = (q + bitlinear(cross, P["cross_layer_q_proj.weight"], eps)).astype(F32)
    new64 = decay[:, 0].astype(F64) * cache["state"] + write[:, 0].astype(F64) * value[:, 0].astype(F64)
    new = new64.astype(F32)
    avg, scs = _decode_window(cache, k, new, q, P["local_entanglement_bias"], thr, R, mimo=False)
    ent = (new + F32(es) * (avg - new)).astype(F32)
    chg = (ent - new).astype(F32)
    cache["state"] = new64
    cache["seq_pos"] += 1
    if dtype == "float32":
        sp = bitlinear(np.tanh(ent), P["state_proj.weight"], eps)
        ep = bitlinear(chg, P["ent_proj.weight"], eps)
        y = (local[:, 0] + gate[:, 0] * sp + ep).astype(F32)
    else:
        sp = bitlinear_f32out(np.tanh(ent), P["state_proj.weight"], eps, dtype)
        ep = bitlinear_f32out(chg, P["ent_proj.weight"], eps, dtype)
        y = cast((local[:, 0] + gate[:, 0] * sp + ep).astype(F32), dtype)
    out = bitlinear(y[:, None], P["out_proj.weight"], eps, dtype)
    if details:
        return out, new64, new, dict(scores=scs, avg=avg, ent=ent, chg=chg)
    return out, new64, new


# ---------------------------------------------------------------- MIMO layer
def mimo_forward(P, cfg, u, cache=None, details=False):
    """``TESMMIMO_Optimized.forward`` prefill, eval, float32 (tesm_mimo.py:914-1062).

    Cross-layer state is ignored by the reference in prefill.  Returns
    (y, final_state_f64 (rank 0), cross_state (B,H,D) = rank-0 last state).
    """
    Dm, D, R, H, Rm = cfg["d_model"], cfg["d_state"], cfg["ent_rank"], cfg["n_heads"], cfg["mimo_rank"]
    eps = cfg.get("bit_eps", 1e-5)
    thr, es = cfg["entanglement_threshold"], cfg["entanglement_scale"]
    u = np.asarray(u, F32)
    B, L, _ = u.shape
    proj = bitlinear(u, P["in_proj.weight"], eps)
    local, value, decay, write, gate, q, k = _split(proj, [Dm, D * H, D * H, D * H, Dm, R * H, R * H])
    decay = sigmoid(decay.reshape(B, L, H, D) + P["decay_bias"][None, None])
    write = sigmoid(write.reshape(B, L, H, D))
    value = np.tanh(value.reshape(B, L, H, D)).astype(F32)
    gate = sigmoid(gate)
    mx, mo = P["mimo_x"], P["mimo_o"]
    base = cfg.get("rope_base", 10000.0)
    q = rope_mimo(q.reshape(B, L, H, R), 0, base)
    k = rope_mimo(k.reshape(B, L, H, R), 0, base)
    bias = P.get("local_entanglement_bias")
    ent = np.zeros((B, L, H, D), F32)
    chg = np.zeros((B, L, H, D), F32)
    states0 = None
    for r in range(Rm):
        upd = ((write * mx[None, None, :, r]).astype(F32) * (value * mx[None, None, :, r]).astype(F32)).astype(F32)
        st = scan_seq(decay, upd)
        if r == 0:
            states0 = st
        if cfg["entanglement_window"] > 0:
            avg = local_ent_mimo(q, k, st, bias, thr)
            e_r = (st + F32(es) * (avg - st)).astype(F32)
        else:
            # global rung (tesm_mimo.py:651-687): heads flattened, sqrt(H*R), no lerp
            rb = global_rel_bias(L, P["global_rel_pos_embed"], P["global_rel_pos_scale"][0],
                                 P["global_rel_pos_bias"][0])
            avg = global_ent(q.reshape(B, L, H * R), k.reshape(B, L, H * R), st.reshape(B, L, H * D), rb, thr,
                             H * R).reshape(B, L, H, D)
            e_r = avg
        c_r = (e_r - st).astype(F32)
        ent = (ent + e_r * mo[None, None, :, r]).astype(F32)
        chg = (chg + c_r * mo[None, None, :, r]).astype(F32)
    final = states0[:, -1].astype(F64)
    if cache is not None:
        Wc = cache["ent_k_cache"].shape[1]
        cache["state"] = final.copy()
        cache["seq_pos"] = L
        if L >= Wc:
            cache["ent_k_cache"] = k[:, -Wc:].copy()
            cache["ent_v_cache"] = states0[:, -Wc:].copy()
        else:
            cache["ent_k_cache"][:, -L:] = k
            cache["ent_v_cache"][:, -L:] = states0[:, -L:]
        cache["cache_idx"] = 0
    sp = bitlinear(np.tanh(ent.reshape(B, L, H * D)), P["state_proj.weight"], eps)
    ep = bitlinear(chg.reshape(B, L, H * D), P["ent_proj.weight"], eps)
    y = (local + gate * sp + ep).astype(F32)
    out = bitlinear(y, P["out_proj.weight"], eps)
    if details:
        tie = np.minimum(np.minimum(quant_tie_margin(np.tanh(ent.reshape(B, L, H * D)), eps),
                                    quant_tie_margin(chg.reshape(B, L, H * D), eps)), quant_tie_margin(y, eps))
        return out, final, states0[:, -1], dict(ent=ent, chg=chg, states0=states0, q=q, k=k, y=y, tie_margin=tie)
    return out, final, states0[:, -1]


def mimo_decode(P, cfg, u, cache, cross=None):
    """``TESMMIMO_Optimized._forward_incremental`` (tesm_mimo.py:753-912).

    mimo_x / mimo_o are not used here by the reference.  cross (B,H,D) is projected per
    head by cross_layer_q_proj.
    """
    Dm, D, R, H = cfg["d_model"], cfg["d_state"], cfg["ent_rank"], cfg["n_heads"]
    eps = cfg.get("bit_eps", 1e-5)
    thr, es = cfg["entanglement_threshold"], cfg["entanglement_scale"]
    u = np.asarray(u, F32)
    B = u.shape[0]
    proj = bitlinear(u, P["in_proj.weight"], eps)
    local, value, decay, write, gate, q, k = _split(proj, [Dm, D * H, D * H, D * H, Dm, R * H, R * H])
    decay = sigmoid(decay.reshape(B, 1, H, D) + P["decay_bias"][None, None])
    write = sigmoid(write.reshape(B, 1, H, D))
    value = np.tanh(value.reshape(B, 1, H, D)).astype(F32)
    gate = sigmoid(gate)
    pos = cache["seq_pos"]
    base = cfg.get("rope_base", 10000.0)
    q = rope_mimo(q.reshape(B, 1, H, R), pos, base)[:, 0]
    k = rope_mimo(k.reshape(B, 1, H, R), pos, base)[:, 0]
    if cross is not None:
        cb = bitlinear(np.asarray(cross, F32).reshape(B * H, D), P["cross_layer_q_proj.weight"], eps)
        q = (q + cb.reshape(B, H, R)).astype(F32)
    new64 = decay[:, 0].astype(F64) * cache["state"] + write[:, 0].astype(F64) * value[:, 0].astype(F64)
    new = new64.astype(F32)
    avg, _ = _decode_window(cache, k, new, q, P["local_entanglement_bias"], thr, R, mimo=True)
    ent = (new + F32(es) * (avg - new)).astype(F32)
    chg = (ent - new).astype(F32)
    cache["state"] = new64
    cache["seq_pos"] += 1
    sp = bitlinear(np.tanh(ent.reshape(B, H * D)), P["state_proj.weight"], eps)
    ep = bitlinear(chg.reshape(B, H * D), P["ent_proj.weight"], eps)
    y = (local[:, 0] + gate[:, 0] * sp + ep).astype(F32)
    out = bitlinear(y[:, None], P["out_proj.weight"], eps)
    return out, new64, new


# ---------------------------------------------------------------- model
def rmsnorm(x, w, eps=1e-5):
    """``RMSNorm.forward`` (tesm_ssm/modules/block.py:14-17), float32."""
    x = np.asarray(x, F32)
    var = (x.astype(F64) ** 2).mean(-1, keepdims=True)
    return (x * (1.0 / np.sqrt(var + eps)).astype(F32) * w).astype(F32)


def ffn(P, x, eps=1e-5, dtype="float32", in_codes=None, return_h=False):
    """``FeedForward.forward`` grouped gate/up path (mixer_seq_simple.py:45-67).  With
    ``dtype="bfloat16"`` the BitLinears take bf16 semantics and silu(g) * u is rounded to bf16
    once (a fused SwiGLU epilogue).  ``in_codes`` = (codes, 1/s) replaces the quantisation of
    x (a test hook, see :func:`bitlinear_codes`)."""
    tg, _, dg = _ternary_cached(P["gate_proj.weight"], eps, dtype, False)
    tu, _, du = _ternary_cached(P["up_proj.weight"], eps, dtype, False)
    if in_codes is None:
        c, s = quant_act(x, eps, dtype)
        inv_s = (1.0 / s.astype(F64))[..., None]
    else:
        c = np.asarray(in_codes[0])[..., :tg.shape[1]]
        inv_s = np.asarray(in_codes[1], F64)[..., None]
    gx = (int_gemm(c, tg).astype(F64) * inv_s * dg).astype(F32)
    ux = (int_gemm(c, tu).astype(F64) * inv_s * du).astype(F32)
    h = cast((gx / (F32(1) + np.exp(-gx)) * ux).astype(F32), dtype)
    out = bitlinear(h, P["down_proj.weight"], eps, dtype)
    return (out, h) if return_h else out


def model_alloc_cache(cfg, batch):
    """``MixerModel.allocate_inference_cache`` (mixer_seq_simple.py:168-169)."""
    return {i: alloc_cache(cfg, batch, cfg.get("use_mimo", False)) for i in range(cfg["n_layer"])}


def model_forward(P, cfg, ids, cache=None, logits_to_keep=0, timings=None):
    """``TESMLMHeadModel.forward`` logits in eval (mixer_seq_simple.py:171-242, :290-345).

    P holds the reference state_dict names (``backbone.layers.{i}.mixer.*`` ...).
    A one-token call with a cache runs every layer incrementally (tesm.py:1188-1191).
    """
    ids = np.asarray(ids)
    B, L = ids.shape
    pos0 = 0
    if cache is not None and L == 1:
        pos0 = cache[0]["seq_pos"]
    emb = P["backbone.embedding.weight"][ids] + P["backbone.position_embedding.weight"][np.arange(pos0, pos0 + L)][None]
    hidden = emb.astype(F32)
    residual = None
    cross = None
    mimo = cfg.get("use_mimo", False)
    neps = cfg.get("norm_epsilon", 1e-5)
    for i in range(cfg["n_layer"]):
        pre = f"backbone.layers.{i}."
        lp = {k[len(pre) + 6:]: v for k, v in P.items() if k.startswith(pre + "mixer.")}
        fp = {k[len(pre) + 4:]: v for k, v in P.items() if k.startswith(pre + "mlp.")}
        residual = hidden if residual is None else (hidden + residual).astype(F32)
        h = rmsnorm(residual, P[pre + "norm.weight"], neps)
        lc = cache[i] if cache is not None else None
        if lc is not None and L == 1:
            if mimo:
                y, _, new = mimo_decode(lp, cfg, h, lc, cross)
                cross = new
            else:
                y, _, new = siso_decode(lp, cfg, h, lc, cross)
                cross = new
        else:
            if mimo:
                y, _, cross = mimo_forward(lp, cfg, h, lc)
            else:
                y, _, states = siso_forward(lp, cfg, h, cross, None, lc)
                cross = states
        residual = (y + residual).astype(F32)
        h2 = rmsnorm(residual, P[pre + "norm2.weight"], neps)
        hidden = ffn(fp, h2)
    residual = (hidden + residual).astype(F32)
    hf = rmsnorm(residual, P["backbone.norm_f.weight"], neps)
    if logits_to_keep > 0:
        hf = hf[:, -logits_to_keep:]
    if timings is not None:
        timings["layers_done"] = time.perf_counter()
    return (hf.astype(F64) @ P["lm_head.weight"].astype(F64).T).astype(F32)
