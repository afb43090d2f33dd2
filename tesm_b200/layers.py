"""Forward paths of the b200 backend, shared by the mirror modules and by the
patch that adds the "b200" rung to the reference classes (integration.py).

Functions read the reference's attribute names off the module they are given,
so the same code serves ``tesm_b200.modules.TESM_SISO`` and the reference's
``tesm_ssm.modules.tesm.TESM_SISO``.  All arithmetic runs in libtesm_b200.so;
torch is used for allocation, views, and the dense tied lm_head (cuBLAS).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import ops
from . import parallel
from ._lib import TesmError
from .paged_cache import PagedStateCache, snapshot_if_due

B200 = "b200"


def require_b200(mod, x, what):
    """Reference-style strict backend check (tesm.py:279-285): no fallback path."""
    backend = getattr(mod, "kernel_backend", B200)
    ok = (backend == B200 and isinstance(x, torch.Tensor) and x.is_cuda and not mod.training
          and not torch.is_grad_enabled())
    if not ok:
        why = []
        if backend != B200:
            why.append(f"backend {backend!r} is not served by tesm_b200")
        if isinstance(x, torch.Tensor) and not x.is_cuda:
            why.append("input is not a CUDA tensor")
        if mod.training:
            why.append("module is in training mode (b200 is inference-only: call .eval())")
        if torch.is_grad_enabled():
            why.append("grad mode is enabled (use torch.no_grad())")
        raise RuntimeError(f"kernel_backend='{backend}' specified but {what} kernel not available: "
                           + "; ".join(why) + ". The b200 backend has no CPU or autograd fallback.")


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().float().contiguous()


def _param_cache(mod, name: str) -> torch.Tensor:
    """fp32 contiguous device copy of a small parameter, refreshed when it changes."""
    p = getattr(mod, name)
    store = mod.__dict__.setdefault("_b200_params", {})
    key = (p.data_ptr(), p._version, p.dtype)
    hit = store.get(name)
    if hit is None or hit[0] != key:
        hit = (key, _f32(p))
        store[name] = hit
    return hit[1]


# ------------------------------------------------------------------ BitLinear
def packed_weight(lin, need_tern: bool = False) -> ops.PackedWeight:
    """Device ternary weight of a BitLinear, rebuilt whenever the weight changes
    (mirrors the eval-mode cache keyed on weight._version, tesm.py:226-236).  A weight imported
    from an INT2 export (``tesm_b200.int2``) takes precedence over the latent weight."""
    imported = lin.__dict__.get("_b200_int2")
    if imported is not None:
        return imported
    w = lin.weight
    key = (w.data_ptr(), w._version, w.dtype, tuple(w.shape))
    cache = lin.__dict__.get("_b200")
    if cache is None or cache[0] != key:
        wc = w.detach()
        if wc.stride(1) != 1:
            wc = wc.contiguous()
        cache = (key, ops.pack_weight(wc, lin.bit_eps, per_row=False, with_tern=False), wc)
        lin.__dict__["_b200"] = cache
    pw = cache[1]
    if need_tern:
        ops.ensure_tern(pw, cache[2])
    return pw


def linear_q(lin, q: ops.QuantAct, out_dtype, out=None):
    """BitLinear on pre-quantised activations."""
    if lin.bias is not None:
        raise TesmError("tesm_b200: BitLinear bias is not on the reference hot path (bias=False everywhere)")
    pw = packed_weight(lin, need_tern=q.layout == ops.LAYOUT_ROWMAJOR)
    return ops.matmul_q(q, pw, out_dtype, out)


def linear(lin, x2d: torch.Tensor, out_dtype=None, out=None):
    if x2d.stride(-1) != 1:
        x2d = x2d.contiguous()
    return linear_q(lin, ops.quantize(x2d, lin.bit_eps), out_dtype or x2d.dtype, out)


def bitlinear_forward(lin, x):
    """``BitLinear.forward`` (tesm.py:287-290): output in the input dtype."""
    shp = x.shape
    y = linear(lin, x.reshape(-1, shp[-1]))
    return y.reshape(*shp[:-1], lin.out_features)


# ------------------------------------------------------------------ caches
def _new_cache(batch, W, state_shape, kshape, vshape, dev, dtype):
    return {
        "use_paged": False,
        "state": torch.zeros(batch, *state_shape, device=dev, dtype=torch.float64),
        "seq_pos": 0,
        "ent_k_cache": torch.zeros(batch, W, *kshape, device=dev, dtype=torch.float32),
        "ent_v_cache": torch.zeros(batch, W, *vshape, device=dev, dtype=torch.float32),
        "cache_idx": 0,
        "cache_filled": False,
        "_ctl": torch.zeros(3, device=dev, dtype=torch.int32),
        "_ctl_host": (0, 0),
    }


def _with_pages(cache, kwargs, max_seqlen, batch, d_state, ent_rank, W, dev):
    """``use_paged_cache=True`` with max_seqlen > 1024 adds the paged snapshot store
    (tesm.py:636-657; page_size and max_gpu_pages keyword arguments as the reference)."""
    if kwargs.get("use_paged_cache", False) and max_seqlen > 1024:
        cache["use_paged"] = True
        cache["paged_cache"] = PagedStateCache(batch_size=batch, d_state=d_state, ent_rank=ent_rank, window=W,
                                               page_size=kwargs.get("page_size", 512),
                                               max_gpu_pages=kwargs.get("max_gpu_pages", 100), device=dev)
    return cache


def siso_alloc_cache(mod, batch_size, max_seqlen, dtype=None, **kwargs):
    """Cache with the reference's keys (tesm.py:620-670); the recurrent state is fp64 like the
    reference, the window caches fp32 on the device, plus a device (seq_pos, cache_idx) pair
    used by the decode kernel."""
    W = max(mod.entanglement_window, 1)
    dev = mod.out_proj.weight.device
    c = _new_cache(batch_size, W, (mod.d_state,), (mod.ent_rank,), (mod.d_state,), dev, dtype)
    return _with_pages(c, kwargs, max_seqlen, batch_size, mod.d_state, mod.ent_rank, W, dev)


def mimo_alloc_cache(mod, batch_size, max_seqlen, dtype=None, **kwargs):
    """MIMO cache (tesm_mimo.py:719-731): state (B, H, D), windows (B, W, H, R|D)."""
    W = max(mod.entanglement_window, 1)
    H = mod.n_heads
    dev = mod.out_proj.weight.device
    c = _new_cache(batch_size, W, (H, mod.d_state), (H, mod.ent_rank), (H, mod.d_state), dev, dtype)
    return _with_pages(c, kwargs, max_seqlen, batch_size, H * mod.d_state, H * mod.ent_rank, W, dev)


def _prepare_cache(cache, dev):
    """Accept caches allocated by either implementation; keep the device control word in
    sync with the host ints the reference API exposes."""
    for k in ("ent_k_cache", "ent_v_cache"):
        t = cache[k]
        if t.dtype != torch.float32 or not t.is_contiguous() or t.device != dev:
            cache[k] = t.to(device=dev, dtype=torch.float32).contiguous()
    st = cache["state"]
    if st.dtype != torch.float64 or not st.is_contiguous() or st.device != dev:
        cache["state"] = st.to(device=dev, dtype=torch.float64).contiguous()
    if "_ctl" not in cache:
        cache["_ctl"] = torch.zeros(3, device=dev, dtype=torch.int32)
        cache["_ctl_host"] = None
    host = (int(cache["seq_pos"]), int(cache.get("cache_idx", 0)))
    if cache.get("_ctl_host") != host:
        cache["_ctl"].copy_(torch.tensor([host[0], host[1], 0], dtype=torch.int32))
        cache["_ctl_host"] = host
    return cache


def _advance_host(cache, W):
    pos, idx = int(cache["seq_pos"]), int(cache.get("cache_idx", 0))
    cache["seq_pos"] = pos + 1
    cache["cache_idx"] = (idx + 1) % W
    cache["_ctl_host"] = (pos + 1, (idx + 1) % W)


def _set_prefilled(cache, L):
    cache["seq_pos"] = L
    cache["cache_idx"] = 0
    cache["_ctl_host"] = (L, 0)


# ------------------------------------------------------------------ SISO layer
def _as_quant(mod, u2d):
    return u2d if isinstance(u2d, ops.QuantAct) else ops.quantize(u2d, mod.in_proj.bit_eps)


def _out_proj(mod, y, act_dtype):
    """out_proj (tesm.py:1261); row-parallel across ranks when tensor parallelism is enabled."""
    tp = parallel.get_tp(mod)
    if tp is not None:
        return parallel.out_proj_tp(mod, y, act_dtype, tp)
    return linear(mod.out_proj, y, act_dtype)


def _tail(mod, proj, M, C, Rc, tanh_e, chg, act_dtype):
    """state_proj / ent_proj, output combine and out_proj (tesm.py:1255-1261; MIMO
    tesm_mimo.py:1040-1052): the int8 codes of tanh(ent) and ent - s side by side, then one
    dual-accumulator GEMM with the combine epilogue (as the SISO window path does)."""
    Dm = mod.d_model
    dev = proj.device
    tern, deq1, deq2, Dp = combine_weight(mod)
    codes = torch.empty(M, 2 * Dp, device=dev, dtype=torch.int8)
    inv1 = torch.empty(M, device=dev, dtype=torch.float32)
    inv2 = torch.empty(M, device=dev, dtype=torch.float32)
    ops.quant_act_into(tanh_e.reshape(M, C), mod.state_proj.bit_eps, codes, 0, inv1)
    ops.quant_act_into(chg.reshape(M, C), mod.ent_proj.bit_eps, codes, Dp, inv2)
    y = torch.empty(M, Dm, device=dev, dtype=act_dtype)
    ops.gemm_combine(codes, Dp, inv1, inv2, tern, deq1, deq2, proj, 0, Dm + 3 * C, M, Dm, y)
    return _out_proj(mod, y, act_dtype)


def combine_weight(mod):
    """[state_proj | ent_proj] ternary rows side by side (each half D rounded up to 128, zero
    padded) for the dual-accumulator combine GEMM, plus the two dequantisation scalars."""
    sw, ew = mod.state_proj.weight, mod.ent_proj.weight
    key = (sw.data_ptr(), sw._version, ew.data_ptr(), ew._version, id(mod.state_proj.__dict__.get("_b200_int2")),
           id(mod.ent_proj.__dict__.get("_b200_int2")))
    hit = mod.__dict__.get("_b200_comb")
    if hit is None or hit[0] != key:
        ps = packed_weight(mod.state_proj, need_tern=True)
        pe = packed_weight(mod.ent_proj, need_tern=True)
        D = ps.K
        Dp = ops.round_up(D, 128)
        tern = torch.cat([ps.tern[:, :Dp], pe.tern[:, :Dp]], dim=1).contiguous()
        hit = (key, tern, ps.deq, pe.deq, Dp)
        mod.__dict__["_b200_comb"] = hit
    return hit[1:]


def siso_prefill(mod, u, cross_layer_state=None, prev_state=None, cache=None, act_dtype=None, shape=None):
    """``TESM_SISO.forward`` prefill in eval (tesm.py:1175-1272).  ``u`` is (B, L, Dm) or a
    pre-quantised QuantAct with ``shape=(B, L)``."""
    B, L = shape if shape is not None else u.shape[:2]
    act_dtype = act_dtype or u.dtype
    Dm, D, R, W = mod.d_model, mod.d_state, mod.ent_rank, mod.entanglement_window
    M = B * L
    q = _as_quant(mod, u if isinstance(u, ops.QuantAct) else u.reshape(M, Dm))
    tp = parallel.mixer_tp(mod)
    if tp is not None:
        return parallel.siso_prefill_tp(mod, q, (B, L), cross_layer_state, prev_state, cache, act_dtype, tp)
    dev = q.codes.device
    proj = linear_q(mod.in_proj, q, act_dtype)
    cross_bias = None
    if cross_layer_state is not None:
        cross_bias = linear(mod.cross_layer_q_proj, cross_layer_state.reshape(M, D).float(), torch.float32)
    states = torch.empty(M, D, device=dev, dtype=torch.float32)
    fin32 = torch.empty(B, D, device=dev, dtype=torch.float32)
    fin64 = torch.empty(B, D, device=dev, dtype=torch.float64)
    h0 = prev_state.to(device=dev, dtype=torch.float64).contiguous() if prev_state is not None else None
    ops.siso_scan(proj, B, L, Dm, D, R, _param_cache(mod, "decay_bias"), h0, states, fin32, fin64,
                  mod.state_scan_chunk_size)
    thr, es, base = mod.entanglement_threshold, mod.entanglement_scale, mod.rope_base
    fused = W > 0 and M > ops.GEMV_MAX_M and W in (4, 8, 16, 32)
    if fused:
        # entanglement -> int8 codes -> one dual-accumulator GEMM with the combine epilogue
        codes, inv1, inv2, Dp = ops.siso_local_ent_codes(
            proj, B, L, Dm, D, R, W, cross_bias, _param_cache(mod, "local_entanglement_bias"), states, thr, es,
            base, act_dtype, mod.state_proj.bit_eps, mod.ent_proj.bit_eps)
    else:
        tanh_e = torch.empty(M, D, device=dev, dtype=act_dtype)
        chg = torch.empty(M, D, device=dev, dtype=act_dtype)
    if not fused and W > 0:
        ops.siso_local_ent(proj, B, L, Dm, D, R, W, cross_bias, _param_cache(mod, "local_entanglement_bias"), states,
                           thr, es, base, tanh_e, chg)
    elif not fused:
        relb = ops.global_relbias(_param_cache(mod, "global_rel_pos_embed"), float(mod.global_rel_pos_scale),
                                  float(mod.global_rel_pos_bias), L)
        ops.siso_global_ent(proj, B, L, Dm, D, R, cross_bias, relb, states, thr, es, base, tanh_e, chg)
    if cache is not None and "state" in cache:
        _prepare_cache(cache, dev)
        ops.cache_fill(proj, states, 1, B, L, Dm, 1, D, R, cache["ent_k_cache"].shape[1], base, fin64,
                       cache["state"], cache["ent_k_cache"], cache["ent_v_cache"], cache["_ctl"])
        _set_prefilled(cache, L)
    if fused:
        tern, deq1, deq2, _ = combine_weight(mod)
        y = torch.empty(M, Dm, device=dev, dtype=act_dtype)
        ops.gemm_combine(codes, Dp, inv1, inv2, tern, deq1, deq2, proj, 0, Dm + 3 * D, M, Dm, y)
        out = _out_proj(mod, y, act_dtype)
    else:
        out = _tail(mod, proj, M, D, R, tanh_e, chg, act_dtype)
    mod.last_entanglement_map = None
    mod.last_entanglement_stats = None
    mod._last_cross_layer_state = states.view(B, L, D)
    mod._last_scan_state_f64 = fin64
    return out.view(B, L, Dm), fin64


def _state_out(cache):
    """The state a decode step returns: a snapshot (the reference returns each step's new fp64
    state as its own tensor, tesm.py:1385-1400, while the cache here is updated in place), or
    None for callers that discard it (decode graphs, generate)."""
    return None if cache.get("_b200_no_state_out") else cache["state"].clone()


def siso_decode(mod, u, cache, cross_layer_state=None, act_dtype=None, shape=None):
    """``TESM_SISO._forward_incremental`` (tesm.py:1274-1400): one token per sequence."""
    B = shape[0] if shape is not None else u.shape[0]
    act_dtype = act_dtype or u.dtype
    Dm, D, R = mod.d_model, mod.d_state, mod.ent_rank
    q = _as_quant(mod, u if isinstance(u, ops.QuantAct) else u.reshape(B, Dm))
    tp = parallel.mixer_tp(mod)
    if tp is not None:
        return parallel.siso_decode_tp(mod, q, B, cache, cross_layer_state, act_dtype, tp)
    dev = q.codes.device
    _prepare_cache(cache, dev)
    snapshot_if_due(cache)
    W = cache["ent_k_cache"].shape[1]
    proj = linear_q(mod.in_proj, q, act_dtype)
    # the cross-layer query bias is computed inside the step kernel (cross_layer_q_proj on the
    # previous layer's fp32 state row)
    xstate = xq = None
    if cross_layer_state is not None:
        xstate = cross_layer_state.reshape(B, D)
        if xstate.dtype != torch.float32 or not xstate.is_contiguous():
            xstate = xstate.float().contiguous()
        xq = packed_weight(mod.cross_layer_q_proj, need_tern=True)
    new_state = torch.empty(B, D, device=dev, dtype=torch.float32)
    # the step emits the int8 codes of tanh(ent) | ent - s; state_proj, ent_proj and the combine
    # then run as one dual-accumulator GEMM, as in prefill
    codes, inv1, inv2, Dp = ops.siso_decode_step_codes(
        proj, B, Dm, D, R, W, _param_cache(mod, "decay_bias"), _param_cache(mod, "local_entanglement_bias"),
        None, cache["state"], cache["ent_k_cache"], cache["ent_v_cache"], cache["_ctl"],
        mod.entanglement_threshold, mod.entanglement_scale, mod.rope_base, act_dtype, mod.state_proj.bit_eps,
        mod.ent_proj.bit_eps, new_state, xstate, xq, mod.cross_layer_q_proj.bit_eps if xq is not None else 0.0)
    _advance_host(cache, W)
    tern, deq1, deq2, _ = combine_weight(mod)
    y = torch.empty(B, Dm, device=dev, dtype=act_dtype)
    ops.gemm_combine(codes, Dp, inv1, inv2, tern, deq1, deq2, proj, 0, Dm + 3 * D, B, Dm, y)
    out = _out_proj(mod, y, act_dtype)
    mod._last_cross_layer_state = new_state
    return out.view(B, 1, Dm), _state_out(cache)


# ------------------------------------------------------------------ MIMO layer
def mimo_prefill(mod, u, cache=None, act_dtype=None, shape=None):
    """``TESMMIMO_Optimized.forward`` prefill in eval (tesm_mimo.py:914-1062)."""
    B, L = shape if shape is not None else u.shape[:2]
    act_dtype = act_dtype or u.dtype
    Dm, D, R, H, RM, W = mod.d_model, mod.d_state, mod.ent_rank, mod.n_heads, mod.mimo_rank, mod.entanglement_window
    C, M = H * D, B * L
    q = _as_quant(mod, u if isinstance(u, ops.QuantAct) else u.reshape(M, Dm))
    tp = parallel.mixer_tp(mod)
    if tp is not None:
        return parallel.mimo_prefill_tp(mod, q, (B, L), cache, act_dtype, tp)
    dev = q.codes.device
    proj = linear_q(mod.in_proj, q, act_dtype)
    states = torch.empty(M, RM, C, device=dev, dtype=torch.float32)
    fin32 = torch.empty(B, C, device=dev, dtype=torch.float32)
    fin64 = torch.empty(B, C, device=dev, dtype=torch.float64)
    ops.mimo_scan(proj, B, L, Dm, H, D, R, RM, _param_cache(mod, "decay_bias"), _param_cache(mod, "mimo_x"), states,
                  fin32, fin64)
    tanh_e = torch.empty(M, C, device=dev, dtype=act_dtype)
    chg = torch.empty(M, C, device=dev, dtype=act_dtype)
    if W > 0 and mod.local_entanglement_bias is not None:
        ops.mimo_local_ent(proj, B, L, Dm, H, D, R, RM, W, _param_cache(mod, "local_entanglement_bias"),
                           _param_cache(mod, "mimo_o"), states, mod.entanglement_threshold, mod.entanglement_scale,
                           mod.rope_base, True, tanh_e, chg)
    else:
        relb = ops.global_relbias(_param_cache(mod, "global_rel_pos_embed"), float(mod.global_rel_pos_scale),
                                  float(mod.global_rel_pos_bias), L)
        ops.mimo_global_ent(proj, B, L, Dm, H, D, R, RM, relb, _param_cache(mod, "mimo_o"), states,
                            mod.entanglement_threshold, mod.rope_base, tanh_e, chg)
    if cache is not None and "state" in cache:
        _prepare_cache(cache, dev)
        ops.cache_fill(proj, states, RM, B, L, Dm, H, D, R, cache["ent_k_cache"].shape[1], mod.rope_base, fin64,
                       cache["state"], cache["ent_k_cache"], cache["ent_v_cache"], cache["_ctl"])
        _set_prefilled(cache, L)
    out = _tail(mod, proj, M, C, H * R, tanh_e, chg, act_dtype)
    mod.last_entanglement_map = None
    mod._last_cross_layer_state = states.view(B, L, RM, H, D)[:, -1, 0]
    final = fin64.view(B, H, D)
    mod._last_scan_state_f64 = final
    return out.view(B, L, Dm), final


def mimo_decode(mod, u, cache, cross_layer_state=None, act_dtype=None, shape=None):
    """``TESMMIMO_Optimized._forward_incremental`` (tesm_mimo.py:753-912)."""
    B = shape[0] if shape is not None else u.shape[0]
    act_dtype = act_dtype or u.dtype
    Dm, D, R, H = mod.d_model, mod.d_state, mod.ent_rank, mod.n_heads
    C = H * D
    q = _as_quant(mod, u if isinstance(u, ops.QuantAct) else u.reshape(B, Dm))
    tp = parallel.mixer_tp(mod)
    if tp is not None:
        return parallel.mimo_decode_tp(mod, q, B, cache, cross_layer_state, act_dtype, tp)
    dev = q.codes.device
    _prepare_cache(cache, dev)
    snapshot_if_due(cache)
    W = cache["ent_k_cache"].shape[1]
    proj = linear_q(mod.in_proj, q, act_dtype)
    cross_bias = None
    if cross_layer_state is not None:
        cs = cross_layer_state
        if cs.dim() != 3:
            raise TesmError("tesm_b200: MIMO decode expects a (B, n_heads, d_state) cross-layer state")
        cross_bias = linear(mod.cross_layer_q_proj, cs.reshape(B * H, D).float(), torch.float32)
    tanh_e = torch.empty(B, C, device=dev, dtype=act_dtype)
    chg = torch.empty(B, C, device=dev, dtype=act_dtype)
    new_state = torch.empty(B, C, device=dev, dtype=torch.float32)
    ops.decode_step(proj, B, Dm, H, D, R, W, _param_cache(mod, "decay_bias"),
                    _param_cache(mod, "local_entanglement_bias"), cross_bias, cache["state"], cache["ent_k_cache"],
                    cache["ent_v_cache"], cache["_ctl"], mod.entanglement_threshold, mod.entanglement_scale,
                    mod.rope_base, tanh_e, chg, new_state)
    _advance_host(cache, W)
    out = _tail(mod, proj, B, C, H * R, tanh_e, chg, act_dtype)
    mod._last_cross_layer_state = new_state.view(B, H, D)
    return out.view(B, 1, Dm), _state_out(cache)


def _is_mimo(mixer):
    return hasattr(mixer, "mimo_rank") and hasattr(mixer, "n_heads")


def mixer_forward(mixer, q_or_u, shape, act_dtype, inference_params=None, cross_layer_state=None, prev_state=None):
    """Dispatch a mixer call the way ``TESM_SISO.forward`` / ``TESMMIMO_Optimized.forward`` do."""
    B, L = shape
    cache = None
    if inference_params is not None:
        cache = inference_params.get("state_cache")
    mimo = _is_mimo(mixer)
    if cache is not None and "state" in cache and L == 1:
        if mimo:
            return mimo_decode(mixer, q_or_u, cache, cross_layer_state, act_dtype, shape)
        return siso_decode(mixer, q_or_u, cache, cross_layer_state, act_dtype, shape)
    if mimo:
        return mimo_prefill(mixer, q_or_u, cache, act_dtype, shape)
    return siso_prefill(mixer, q_or_u, cross_layer_state, prev_state, cache, act_dtype, shape)


# ------------------------------------------------------------------ norms / blocks / FFN
def rmsnorm(mod, x):
    """``RMSNorm.forward`` (block.py:14-17) on the device."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1]).contiguous()
    y = torch.empty_like(x2)
    ops.add_rmsnorm_quant(x2, None, None, _param_cache(mod, "weight"), mod.eps, 0.0, None, y)
    return y.view(shp)


def _norm_eps(norm):
    return getattr(norm, "eps", 1e-5)


def _norm_quant(norm, x2d, residual, residual_out, qeps):
    if not hasattr(norm, "weight") or norm.__class__.__name__ == "LayerNorm":
        raise TesmError("tesm_b200: only RMSNorm (rms_norm=True) blocks are supported")
    q = ops.alloc_quant(x2d.shape[0], x2d.shape[1], x2d.device)
    ops.add_rmsnorm_quant(x2d, residual, residual_out, _param_cache(norm, "weight"), _norm_eps(norm), qeps, q)
    return q


SWIGLU_BLK = 128


def ffn_packed(ffn):
    """Fused gate/up weight of one FeedForward (mixer_seq_simple.py:45-57): each projection keeps
    its own per-tensor ternary scale, expressed as a per-row dequantisation vector.  When
    d_intermediate % 128 == 0 the rows are interleaved in blocks of 128 ([gate | up] per block)
    so the tensor-core GEMM applies the SiLU gate in its epilogue."""
    g, u = ffn.gate_proj.weight, ffn.up_proj.weight
    gi, ui = ffn.gate_proj.__dict__.get("_b200_int2"), ffn.up_proj.__dict__.get("_b200_int2")
    key = (g.data_ptr(), g._version, u.data_ptr(), u._version, id(gi), id(ui))
    hit = ffn.__dict__.get("_b200_gu")
    if (hit is None or hit[0] != key) and (gi is not None or ui is not None):
        # imported INT2 weights: interleave the two imported (or packed latent) weights' rows
        pg, pu = packed_weight(ffn.gate_proj, True), packed_weight(ffn.up_proj, True)
        Fd, K = pg.N, pg.K
        dev = pg.packed.device
        blk = SWIGLU_BLK if Fd % SWIGLU_BLK == 0 else 0
        f = torch.arange(Fd, device=dev)
        packed = torch.empty(2 * Fd, pg.packed.shape[1], device=dev, dtype=torch.uint8)
        tern = torch.empty(2 * Fd, pg.tern.shape[1], device=dev, dtype=torch.int8)
        deq = torch.empty(2 * Fd, device=dev, dtype=torch.float32)
        for i, pw_i in enumerate((pg, pu)):
            dst = (f // blk) * 2 * blk + i * blk + f % blk if blk else f + i * Fd
            packed[dst] = pw_i.packed
            tern[dst] = pw_i.tern
            deq[dst] = pw_i.deq.expand(Fd)
        hit = (key, ops.PackedWeight(packed, tern, deq.clone(), deq, 2 * Fd, K, True), blk)
        ffn.__dict__["_b200_gu"] = hit
    if hit is None or hit[0] != key:
        Fd, K = g.shape
        Kp = ops.round_up(K, 256)
        dev = g.device
        blk = SWIGLU_BLK if Fd % SWIGLU_BLK == 0 else 0
        packed = torch.empty(2 * Fd, Kp // 4, device=dev, dtype=torch.uint8)
        tern = torch.empty(2 * Fd, Kp, device=dev, dtype=torch.int8)
        scale = torch.empty(2, device=dev, dtype=torch.float32)
        deq2 = torch.empty(2, device=dev, dtype=torch.float32)
        tmp_p = torch.empty(Fd, Kp // 4, device=dev, dtype=torch.uint8)
        tmp_t = torch.empty(Fd, Kp, device=dev, dtype=torch.int8)
        rows = torch.arange(2 * Fd, device=dev)
        for i, w in enumerate((g, u)):
            wc = w.detach().contiguous()
            ops.pack_into(wc, ffn.gate_proj.bit_eps, tmp_p, tmp_t, scale[i:i + 1], deq2[i:i + 1])
            f = torch.arange(Fd, device=dev)
            dst = (f // blk) * 2 * blk + i * blk + f % blk if blk else f + i * Fd
            packed[dst] = tmp_p
            tern[dst] = tmp_t
            rows[dst] = i
        deq = deq2[rows]
        pw = ops.PackedWeight(packed, tern, deq.clone(), deq, 2 * Fd, K, True)
        hit = (key, pw, blk)
        ffn.__dict__["_b200_gu"] = hit
    return hit[1], hit[2]


def ffn_q(ffn, q: ops.QuantAct, act_dtype):
    """``FeedForward.forward`` on pre-quantised input (mixer_seq_simple.py:59-67)."""
    tp = parallel.get_tp(ffn)
    if tp is not None:
        return parallel.ffn_q_tp(ffn, q, act_dtype, tp)
    pw, blk = ffn_packed(ffn)
    Fd = ffn.gate_proj.out_features
    if blk and q.layout == ops.LAYOUT_ROWMAJOR:
        h = ops.gemm_swiglu(q, pw, act_dtype)
    else:
        gu = ops.matmul_q(q, pw, act_dtype)
        h = torch.empty(q.M, Fd, device=gu.device, dtype=act_dtype)
        ops.silu_mul(gu, Fd, h, blk)
    return linear(ffn.down_proj, h, act_dtype)


def ffn_forward(ffn, x):
    shp = x.shape
    x2 = x.reshape(-1, shp[-1]).contiguous()
    q = ops.quantize(x2, ffn.gate_proj.bit_eps)
    return ffn_q(ffn, q, x.dtype).view(*shp[:-1], ffn.down_proj.out_features)


def block_forward(block, hidden_states, residual=None, inference_params=None, prev_state=None, **mixer_kwargs):
    """``Block.forward`` (block.py:28-45): residual add + RMSNorm fused with the mixer's
    input quantisation, and again before the FFN."""
    B, L, Dm = hidden_states.shape
    act_dtype = hidden_states.dtype
    M = B * L
    x2 = hidden_states.reshape(M, Dm).contiguous()
    res2 = residual.reshape(M, Dm).contiguous().float() if residual is not None else None
    res_out = torch.empty(M, Dm, device=x2.device, dtype=torch.float32)
    mixer = block.mixer
    q = _norm_quant(block.norm, x2, res2, res_out, mixer.in_proj.bit_eps)
    y, final_state = mixer_forward(mixer, q, (B, L), act_dtype, inference_params,
                                   mixer_kwargs.get("cross_layer_state"), prev_state)
    q2 = _norm_quant(block.norm2, y.reshape(M, Dm), res_out, res_out, block.mlp.gate_proj.bit_eps)
    h = ffn_q(block.mlp, q2, act_dtype)
    return h.view(B, L, -1), res_out.view(B, L, Dm), final_state


# ------------------------------------------------------------------ model
def mixer_model_forward(model, input_ids, inference_params=None, prev_states=None, **mixer_kwargs):
    """``MixerModel.forward`` in eval (mixer_seq_simple.py:171-242)."""
    B, L = input_ids.shape
    if L == 0:
        raise ValueError("Input sequence length is 0")
    if L > model.config.max_seq_len:
        raise ValueError(f"Sequence length {L} exceeds max_seq_len {model.config.max_seq_len}")
    caches = inference_params.get("state_cache") if inference_params is not None else None
    pos_offset = 0
    if caches is not None and L == 1:
        c0 = caches.get(0)
        if c0 is not None and "seq_pos" in c0:
            pos_offset = int(c0["seq_pos"])
    emb = model.embedding.weight
    require_b200(model.layers[0].mixer, input_ids, "MixerModel")
    ids = input_ids.contiguous()
    hidden = torch.empty(B * L, emb.shape[1], device=ids.device, dtype=emb.dtype)
    # one-token steps read the position from layer 0's device control word, so a captured
    # decode graph replays with the right offset
    pos_dev = caches[0]["_ctl"] if (caches is not None and L == 1 and caches.get(0) is not None
                                     and "_ctl" in caches[0]) else None
    if pos_dev is not None:
        _prepare_cache(caches[0], ids.device)
    ops.embed(ids, emb, model.position_embedding.weight, pos_dev, pos_offset, hidden)
    hidden = hidden.view(B, L, -1)
    residual = None
    cross = None
    final_states = []
    for i, layer in enumerate(model.layers):
        ps = prev_states[i] if prev_states is not None else None
        lp = None
        if caches is not None and caches.get(i) is not None:
            lp = {"state_cache": caches[i]}
        hidden, residual, fs = block_forward(layer, hidden, residual, inference_params=lp, prev_state=ps,
                                             cross_layer_state=cross, **mixer_kwargs)
        if fs is not None:
            final_states.append(fs)
        cross = getattr(layer.mixer, "_last_cross_layer_state", None)
    M = B * L
    hf = torch.empty(M, hidden.shape[-1], device=hidden.device, dtype=model.norm_f.weight.dtype)
    res_out = torch.empty(M, hidden.shape[-1], device=hidden.device, dtype=torch.float32)
    ops.add_rmsnorm_quant(hidden.reshape(M, -1).contiguous(), residual.reshape(M, -1), res_out,
                          _param_cache(model.norm_f, "weight"), _norm_eps(model.norm_f), 0.0, None, hf)
    return hf.view(B, L, -1), [], None, final_states


def lm_head(lm, hs):
    """The dense tied lm_head (mixer_seq_simple.py:250-252, :334).  bf16 models: the tcgen05
    bf16 GEMM (tesm_b200_gemm_bf16); under tensor parallelism every rank computes its vocabulary
    range and the logits are all-gathered.  fp32 models: torch's F.linear (cuBLAS)."""
    w = lm.lm_head.weight
    shp = hs.shape
    x = hs.reshape(-1, shp[-1]).to(w.dtype)
    if w.dtype != torch.bfloat16 or shp[-1] % 8 or w.stride(0) % 8 or w.stride(1) != 1:
        return F.linear(x, w).view(*shp[:-1], w.shape[0])
    x = x.contiguous()
    V = w.shape[0]
    tp = parallel.get_tp(lm.backbone.layers[0].mlp)
    if tp is not None and V % tp.world == 0:
        v0, v1 = parallel.shard_range(V, tp.world, tp.rank)
        logits = parallel._gather_cols(ops.gemm_bf16(x, w[v0:v1]), tp)
    else:
        logits = ops.gemm_bf16(x, w)
    return logits.view(*shp[:-1], V)


def lm_forward(lm, input_ids, labels=None, inference_params=None, prev_states=None, logits_to_keep=0, **kwargs):
    """``TESMLMHeadModel.forward`` (mixer_seq_simple.py:290-345) without vocabulary suppression."""
    if getattr(lm, "vocab_suppression", False):
        raise TesmError("tesm_b200: vocab_suppression logits are outside the b200 hot path")
    hidden, maps, stats, final_states = mixer_model_forward(lm.backbone, input_ids, inference_params, prev_states)
    sl = slice(-logits_to_keep, None) if isinstance(logits_to_keep, int) and logits_to_keep > 0 else slice(None)
    hs = hidden[:, sl, :]
    logits = lm_head(lm, hs)
    loss = None
    if labels is not None:
        shift_logits = logits[..., :-1, :].contiguous()
        shift_labels = labels[..., 1:].contiguous()
        loss = F.cross_entropy(shift_logits.view(-1, shift_logits.size(-1)).float(), shift_labels.view(-1),
                               ignore_index=lm.tesm_config.label_ignore_index)
    from .models import TESMCausalLMOutput
    return TESMCausalLMOutput(loss=loss, logits=logits, hidden_states=hidden, entanglement_maps=maps,
                              entanglement_stats=stats), final_states


class DecodeGraph:
    """One decode step of a TESMLMHeadModel captured in a CUDA graph.

    The graph replays embedding -> every layer's incremental step -> lm_head for the tokens in
    a static input buffer.  ``greedy=True`` also captures the argmax and writes the chosen tokens
    back into that buffer, so ``step()`` chains steps on the device; ``greedy=False`` leaves the
    next-token choice to the caller (sampling outside the graph): ``step_logits(tokens)`` copies
    the tokens in, replays and returns the last-position logits.  The host mirrors of each
    layer's ``seq_pos`` / ``cache_idx`` are advanced after every replay (the device copies are
    advanced inside the graph by the decode kernels).
    """

    def __init__(self, lm, inference_params, first_tokens, greedy=True):
        self.lm = lm
        self.ip = inference_params
        self.caches = inference_params["state_cache"]
        self.ids = first_tokens.clone()
        self.greedy = greedy
        for c in self.caches.values():
            _prepare_cache(c, self.ids.device)
        # warm-up outside capture (allocates the split-K workspace, packs nothing new)
        snap = [(c["state"].clone(), c["ent_k_cache"].clone(), c["ent_v_cache"].clone(), c["_ctl"].clone(),
                 c["seq_pos"], c["cache_idx"], c["_ctl_host"],
                 {k: v.clone() for k, v in c["_tp"].items()} if "_tp" in c else None)
                for c in self.caches.values()]
        self.lm(self.ids, inference_params=self.ip)
        for c, s in zip(self.caches.values(), snap):
            c["state"].copy_(s[0]); c["ent_k_cache"].copy_(s[1]); c["ent_v_cache"].copy_(s[2]); c["_ctl"].copy_(s[3])
            c["seq_pos"], c["cache_idx"], c["_ctl_host"] = s[4], s[5], s[6]
            if s[7] is not None:  # channel-parallel mixers keep their shard of the cache apart
                for k, v in s[7].items():
                    c["_tp"][k].copy_(v)
        torch.cuda.synchronize()
        hosts = [(c["seq_pos"], c["cache_idx"], c["_ctl_host"]) for c in self.caches.values()]
        self.graph = torch.cuda.CUDAGraph()
        for c in self.caches.values():  # the replayed steps return no per-layer state snapshots
            c["_b200_no_state_out"] = True
        try:
            with torch.cuda.graph(self.graph):
                out, _ = self.lm(self.ids, inference_params=self.ip)
                self.logits = out.logits
                if greedy:
                    self.ids.copy_(out.logits[:, -1, :].argmax(dim=-1, keepdim=True))
        finally:
            for c in self.caches.values():
                c.pop("_b200_no_state_out", None)
        for c, h in zip(self.caches.values(), hosts):  # capture ran no kernel; restore the mirrors
            c["seq_pos"], c["cache_idx"], c["_ctl_host"] = h

    def _replay(self):
        for c in self.caches.values():  # paged snapshots are host-driven, outside the graph
            snapshot_if_due(c)
        self.graph.replay()
        for c in self.caches.values():
            _advance_host(c, c["ent_k_cache"].shape[1])

    def step(self):
        """Greedy graphs: one step on the tokens in the buffer; returns the next tokens."""
        self._replay()
        return self.ids

    def step_logits(self, tokens):
        """One step on ``tokens`` (B, 1); returns the (B, vocab) logits of that position."""
        self.ids.copy_(tokens)
        self._replay()
        return self.logits[:, -1, :]


def _sample(logits, temperature, top_k):
    """Next-token choice of ``TESMLMHeadModel.generate`` (mixer_seq_simple.py:659-668)."""
    if temperature <= 0:
        return logits.argmax(dim=-1, keepdim=True)
    if temperature != 1.0:
        logits = logits / temperature
    if top_k > 0:
        v, _ = torch.topk(logits, min(top_k, logits.size(-1)))
        logits = logits.masked_fill(logits < v[:, [-1]], float("-inf"))
    return torch.multinomial(torch.softmax(logits.float(), dim=-1), num_samples=1)


GRAPH_MIN_TOKENS = 8  # fewer new tokens than this: eager steps (capturing a graph costs more)


@torch.no_grad()
def generate(lm, input_ids, max_new_tokens=64, temperature=1.0, top_k=0, use_cache=True, use_graph=None):
    """``TESMLMHeadModel.generate`` (mixer_seq_simple.py:617-703) without vocabulary
    suppression: prefill with the cache, then one incremental step per new token.  The steps
    replay a captured decode graph (``DecodeGraph(greedy=False)``); sampling (temperature, top-k,
    multinomial) and the EOS test run between replays, as the reference runs them between its
    forward calls.  ``use_graph=False`` runs every step eagerly (same results)."""
    lm.eval()
    generated = input_ids
    cfg = lm.tesm_config
    ip = {"state_cache": lm.backbone.allocate_inference_cache(input_ids.shape[0], cfg.max_seq_len)} if use_cache \
        else None
    out, _ = lm(input_ids, inference_params=ip)
    logits = out.logits[:, -1, :]
    eos = getattr(cfg, "eos_token_id", None)
    if use_graph is None:
        use_graph = use_cache and max_new_tokens >= GRAPH_MIN_TOKENS
    graph = None
    for i in range(max_new_tokens):
        nxt = _sample(logits, temperature, top_k)
        generated = torch.cat([generated, nxt], dim=1)
        if eos is not None and (nxt == eos).all():
            break
        if i == max_new_tokens - 1:
            break  # the reference computes one more step whose logits it never uses
        if use_cache and use_graph:
            if graph is None:
                graph = DecodeGraph(lm, ip, nxt, greedy=False)
            logits = graph.step_logits(nxt)
        elif use_cache:
            for c in ip["state_cache"].values():  # generate discards the per-layer states
                c["_b200_no_state_out"] = True
            out, _ = lm(nxt, inference_params=ip)
            logits = out.logits[:, -1, :]
        else:
            out, _ = lm(generated[:, -cfg.max_seq_len:])
            logits = out.logits[:, -1, :]
    return generated
