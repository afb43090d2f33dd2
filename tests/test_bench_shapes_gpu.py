"""Parity at the shapes the benchmark runs (4 and 5), GPU vs the oracle.

The kernel-level tests elsewhere use short sequences; these run the same kernels at the
sequence lengths and widths that ``bench.py`` times:

* config 3: SISO scan at L = 8192, D = 256 (bf16 projections, decay ~ 0.95 so the fp32
  look-back chains over the whole sequence), local entanglement at L = 8192, and the
  tcgen05 global-entanglement kernel at L = 8192 (R = 64, D = 256);
* config 4: the MIMO scan + window kernels at L = 16384 (H16, D64, R48, RM4), and a
  ``TESMMIMO_Optimized`` layer forward at L = 2048 (fp32 at 1e-3, bf16 at 2e-2);
* config 5 width: a 2-layer ``TESMLMHeadModel`` (d_model 4096, d_state 256, d_intermediate
  11008, vocab 32000, bf16) prefill of 1 x 256 tokens, and a batch-256 decode of a few steps
  through the captured decode graph, logits at the bf16 bar of 2e-2.

Reference paths: tesm.py:1091-1164 (scan), :922-952 (local), :963-1043 (global),
tesm_mimo.py:914-1062 (MIMO layer), mixer_seq_simple.py:171-345 (model).  Flip-aware
comparison as in the kernel tests: ternary decisions whose oracle score is within a small
margin of the threshold may legitimately differ, and rows touched by one are excluded or
checked against both branches.
"""
import math

import numpy as np
import pytest
import torch

import oracle as O
from helpers import max_rel, mimo_cfg, model_cfg, params_np, randn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(lib):
    from tesm_b200 import ops as _ops
    return _ops


def _split(P, Dm, C, Rc):
    o = np.cumsum([0, Dm, C, C, C, Dm, Rc, Rc])
    return [P[:, o[i]:o[i + 1]] for i in range(7)]


def _bf16_proj(M, N, seed):
    P = randn((M, N), seed).to(torch.bfloat16)
    return P, P.float().numpy()


def _ambiguous(scores, thr, tol):
    s = np.abs(np.nan_to_num(scores, nan=1e9))
    return np.abs(s - thr) < tol * np.maximum(1.0, s)


# ------------------------------------------------------------------ config 3 kernels
@pytest.mark.parametrize("decay_bias", [0.0, 3.0])
def test_siso_scan_cfg3_length(ops, decay_bias):
    """B = 1 sequence of config 3 (L 8192, D 256, d_model 2048) with bf16 projections."""
    B, L, Dm, D, R = 1, 8192, 2048, 256, 64
    Pt, Pn = _bf16_proj(B * L, 2 * Dm + 3 * D + 2 * R, 300)
    db = torch.full((D,), decay_bias) + randn((D,), 301) * 0.3
    _, val, dec, wr, _, _, _ = _split(Pn, Dm, D, R)
    a = O.sigmoid(dec.reshape(B, L, D) + db.numpy())
    u = (O.sigmoid(wr) * np.tanh(val)).reshape(B, L, D)
    ref, fin = O.scan_chunked_f64(a, u)
    st = torch.empty(B * L, D, device="cuda")
    f32 = torch.empty(B, D, device="cuda")
    f64 = torch.empty(B, D, device="cuda", dtype=torch.float64)
    ops.siso_scan(Pt.cuda(), B, L, Dm, D, R, db.cuda(), None, st, f32, f64)
    assert ops.device_status() == 0
    assert max_rel(st.cpu().numpy().reshape(B, L, D), ref) <= 1e-5
    assert max_rel(f64.cpu().numpy(), fin) <= 1e-5


def test_siso_local_ent_cfg3_length(ops):
    """Window kernel (bf16 and int8-codes outputs) over one config-3 sequence."""
    B, L, Dm, D, R, W = 1, 8192, 2048, 256, 64, 16
    Pt, Pn = _bf16_proj(B * L, 2 * Dm + 3 * D + 2 * R, 310)
    st = randn((B, L, D), 311)
    bias = randn((W,), 312) * 0.3
    thr, es = 0.1, 0.2
    q = O.rope(Pn[:, 2 * Dm + 3 * D:2 * Dm + 3 * D + R].reshape(B, L, R))
    k = O.rope(Pn[:, 2 * Dm + 3 * D + R:].reshape(B, L, R))
    avg, sc = O.local_ent(q, k, st.numpy(), bias.numpy(), thr, return_scores=True)
    ent = st.numpy() + np.float32(es) * (avg - st.numpy())
    th = torch.empty(B * L, D, device="cuda")
    ch = torch.empty(B * L, D, device="cuda")
    ops.siso_local_ent(Pt.cuda(), B, L, Dm, D, R, W, None, bias.cuda(), st.cuda(), thr, es, 1e4, th, ch)
    assert ops.device_status() == 0
    amb = _ambiguous(sc.reshape(B * L, -1), thr, 2e-5).any(-1)
    assert amb.mean() < 1e-2
    keep = ~amb
    assert max_rel(th.cpu().numpy()[keep], np.tanh(ent).reshape(B * L, D)[keep]) <= 1e-5
    assert max_rel(ch.cpu().numpy()[keep], (ent - st.numpy()).reshape(B * L, D)[keep]) <= 1e-4
    # int8-codes mode (what the model's prefill runs): codes of tanh(ent) and ent - s with
    # per-row scales, compared through their dequantised values (one code of rounding slack)
    c, inv1, inv2, Dp = ops.siso_local_ent_codes(Pt.cuda(), B, L, Dm, D, R, W, None, bias.cuda(), st.cuda(), thr,
                                                 es, 1e4, torch.float32, 1e-5, 1e-5)
    assert ops.device_status() == 0
    c = c.cpu().numpy().astype(np.float64)
    d1 = c[:, :D] * inv1.cpu().numpy().astype(np.float64)[:, None]
    d2 = c[:, Dp:Dp + D] * inv2.cpu().numpy().astype(np.float64)[:, None]
    t_ref = np.tanh(ent).reshape(B * L, D)
    g_ref = (ent - st.numpy()).reshape(B * L, D)
    step1 = np.abs(t_ref).max(-1, keepdims=True) / 127.0
    step2 = np.abs(g_ref).max(-1, keepdims=True) / 127.0
    assert (np.abs(d1 - t_ref)[keep] <= 0.5 * step1[keep] * 1.001 + 1e-6).all()
    assert (np.abs(d2 - g_ref)[keep] <= 0.5 * step2[keep] * 1.001 + 1e-6).all()


def test_siso_global_ent_tc_cfg3_length(ops):
    """tcgen05 global entanglement over one config-3 sequence (L 8192, R 64, D 256).

    A row holds up to 8192 scores, so rows with one score on the threshold are checked
    against both branches of that decision instead of being dropped; rows with more than one
    are excluded (they must stay rare)."""
    B, L, Dm, D, R = 1, 8192, 2048, 256, 64
    Pt, Pn = _bf16_proj(B * L, 2 * Dm + 3 * D + 2 * R, 320)
    st = randn((B, L, D), 321)
    emb = randn((64,), 322) * 0.02
    thr, es = 0.1, 0.2
    q = O.rope(Pn[:, 2 * Dm + 3 * D:2 * Dm + 3 * D + R].reshape(B, L, R))[0]
    k = O.rope(Pn[:, 2 * Dm + 3 * D + R:].reshape(B, L, R))[0]
    v = st.numpy()[0].astype(np.float64)
    relb = ops.global_relbias(emb.cuda(), 1.0, 0.0, L)
    rb = relb.cpu().numpy()
    assert max_rel(rb, O.global_rel_bias(L, emb.numpy(), 1.0, 0.0)) <= 1e-5
    i = np.arange(L)
    th = torch.empty(B * L, D, device="cuda")
    ch = torch.empty(B * L, D, device="cuda")
    ops.siso_global_ent(Pt.cuda(), B, L, Dm, D, R, None, relb, st.cuda(), thr, es, 1e4, th, ch, force="tc")
    assert ops.device_status() == 0
    th = th.cpu().numpy().astype(np.float64)
    ch = ch.cpu().numpy().astype(np.float64)
    inv = np.float32(1.0 / math.sqrt(R))
    bad_rows, multi = 0, 0
    for r0 in range(0, L, 1024):  # row blocks keep the oracle's L x L intermediates small
        r1 = r0 + 1024
        rows = i[r0:r1]
        sc = (q[r0:r1] @ k.T * inv).astype(np.float32) + rb[(rows[:, None] - i[None, :]) + L - 1]
        causal = rows[:, None] >= i[None, :]
        tern = np.where(sc > thr, 1.0, np.where(sc < -thr, -1.0, 0.0)) * causal
        num = tern @ v
        norm = np.abs(tern).sum(-1)
        amb = _ambiguous(np.where(causal, sc, np.nan), thr, 5e-6)
        namb = amb.sum(-1)
        multi += int((namb > 1).sum())
        for j, rr in enumerate(rows):
            if namb[j] > 1:
                continue
            cands = [(num[j], norm[j])]
            if namb[j] == 1:
                c = int(np.nonzero(amb[j])[0][0])
                alt = 0.0 if tern[j, c] != 0 else np.sign(sc[j, c])
                cands.append((num[j] + (alt - tern[j, c]) * v[c], norm[j] + abs(alt) - abs(tern[j, c])))
            s = v[rr]
            ok = False
            for n_, d_ in cands:
                avg = n_ / max(d_, 1.0)
                ent = s + es * (avg - s)
                if np.abs(th[rr] - np.tanh(ent)).max() <= 1e-3 and np.abs(ch[rr] - (ent - s)).max() <= 1e-2 * max(
                        np.abs(ent - s).max(), 1e-3):
                    ok = True
                    break
            bad_rows += not ok
    assert multi < 0.05 * L, f"{multi} rows with several threshold scores"
    assert bad_rows == 0, f"{bad_rows} rows differ beyond 1e-3"


# ------------------------------------------------------------------ config 4 kernels
def test_mimo_scan_ent_cfg4_length(ops):
    """MIMO scan (4 ranks) + window kernel over one config-4 sequence (L 16384, H16, D64)."""
    B, L, Dm, H, D, R, RM, W = 1, 16384, 2048, 16, 64, 48, 4, 16
    C, Rc = H * D, H * R
    Pt, Pn = _bf16_proj(B * L, 2 * Dm + 3 * C + 2 * Rc, 400)
    db = torch.full((H, D), 3.0) + randn((H, D), 401) * 0.3
    mx = 1.0 / RM + randn((H, RM, D), 402) * 0.05
    mo = 1.0 / RM + randn((H, RM, D), 403) * 0.05
    bias = randn((H, W), 404) * 0.02
    thr, es = 0.5, 0.2
    _, val, dec, wr, _, qp, kp = _split(Pn, Dm, C, Rc)
    a = O.sigmoid(dec.reshape(B, L, H, D) + db.numpy())
    w = O.sigmoid(wr.reshape(B, L, H, D))
    v = np.tanh(val.reshape(B, L, H, D)).astype(np.float32)
    q = O.rope_mimo(qp.reshape(B, L, H, R))
    k = O.rope_mimo(kp.reshape(B, L, H, R))
    states = torch.empty(B * L, RM, C, device="cuda")
    f32 = torch.empty(B, C, device="cuda")
    f64 = torch.empty(B, C, device="cuda", dtype=torch.float64)
    Pd = Pt.cuda()
    ops.mimo_scan(Pd, B, L, Dm, H, D, R, RM, db.cuda(), mx.cuda(), states, f32, f64)
    th = torch.empty(B * L, C, device="cuda")
    ch = torch.empty(B * L, C, device="cuda")
    ops.mimo_local_ent(Pd, B, L, Dm, H, D, R, RM, W, bias.cuda(), mo.cuda(), states, thr, es, 1e4, True, th, ch)
    assert ops.device_status() == 0
    stg = states.cpu().numpy().reshape(B, L, RM, H, D)
    ent_ref = np.zeros((B, L, H, D), np.float32)
    chg_ref = np.zeros((B, L, H, D), np.float32)
    sc_any = None
    for r in range(RM):
        upd = (w * mx.numpy()[None, None, :, r]) * (v * mx.numpy()[None, None, :, r])
        st = O.scan_seq(a, upd.astype(np.float32))
        assert max_rel(stg[:, :, r], st) <= 1e-5, f"rank {r} states"
        avg, sc = O.local_ent_mimo(q, k, st, bias.numpy(), thr, return_scores=True)
        sc_any = sc
        e_r = st + np.float32(es) * (avg - st)
        ent_ref += mo.numpy()[None, None, :, r] * e_r
        chg_ref += mo.numpy()[None, None, :, r] * (e_r - st)
    amb = _ambiguous(sc_any.reshape(B * L, -1), thr, 2e-5).any(-1)
    assert amb.mean() < 1e-2
    keep = ~amb
    assert max_rel(th.cpu().numpy()[keep], np.tanh(ent_ref).reshape(B * L, C)[keep]) <= 1e-5
    assert max_rel(ch.cpu().numpy()[keep], chg_ref.reshape(B * L, C)[keep]) <= 1e-4


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_mimo_layer_cfg4(lib, dtype):
    """TESMMIMO_Optimized at config 4's shape (d_model 2048, 16 heads, d_state 64, window 16,
    seed-0 init) over one sequence of 2048 tokens.  fp32: tokens whose oracle window scores
    sit within 2e-5 of the threshold are excluded (the int8 codes of the fp32 input are
    bit-exact, so those are the only decisions that can flip); bf16 activations: 2e-2 over all
    tokens."""
    from tesm_b200.modules import TESMMIMO_Optimized
    torch.manual_seed(0)
    m = TESMMIMO_Optimized(d_model=2048, n_heads=16, d_state=64, entanglement_window=16, max_seq_len=2048,
                           kernel_backend="b200").eval()
    P = params_np(m)
    B, L = 1, 2048
    x = randn((B, L, 2048), 410)
    y_ref, fin_ref, _, det = O.mimo_forward(P, mimo_cfg(m), x.numpy(), details=True)
    m = m.cuda()
    with torch.no_grad():
        xd = x.cuda() if dtype == "f32" else x.cuda().to(torch.bfloat16)
        y, fs = m(xd)
    y = y.float().cpu().numpy()
    if dtype == "bf16":
        assert max_rel(y, y_ref) <= 2e-2
        return
    _, sc = O.local_ent_mimo(det["q"], det["k"], det["states0"], P["local_entanglement_bias"],
                             m.entanglement_threshold, return_scores=True)
    amb = _ambiguous(sc.reshape(B, L, -1), m.entanglement_threshold, 2e-5).any(-1)
    assert amb.mean() < 2e-2
    assert max_rel(y[~amb], y_ref[~amb]) <= 1e-3
    assert max_rel(fs.cpu().numpy(), fin_ref) <= 1e-5


# ------------------------------------------------------------------ config 5 width
CFG5 = dict(d_model=4096, d_state=256, entanglement_window=16, vocab_size=32000, d_intermediate=11008,
            max_seq_len=4608, ent_rank=64)


def _cfg5_model(n_layer, dtype):
    from tesm_b200.models import TESMConfig, TESMLMHeadModel
    torch.manual_seed(0)
    cfg = TESMConfig(kernel_backend="b200", n_layer=n_layer, **CFG5)
    with torch.device("cuda"):
        m = TESMLMHeadModel(cfg, dtype=dtype).eval()
    return m, params_np(m), model_cfg(cfg)


def _oracle_block(P, ocfg, i, hidden, residual, cross, cache=None, in_codes=None, ffn_codes=None,
                  dtype="float32"):
    """``Block.forward`` of layer i (block.py:28-45 with the FFN of mixer_seq_simple.py:59-67)
    in the oracle, from given (hidden, residual, cross-layer state) and optionally the int8
    codes (and 1/s) handed to in_proj and to the FFN.  Returns the FFN output,
    the residual, the new cross-layer state, the window scores of the entanglement and, per
    token, the distance of the state_proj / ent_proj inputs (tanh(ent), ent - s) to an int8
    rounding tie: with K = d_state = 256 one code flip there moves y by ~1e-3 of its range."""
    pre = f"backbone.layers.{i}."
    lp = {k[len(pre) + 6:]: v for k, v in P.items() if k.startswith(pre + "mixer.")}
    fp = {k[len(pre) + 4:]: v for k, v in P.items() if k.startswith(pre + "mlp.")}
    res = hidden if residual is None else (hidden + residual).astype(np.float32)
    h = O.rmsnorm(res, P[pre + "norm.weight"], ocfg["norm_epsilon"])
    if cache is not None and hidden.shape[1] == 1:
        y, _, new, det = O.siso_decode(lp, ocfg, h, cache, cross, details=True, in_codes=in_codes, dtype=dtype)
        scores = det["scores"][:, None]
        new_cross = new
    else:
        y, _, states, det = O.siso_forward(lp, ocfg, h, cross, None, cache, details=True, in_codes=in_codes,
                                           dtype=dtype)
        scores, new_cross = det["scores"], states
    if dtype == "float32":
        tie = np.minimum(O.quant_tie_margin(np.tanh(det["ent"])), O.quant_tie_margin(det["chg"]))
        if tie.ndim == 1:
            tie = tie[:, None]
    else:  # bf16 semantics round x * s to bf16 first, so exact .5 products are common; both
        tie = np.full(scores.shape[:2], np.inf)  # sides then round them the same way
    res2 = (y + res).astype(np.float32)
    # the FFN can be fed the device's own int8 codes of its input: RMSNorm + requantisation
    # + SwiGLU + requantisation amplify a 6e-4 residual difference (rounding ties upstream) ~25x
    h2 = O.rmsnorm(res2, P[pre + "norm2.weight"], ocfg["norm_epsilon"])
    f, hsw = O.ffn(fp, h2, dtype=dtype, in_codes=ffn_codes, return_h=True)
    return (f, hsw), res2, new_cross, scores, tie


def _b200_layers(m, ids, ip=None):
    """Run the b200 blocks one by one and record each block's inputs, the int8 codes and 1/s
    its fused residual + RMSNorm + quantisation kernel hands to in_proj, and its outputs."""
    from tesm_b200 import layers as LY, ops
    bb = m.backbone
    ids = ids.cuda()
    B, L = ids.shape
    pos0 = 0
    if ip is not None and L == 1:
        pos0 = ip["state_cache"][0]["seq_pos"]
    hidden = (bb.embedding.weight[ids] + bb.position_embedding.weight[pos0:pos0 + L][None]).to(bb.embedding.weight.dtype)
    residual, cross, rec = None, None, []
    for i, layer in enumerate(bb.layers):
        lp = {"state_cache": ip["state_cache"][i]} if ip is not None else None
        inp = (hidden, residual, cross)
        M = B * L
        scratch = torch.empty(M, hidden.shape[-1], device=ids.device)
        q = LY._norm_quant(layer.norm, hidden.reshape(M, -1).contiguous(),
                           None if residual is None else residual.reshape(M, -1).float().contiguous(), scratch,
                           layer.mixer.in_proj.bit_eps)
        assert q.layout == ops.LAYOUT_ROWMAJOR
        codes = (q.codes.cpu().numpy()[:, :hidden.shape[-1]].reshape(B, L, -1), q.inv.cpu().numpy().reshape(B, L))
        hidden, residual, _ = LY.block_forward(layer, hidden, residual, inference_params=lp, cross_layer_state=cross)
        cross = layer.mixer._last_cross_layer_state
        # the FFN's input codes: RMSNorm of the block's residual (0 + residual is exact)
        q2 = LY._norm_quant(layer.norm2, torch.zeros(M, hidden.shape[-1], device=ids.device, dtype=hidden.dtype),
                            residual.reshape(M, -1).float().contiguous(), scratch, layer.mlp.gate_proj.bit_eps)
        codes2 = (q2.codes.cpu().numpy()[:, :hidden.shape[-1]].reshape(B, L, -1), q2.inv.cpu().numpy().reshape(B, L))
        # the FFN's SwiGLU output silu(gate) * up, as ffn_q computes it before down_proj
        pw, blk = LY.ffn_packed(layer.mlp)
        if blk and q2.layout == ops.LAYOUT_ROWMAJOR:
            hsw = ops.gemm_swiglu(q2, pw, hidden.dtype)
        else:
            gu = ops.matmul_q(q2, pw, hidden.dtype)
            hsw = torch.empty(M, layer.mlp.gate_proj.out_features, device=ids.device, dtype=hidden.dtype)
            ops.silu_mul(gu, layer.mlp.gate_proj.out_features, hsw, blk)
        rec.append((inp + (codes, codes2, hsw.float().cpu().numpy().reshape(B, L, -1)), (hidden, residual)))
    return rec


def _np(t):
    return None if t is None else t.float().cpu().numpy()


def _per_layer_check(m, P, ocfg, ids, tol, margin, max_excl, ip=None, ocache=None, dtype="float32"):
    """Teacher-forced comparison: every b200 block against the oracle block fed the b200
    block's own inputs, so ternary decisions that flip in one layer do not cascade into the
    next, and handed the int8 codes the device quantised for in_proj and for the FFN, so that
    a rounding tie upstream cannot move one side's quantisation scale.  Tokens with a window
    score within `margin` of the threshold are excluded."""
    thr = ocfg["entanglement_threshold"]
    with torch.no_grad():
        rec = _b200_layers(m, ids, ip)
    for i, ((h_in, r_in, c_in, codes, codes2, hsw), (h_out, r_out)) in enumerate(rec):
        c_np = _np(c_in)
        if c_np is not None and ids.shape[1] > 1:
            c_np = c_np.reshape(ids.shape[0], ids.shape[1], -1)
        (f_ref, hsw_ref), r_ref, _, sc, tie = _oracle_block(P, ocfg, i, _np(h_in), _np(r_in), c_np,
                                                            None if ocache is None else ocache[i], in_codes=codes,
                                                            ffn_codes=codes2, dtype=dtype)
        # the SwiGLU product, then down_proj from the device's own product (its int8
        # requantisation rescales every code when the row maximum moves by one bf16 ulp)
        assert max_rel(hsw, hsw_ref) <= tol, f"layer {i} silu(gate) * up"
        pre = f"backbone.layers.{i}.mlp."
        f_ref = O.bitlinear(hsw, P[pre + "down_proj.weight"], 1e-5, dtype)
        amb = _ambiguous(sc.reshape(sc.shape[0], sc.shape[1], -1), thr, margin).any(-1) | (tie < 2e-5)
        assert amb.mean() < max_excl, f"layer {i}: {amb.mean():.3f} of tokens at the threshold"
        keep = ~amb
        ho, ro = _np(h_out).reshape(f_ref.shape), _np(r_out).reshape(r_ref.shape)
        assert max_rel(ro[keep], r_ref[keep]) <= tol, f"layer {i} residual"
        assert max_rel(ho[keep], f_ref[keep]) <= tol, f"layer {i} ffn output"
    return rec


def test_model_cfg5_width_prefill_per_layer_f32(lib):
    """Two config-5 layers (d_model 4096, d_state 256, d_intermediate 11008), fp32, 1 x 256
    tokens, each block teacher-forced against the oracle at 1e-3; then the final norm and tied
    lm_head from the last block's output (all 32000 logits of every position).  Excluded:
    tokens with a window score within 2e-4 of the threshold (one int8 code flip in in_proj's
    input, from a rounding tie of the 4096-wide RMSNorm output, moves a score by ~1e-4) and
    tokens whose state_proj / ent_proj input sits at a rounding tie."""
    dtype, tol = torch.float32, 1e-3
    m, P, ocfg = _cfg5_model(2, dtype)
    ids = torch.randint(0, 32000, (1, 256), generator=torch.Generator().manual_seed(500))
    rec = _per_layer_check(m, P, ocfg, ids, tol, 2e-4, 0.05)
    (h_last, r_last) = rec[-1][1]
    res = (_np(h_last) + _np(r_last)).astype(np.float32)
    hf = O.rmsnorm(res, P["backbone.norm_f.weight"], ocfg["norm_epsilon"])
    ref = (hf.astype(np.float64) @ P["lm_head.weight"].astype(np.float64).T)
    from tesm_b200 import ops
    with torch.no_grad():
        M = res.shape[0] * res.shape[1]
        out = torch.empty(M, 4096, device="cuda", dtype=m.backbone.norm_f.weight.dtype)
        ro = torch.empty(M, 4096, device="cuda")
        ops.add_rmsnorm_quant(h_last.reshape(M, -1).contiguous(), r_last.reshape(M, -1).contiguous(), ro,
                              m.backbone.norm_f.weight.float().contiguous(), 1e-5, 0.0, None, out)
        logits = torch.nn.functional.linear(out, m.lm_head.weight)
    assert max_rel(logits.float().cpu().numpy(), ref.reshape(M, -1)) <= tol


def test_model_cfg5_width_prefill_per_layer_bf16(lib):
    """The same two layers with bf16 activations, teacher-forced per block at the bf16 bar of
    2e-2 against the oracle in bf16 mode: every BitLinear with the reference's bf16 semantics
    (weight scale, x * s and codes rounded as torch rounds them in bf16, tesm.py:206-215),
    bf16 projections, fp32 scan and entanglement.  The fp32-semantics oracle is not the
    reference for a bf16 model: the reference's own BitLinear in bf16 differs from its fp32 run
    by ~7% of the output range at K = 4096 (the bf16 weight scale moves ternary thresholds)."""
    m, P, ocfg = _cfg5_model(2, torch.bfloat16)
    ids = torch.randint(0, 32000, (1, 256), generator=torch.Generator().manual_seed(500))
    _per_layer_check(m, P, ocfg, ids, 2e-2, 1e-3, 0.05, dtype="bfloat16")


def test_model_cfg5_width_end_to_end_f32(lib):
    """Whole-model logits (2 config-5 layers, fp32, 1 x 256): ternary decisions make the model
    discontinuous, and a decision that flips in layer 0 reaches later tokens of layer 1 through
    its scan.  The b200 logits must stay as close to the oracle as the oracle stays to itself
    under a one-ulp perturbation of the embedding table (median and 95th percentile of the
    per-token error), and match it to 1e-3 at half of the positions or more."""
    m, P, ocfg = _cfg5_model(2, torch.float32)
    ids = torch.randint(0, 32000, (1, 256), generator=torch.Generator().manual_seed(500))
    O.memo_weights(True)
    try:
        ref = O.model_forward(P, ocfg, ids.numpy())
        P2 = dict(P)
        P2["backbone.embedding.weight"] = np.nextafter(P["backbone.embedding.weight"], np.float32(np.inf))
        ref2 = O.model_forward(P2, ocfg, ids.numpy())
    finally:
        O.memo_weights(False)
    with torch.no_grad():
        out, _ = m(ids.cuda())
    lg = out.logits.cpu().numpy()
    den = np.abs(ref).max()
    e_k = np.abs(lg - ref).max(-1)[0] / den
    e_o = np.abs(ref2 - ref).max(-1)[0] / den
    assert np.median(e_k) <= max(3 * np.median(e_o), 1e-3)
    assert np.quantile(e_k, 0.95) <= max(3 * np.quantile(e_o, 0.95), 1e-3)
    assert (e_k <= 1e-3).mean() >= 0.5 * (e_o <= 1e-3).mean()


def test_model_cfg5_width_decode_b256_f32(lib):
    """One config-5 layer (d_model 4096, d_intermediate 11008), fp32, batch 256: a 16-token
    prompt, then 3 one-token decode steps, each block teacher-forced against the oracle's
    incremental decode (tesm.py:1274-1400) from the device's cache at 1e-3, excluding
    sequences with a window score within 2e-4 of the threshold or a state_proj / ent_proj
    input at a rounding tie.  With one layer the cache (scan state, window keys and states) does
    not depend on any ternary decision; it is compared after the prompt."""
    m, P, ocfg = _cfg5_model(1, torch.float32)
    Bd = 256
    prompt = torch.randint(0, 32000, (Bd, 16), generator=torch.Generator().manual_seed(501))
    ocache = O.model_alloc_cache(ocfg, Bd)
    O.memo_weights(True)
    try:
        with torch.no_grad():
            ip = {"state_cache": m.backbone.allocate_inference_cache(Bd, 4608)}
            o, _ = m(prompt.cuda(), inference_params=ip, logits_to_keep=1)
        O.model_forward(P, ocfg, prompt.numpy(), ocache, logits_to_keep=1)
        # the prompt's int8 codes can differ at rounding ties of the 4096-wide RMSNorm output
        # (summation order), which moves the cached states by ~1e-4
        c = ip["state_cache"][0]
        assert max_rel(c["state"].cpu().numpy(), ocache[0]["state"]) <= 1e-3
        assert max_rel(c["ent_k_cache"].cpu().numpy(), ocache[0]["ent_k_cache"]) <= 1e-3
        assert max_rel(c["ent_v_cache"].cpu().numpy(), ocache[0]["ent_v_cache"]) <= 1e-3
        tok = o.logits[:, -1:].argmax(-1).cpu()
        for s in range(3):
            # the oracle step starts from the device's cache (teacher forcing across steps)
            c = ip["state_cache"][0]
            oc = {0: {"state": c["state"].cpu().numpy(), "ent_k_cache": c["ent_k_cache"].cpu().numpy(),
                      "ent_v_cache": c["ent_v_cache"].cpu().numpy(), "seq_pos": int(c["seq_pos"]),
                      "cache_idx": int(c["cache_idx"])}}
            _per_layer_check(m, P, ocfg, tok, 1e-3, 2e-4, 0.05, ip=ip, ocache=oc)
            ref = O.model_forward(P, ocfg, tok.numpy(), ocache)
            tok = torch.from_numpy(ref[:, -1].argmax(-1)[:, None].astype(np.int64))
    finally:
        O.memo_weights(False)
    assert ip["state_cache"][0]["seq_pos"] == 19


def test_decode_graph_matches_eager_cfg5_width(lib):
    """The captured decode step (DecodeGraph) at config-5 width and batch 256 replays exactly
    what the eager one-token forward computes: same logits (1e-5) and tokens over 4 steps."""
    from tesm_b200.layers import DecodeGraph
    m, _, _ = _cfg5_model(2, torch.bfloat16)
    Bd = 256
    prompt = torch.randint(0, 32000, (Bd, 16), generator=torch.Generator().manual_seed(502)).cuda()
    runs = []
    with torch.no_grad():
        for use_graph in (False, True):
            ip = {"state_cache": m.backbone.allocate_inference_cache(Bd, 4608)}
            o, _ = m(prompt, inference_params=ip, logits_to_keep=1)
            tok = o.logits[:, -1:].argmax(-1)
            lg, tk = [], []
            g = DecodeGraph(m, ip, tok) if use_graph else None
            for _ in range(4):
                if use_graph:
                    tok = g.step().clone()
                    lg.append(g.logits[:, -1].float().cpu().numpy())
                else:
                    o, _ = m(tok, inference_params=ip)
                    lg.append(o.logits[:, -1].float().cpu().numpy())
                    tok = o.logits[:, -1:].argmax(-1)
                tk.append(tok.cpu().numpy())
            runs.append((lg, tk))
    for a, b in zip(runs[0][0], runs[1][0]):
        assert max_rel(b, a) <= 1e-5
    for a, b in zip(runs[0][1], runs[1][1]):
        assert np.array_equal(a, b)
