"""BitLinear kernels vs the oracle and the reference's golden vectors (GPU).

Bar: bit-exact ternary codes / packed bytes / int8 activation codes / int32
accumulators; outputs within max-rel 1e-5 (fp32) and 2e-2 (bf16).
"""
import numpy as np
import pytest
import torch

import cases
import oracle as O
from helpers import golden, max_rel, randn

pytestmark = pytest.mark.gpu

DT = {"float32": torch.float32, "bfloat16": torch.bfloat16}


def gemv_positions(Kp):
    """Stored byte offset of natural column k in the GEMV code layout."""
    k = np.arange(Kp)
    s, r = k // 256, k % 256
    tig, u, e = r // 64, (r // 16) % 4, r % 16
    i, sw = e // 4, e % 4
    return s * 256 + u * 64 + tig * 16 + sw * 4 + i


@pytest.fixture(scope="module")
def ops(lib):
    from tesm_b200 import ops as _ops
    return _ops


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("NK", [(80, 96), (19, 37), (256, 1000), (11008, 4096)])
def test_pack_bit_exact(ops, dtype, NK):
    N, K = NK
    w = (randn((N, K), 5) * 0.02).to(DT[dtype])
    t_ref, scale_ref, deq_ref = O.ternary_weight(w.float().numpy(), 1e-5, dtype)
    pw = ops.pack_weight(w.cuda(), 1e-5, with_tern=True)
    torch.cuda.synchronize()
    assert float(pw.scale.cpu()[0]) == float(scale_ref), "absmean scale differs"
    assert float(pw.deq.cpu()[0]) == float(deq_ref)
    packed = pw.packed.cpu().numpy()
    assert np.array_equal(packed[:, :(K + 3) // 4], O.pack_int2(t_ref)), "packed bytes differ"
    assert np.all(packed[:, (K + 3) // 4:] == 0x55), "padding must be code 1 (t=0)"
    tern = pw.tern.cpu().numpy()
    assert np.array_equal(tern[:, :K], t_ref) and not tern[:, K:].any()


@pytest.mark.parametrize("c", cases.BITLINEAR, ids=lambda c: c["name"])
def test_golden_codes(ops, c):
    g = golden("bitlinear_" + c["name"])
    dt = DT[c["dtype"]]
    w = (randn((c["N"], c["K"]), 3) * c["wstd"]).to(dt).cuda()
    x = randn(c["xshape"], 1, dt).cuda().reshape(-1, c["K"])
    pw = ops.pack_weight(w, 1e-5, with_tern=True)
    assert np.array_equal(pw.tern.cpu().numpy()[:, :c["K"]], g["t"])
    codes, inv, _ = ops.quant_act(x, 1e-5, ops.LAYOUT_ROWMAJOR)
    assert np.array_equal(codes.cpu().numpy()[:, :c["K"]], g["codes"].reshape(-1, c["K"]))
    for path in ("gemv", "gemm"):
        y, acc = ops.bitlinear_2d(x, pw, 1e-5, dt, acc=True, force=path)
        assert np.array_equal(acc.cpu().numpy(), g["acc"]), path
        tol = 2e-2 if c["dtype"] == "bfloat16" else 1e-5
        assert max_rel(y.float().cpu().numpy(), g["y"].reshape(y.shape)) <= tol, path


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("MK", [(1, 4096), (7, 37), (33, 11008), (300, 96), (2048, 256), (1500, 1000)])
def test_quant_codes_bit_exact(ops, dtype, MK):
    M, K = MK
    x = (randn((M, K), 7) * 3).to(DT[dtype])
    x[0, :5] = 0  # exact zeros and a near-tie row
    if M > 1:
        x[1] = torch.linspace(-1, 1, K).to(DT[dtype])
    c_ref, s_ref = O.quant_act(x.float().numpy(), 1e-5, dtype)
    xc = x.cuda()
    codes, inv, _ = ops.quant_act(xc, 1e-5, ops.LAYOUT_ROWMAJOR)
    assert np.array_equal(codes.cpu().numpy()[:, :K], c_ref)
    np.testing.assert_allclose(inv.cpu().numpy(), 1.0 / s_ref, rtol=1e-6)
    gc, ginv, rs = ops.quant_act(xc, 1e-5, ops.LAYOUT_GEMV)
    Kp = (K + 255) // 256 * 256
    pos = gemv_positions(Kp)
    g = gc.cpu().numpy()
    nat = g[:, pos]
    assert np.array_equal(nat[:, :K], c_ref) and not nat[:, K:].any()
    assert np.array_equal(rs.cpu().numpy(), c_ref.astype(np.int64).sum(1))


SHAPES = [(1, 11008, 4096), (16, 11008, 4096), (16, 4096, 11008), (3, 80, 96), (8, 19, 37), (9, 300, 300),
          (33, 1000, 520), (64, 130, 4096)]


@pytest.mark.parametrize("MNK", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_gemv_exact(ops, MNK):
    M, N, K = MNK
    w = randn((N, K), 11) * 0.02
    x = randn((M, K), 12)
    t, _, deq = O.ternary_weight(w.numpy(), 1e-5)
    c, s = O.quant_act(x.numpy(), 1e-5)
    acc_ref = O.int_gemm(c, t)
    pw = ops.pack_weight(w.cuda(), 1e-5, with_tern=False)
    y, acc = ops.bitlinear_2d(x.cuda(), pw, 1e-5, torch.float32, acc=True, force="gemv")
    assert np.array_equal(acc.cpu().numpy(), acc_ref)
    y_ref = O.bitlinear(x.numpy(), w.numpy(), 1e-5)
    assert max_rel(y.cpu().numpy(), y_ref) <= 1e-5


GEMM_SHAPES = [(65, 80, 96), (128, 256, 256), (300, 1000, 520), (1000, 11008, 4096), (256, 4096, 11008),
               (77, 130, 37), (4096, 512, 2048), (128, 4096, 4096), (200, 300, 2048), (300, 1000, 2048),
               (4500, 8000, 1000)]
# M <= 256 runs the skinny-tile kernel; (300, 1000, 2048) has fewer tiles than SMs -> split-K;
# (4500, 8000, 1000) has enough 256 x 256 tiles for CTA pairs (ragged M, N and K)


@pytest.mark.parametrize("MNK", GEMM_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("out", ["float32", "bfloat16"])
def test_gemm_exact(ops, MNK, out):
    M, N, K = MNK
    w = randn((N, K), 21) * 0.02
    x = randn((M, K), 22)
    t, _, deq = O.ternary_weight(w.numpy(), 1e-5)
    c, s = O.quant_act(x.numpy(), 1e-5)
    acc_ref = O.int_gemm(c, t)
    pw = ops.pack_weight(w.cuda(), 1e-5, with_tern=True)
    y, acc = ops.bitlinear_2d(x.cuda(), pw, 1e-5, DT[out], acc=True, force="gemm")
    a = acc.cpu().numpy()
    bad = np.argwhere(a != acc_ref)
    assert bad.size == 0, f"{len(bad)} mismatching accumulators, first at {bad[:4].tolist()}"
    y_ref = O.bitlinear(x.numpy(), w.numpy(), 1e-5)
    assert max_rel(y.float().cpu().numpy(), y_ref) <= (1e-5 if out == "float32" else 8e-3)


def test_per_row_scale(ops):
    N, K, M = 300, 512, 20
    w = randn((N, K), 31) * torch.linspace(0.01, 0.1, N)[:, None]
    x = randn((M, K), 32)
    y_ref = O.bitlinear(x.numpy(), w.numpy(), 1e-5, per_row=True)
    pw = ops.pack_weight(w.cuda(), 1e-5, per_row=True, with_tern=True)
    for path in ("gemv", "gemm"):
        y = ops.bitlinear_2d(x.cuda(), pw, 1e-5, torch.float32, force=path)
        assert max_rel(y.cpu().numpy(), y_ref) <= 1e-5, path


def test_module_forward(lib):
    from tesm_b200.modules import BitLinear
    c = cases.BITLINEAR[0]
    g = golden("bitlinear_" + c["name"])
    torch.manual_seed(0)
    lay = BitLinear(c["K"], c["N"]).cuda().eval()
    with torch.no_grad():
        lay.weight.copy_((randn((c["N"], c["K"]), 3) * c["wstd"]).cuda())
        y = lay(randn(c["xshape"], 1).cuda())
    assert y.shape == tuple(c["xshape"][:-1]) + (c["N"],)
    assert max_rel(y.cpu().numpy(), g["y"]) <= 1e-5
    lay.train()
    with pytest.raises(RuntimeError, match="kernel_backend='b200' specified but BitLinear kernel not available"):
        lay(randn(c["xshape"], 1).cuda())


@pytest.mark.parametrize("M,Dm", [(20, 256), (300, 256), (200, 2048), (300, 2048), (13000, 256)])
def test_ffn_swiglu_interleaved(lib, M, Dm):
    """FeedForward with d_intermediate % 128 == 0: gate/up rows interleaved in 128-blocks; the
    tensor-core path applies silu(gate)*up in the GEMM epilogue, the GEMV path in a kernel."""
    from tesm_b200.models import FeedForward, TESMConfig
    cfg = TESMConfig(d_model=Dm, d_intermediate=384, kernel_backend="b200")
    torch.manual_seed(0)
    ffn = FeedForward(cfg)
    for lin in (ffn.gate_proj, ffn.up_proj, ffn.down_proj):
        torch.nn.init.normal_(lin.weight, std=0.02)
    P = {k: v.detach().numpy() for k, v in ffn.state_dict().items()}
    x = randn((M, Dm), 41)
    ref = O.ffn(P, x.numpy())
    g, u = ffn.gate_proj.weight.detach().numpy(), ffn.up_proj.weight.detach().numpy()
    c, s = O.quant_act(x.numpy())
    tg, _, dg = O.ternary_weight(g)
    tu, _, du = O.ternary_weight(u)
    inv = (1.0 / s.astype(np.float64))[:, None]
    gx = O.int_gemm(c, tg) * inv * dg
    ux = O.int_gemm(c, tu) * inv * du
    h = (gx / (1 + np.exp(-gx)) * ux).astype(np.float32)
    tie = O.quant_tie_margin(h) < 1e-4  # h goes through expf on the device: wider tie band
    ffn = ffn.cuda().eval()
    with torch.no_grad():
        y = ffn(x.cuda()).cpu().numpy()
    assert tie.mean() < 0.2
    assert max_rel(y[~tie], ref[~tie]) <= 1e-4


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("MNK", [(4133, 4096, 256), (200, 200, 128), (50, 96, 256), (1000, 1000, 384)])
def test_gemm_combine_epilogue(ops, dtype, MNK):
    """Dual-accumulator GEMM with the combine epilogue (tesm.py:1256-1260):
    out = local + sigmoid(gate) * acc1 * inv1 * deq1 + acc2 * inv2 * deq2, against the exact
    int accumulators in fp64.  bf16 runs the TMA-staged epilogue (ragged M and N, row quarters
    of the last tile past M), fp32 the register path."""
    M, N, Kh = MNK
    g = torch.Generator().manual_seed(M + N)
    codes = torch.randint(-128, 128, (M, 2 * Kh), generator=g, dtype=torch.int8)
    tern = torch.randint(-1, 2, (N, 2 * Kh), generator=g, dtype=torch.int8)
    inv1 = torch.rand(M, generator=g) * 1e-2
    inv2 = torch.rand(M, generator=g) * 1e-2
    deq1, deq2 = torch.tensor([0.03]), torch.tensor([0.05])
    c_local, c_gate = 8, 16 + N  # columns inside a wider proj row, 16-byte aligned offsets
    ldp = c_gate + N + 24
    proj = (torch.randn(M, ldp, generator=g) * 2).to(DT[dtype])
    out = torch.full((M, N), float("nan"), dtype=DT[dtype], device="cuda")
    ops.gemm_combine(codes.cuda(), Kh, inv1.cuda(), inv2.cuda(), tern.cuda(), deq1.cuda(), deq2.cuda(), proj.cuda(),
                     c_local, c_gate, M, N, out)
    c64, t64 = codes.double(), tern.double()
    a1 = c64[:, :Kh] @ t64[:, :Kh].T
    a2 = c64[:, Kh:] @ t64[:, Kh:].T
    pf = proj.double()
    loc, gate = pf[:, c_local:c_local + N], pf[:, c_gate:c_gate + N]
    ref = loc + torch.sigmoid(gate) * a1 * (inv1.double()[:, None] * 0.03) + a2 * (inv2.double()[:, None] * 0.05)
    got = out.cpu().double()
    assert torch.isfinite(got).all()
    tol = 1e-5 if dtype == "float32" else 8e-3
    err = ((got - ref).abs() / (ref.abs() + 1.0)).max().item()
    assert err <= tol, err
    # the same epilogue on accumulators summed elsewhere (tensor-parallel MIMO tail): bit for bit
    out2 = torch.empty_like(out)
    ops.combine_acc(a1.to(torch.int32).cuda(), a2.to(torch.int32).cuda(), inv1.cuda(), inv2.cuda(), deq1.cuda(),
                    deq2.cuda(), proj.cuda(), c_local, c_gate, out2)
    assert torch.equal(out2, out)


@pytest.mark.parametrize("MNK", [(1, 32000, 4096), (32, 32000, 4096), (256, 32000, 4096), (300, 1000, 520),
                                 (77, 130, 72)], ids=lambda s: "x".join(map(str, s)))
def test_gemm_bf16_lm_head(ops, MNK):
    """The tied lm_head GEMM (mixer_seq_simple.py:334) on tcgen05 kind::f16: bf16 operands, fp32
    accumulation, against an fp64 product of the same bf16 values (fp32 output at 1e-5 of the
    range; bf16 output within its rounding)."""
    M, N, K = MNK
    a = (randn((M, K), 91)).to(torch.bfloat16)
    b = (randn((N, K), 92) * 0.02).to(torch.bfloat16)
    ref = a.double() @ b.double().T
    y32 = ops.gemm_bf16(a.cuda(), b.cuda(), torch.float32)
    y16 = ops.gemm_bf16(a.cuda(), b.cuda(), torch.bfloat16)
    assert max_rel(y32.cpu().numpy(), ref.numpy()) <= 1e-5
    assert max_rel(y16.float().cpu().numpy(), ref.numpy()) <= 8e-3
