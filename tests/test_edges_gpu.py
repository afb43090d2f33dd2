"""Edge cases against the oracle (GPU): empty batches, single-token sequences, all-zero weights
and activations, extreme magnitudes, one-sequence decode.  Same bars as the other parity tests:
bit-exact integer work, max-rel 1e-3 on fp32 layer outputs."""
import numpy as np
import pytest
import torch

import oracle as O
from helpers import build_siso, max_rel, params_np, randn, siso_cfg

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(lib):
    from tesm_b200 import ops as _ops
    return _ops


def test_empty_batch_bitlinear(lib):
    from tesm_b200.modules import BitLinear
    torch.manual_seed(0)
    lin = BitLinear(64, 48).cuda().eval()
    with torch.no_grad():
        for shape in [(0, 64), (2, 0, 64)]:
            y = lin(torch.zeros(*shape, device="cuda"))
            assert y.shape == shape[:-1] + (48,)


def test_zero_weight_and_zero_rows(ops):
    """mean|W| = 0 clamps to bit_eps (every code 0); an all-zero activation row clamps max|x| to
    eps (codes 0, inverse scale eps / 127)."""
    w = torch.zeros(40, 96)
    t_ref, s_ref, _ = O.ternary_weight(w.numpy(), 1e-5)
    pw = ops.pack_weight(w.cuda(), 1e-5, with_tern=True)
    assert np.array_equal(pw.tern.cpu().numpy()[:, :96], t_ref)
    pk = pw.packed.cpu().numpy()
    assert np.array_equal(pk[:, :24], O.pack_int2(t_ref)) and (pk[:, 24:] == 0x55).all()  # pad code 1
    x = torch.zeros(3, 96)
    x[1] = randn((96,), 3)
    c_ref, s = O.quant_act(x.numpy(), 1e-5)
    codes, inv, _ = ops.quant_act(x.cuda(), 1e-5, ops.LAYOUT_ROWMAJOR)
    assert np.array_equal(codes.cpu().numpy()[:, :96], c_ref)
    np.testing.assert_allclose(inv.cpu().numpy(), 1.0 / s, rtol=1e-6)
    y = ops.bitlinear_2d(x.cuda(), pw, 1e-5, torch.float32, force="gemm")
    assert not y.cpu().numpy().any()


@pytest.mark.parametrize("scale", [1e-30, 1e30])
def test_extreme_activation_magnitudes(ops, scale):
    x = randn((5, 256), 9) * scale
    c_ref, _ = O.quant_act(x.numpy(), 1e-5)
    codes, _, _ = ops.quant_act(x.cuda(), 1e-5, ops.LAYOUT_ROWMAJOR)
    assert np.array_equal(codes.cpu().numpy()[:, :256], c_ref)


def test_single_token_prefill_then_decode(lib):
    """A one-token first call with a cache takes the reference's incremental path
    (TESM_SISO.forward routes seqlen == 1 to _forward_incremental, tesm.py:1175-1190): the
    token lands in ring slot 0 and cache_idx becomes 1.  Then three more decode steps, one
    sequence, against the oracle."""
    kw = dict(d_model=64, d_state=32, ent_rank=16, entanglement_window=8, max_seq_len=32)
    m = build_siso(kw).cuda().eval()
    P = params_np(build_siso(kw))
    cfg = siso_cfg(m)
    ip = {"state_cache": m.allocate_inference_cache(1, 32)}
    cache_ref = O.alloc_cache(cfg, 1)
    with torch.no_grad():
        for s in range(4):
            xt = randn((1, 1, 64), 40 + s)
            yr, sr = O.siso_decode(P, cfg, xt.numpy(), cache_ref)[:2]
            yt, st = m(xt.cuda(), inference_params=ip)
            assert max_rel(yt.cpu().numpy(), yr) <= 1e-3, s
            assert max_rel(st.cpu().numpy(), sr) <= 1e-5, s
    assert ip["state_cache"]["cache_idx"] == 4 and ip["state_cache"]["seq_pos"] == 4
