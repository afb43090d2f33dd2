"""Loading the reference's INT2 export (golden fixture written by export_model_to_int2) on the GPU:
unpacked ternary operand, model parity and the export round trip."""
import numpy as np
import pytest
import torch

from helpers import build_model, golden, max_rel, randn
import cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(lib):
    from tesm_b200 import ops
    return ops


def _fixture_dict(g):
    return {str(n): {"packed_weight": torch.from_numpy(g[str(n) + "/packed"]),
                     "weight_scale": torch.tensor(float(g[str(n) + "/scale"])), "bias": None,
                     "in_features": int(g[str(n) + "/shape"][1]), "out_features": int(g[str(n) + "/shape"][0])}
            for n in g["names"]}


@pytest.mark.parametrize("NK", [(300, 4096), (17, 37), (64, 256)])
def test_unpack_matches_pack(ops, NK):
    N, K = NK
    w = (randn((N, K), 61) * 0.02).cuda()
    pw = ops.pack_weight(w, 1e-5, with_tern=True)
    imp = ops.packed_from_int2(pw.packed[:, :(K + 3) // 4].cpu(), pw.scale.cpu(), K, "cuda")
    assert torch.equal(imp.packed, pw.packed)
    assert torch.equal(imp.tern, pw.tern)


def test_export_loads_into_the_model(lib):
    from tesm_b200 import int2
    g = golden("int2_export_tiny")
    c = cases.MODEL[0]
    ref = golden("model_tiny")
    m = build_model(c["cfg"]).cuda()
    ids = torch.from_numpy(ref["ids"]).cuda()
    with torch.no_grad():
        base = m(ids)[0].logits.float().cpu().numpy()
    # our packing of the latent weights equals the reference's export, byte for byte
    ours = int2.export_model_to_int2(m)
    for name, d in _fixture_dict(g).items():
        assert torch.equal(ours[name]["packed_weight"], d["packed_weight"]), name
    assert int2.load_int2_weights_to_model(m, _fixture_dict(g)) == len(g["names"])
    with torch.no_grad():
        imp = m(ids)[0].logits.float().cpu().numpy()
    assert max_rel(imp, base) <= 1e-5
    assert max_rel(imp, ref["logits"]) <= 1e-3
    int2.clear_int2_weights(m)
    with torch.no_grad():
        again = m(ids)[0].logits.float().cpu().numpy()
    assert np.array_equal(again, base)
