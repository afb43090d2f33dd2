"""The reference's on-disk INT2 export (golden fixture from export_model_to_int2) against the
oracle, and the loader's argument checks (CPU)."""
import numpy as np
import pytest
import torch

import oracle as O
from helpers import build_model, golden, sd_hash
import cases


def test_export_fixture_matches_oracle_packing():
    g = golden("int2_export_tiny")
    m = build_model(cases.MODEL[0]["cfg"], backend="b200")
    assert sd_hash(m) == str(g["sd_sha256"]), "mirror init does not reproduce the exported model"
    lins = dict(m.named_modules())
    for name in g["names"]:
        name = str(name)
        w = lins[name].weight.detach().numpy()
        t, scale, _ = O.ternary_weight(w, 1e-5)
        assert np.array_equal(g[name + "/packed"], O.pack_int2(t)), name
        assert tuple(g[name + "/shape"]) == w.shape
        # the export's 1/mean|W| comes from torch's fp32 mean; within one rounding of BitLinear's
        np.testing.assert_allclose(np.float32(g[name + "/scale"]), np.float32(scale), rtol=2.5e-7, atol=0)


def test_loader_rejects_mismatches():
    from tesm_b200 import int2
    m = build_model(cases.MODEL[0]["cfg"], backend="b200")
    good = {"packed_weight": torch.zeros(16, 8, dtype=torch.uint8), "weight_scale": torch.tensor(1.0),
            "bias": None, "in_features": 32, "out_features": 16}
    with pytest.raises(KeyError):
        int2.load_int2_weights_to_model(m, {"backbone.no_such_layer": good})
    bad = dict(good, in_features=64)
    with pytest.raises(ValueError):
        int2.load_int2_weights_to_model(m, {"backbone.layers.0.mixer.cross_layer_q_proj": bad})
