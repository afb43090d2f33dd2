"""On-disk INT2 weights: the reference's export format (tesm_ssm/utils/int2_quantization.py).

``export_model_to_int2`` (int2_quantization.py:196-217) writes, per BitLinear, the packed
ternary bytes of ``pack_int2_to_uint8`` (:21-60: code t+1, four per byte, lowest column in the
low bits, K padded to a multiple of 4 with code 1) and ``weight_scale = 1 / mean|W|``.  Loading
such an export here keeps the bytes as they are -- no round trip through latent weights -- and
installs them as the ternary weight of the matching b200 BitLinear:

* the module still runs BitLinear's forward (per-token int8 activation quantisation,
  tesm.py:206-209, then the int8 x ternary GEMM); the dequantisation factor is
  fl(1 / weight_scale), which equals BitLinear's absmean scale up to one rounding;
* the reference's own loader instead swaps each BitLinear for an ``Int2Linear`` that multiplies
  unquantised activations (:115-173, :220-245); that layer is not reproduced;
* imported weights take precedence over the latent ``weight`` until ``clear_int2_weights``;
  capture decode CUDA graphs after importing; tensor-parallel shards are not cut from imports.
"""
from __future__ import annotations

from typing import Dict

import torch

from . import ops
from .layers import packed_weight


def _bitlinears(model: torch.nn.Module):
    for name, mod in model.named_modules():
        if hasattr(mod, "bit_eps") and hasattr(mod, "weight") and hasattr(mod, "in_features"):
            yield name, mod


def export_model_to_int2(model: torch.nn.Module) -> Dict[str, Dict]:
    """Per BitLinear {packed_weight (uint8, N x ceil(K/4)), weight_scale, bias, in_features,
    out_features}, the dictionary ``export_model_to_int2`` of the reference writes."""
    out = {}
    for name, lin in _bitlinears(model):
        pw = packed_weight(lin)
        K = lin.in_features
        out[name] = {
            "packed_weight": pw.packed[:, :(K + 3) // 4].cpu().clone(),
            "weight_scale": pw.scale.reshape(()).cpu().clone(),
            "bias": lin.bias.detach().cpu() if lin.bias is not None else None,
            "in_features": K,
            "out_features": lin.out_features,
        }
    return out


def load_int2_weights_to_model(model: torch.nn.Module, exported: Dict[str, Dict]) -> int:
    """Install the exported INT2 weights into the model's BitLinear layers (on the device of
    each layer's latent weight).  Returns the number of layers loaded; a layer name absent from
    the model, or a shape mismatch, raises."""
    lins = dict(_bitlinears(model))
    n = 0
    for name, d in exported.items():
        if name not in lins:
            raise KeyError(f"INT2 export has layer {name!r}, which the model does not")
        lin = lins[name]
        if (d["out_features"], d["in_features"]) != (lin.out_features, lin.in_features):
            raise ValueError(f"{name}: export is {d['out_features']} x {d['in_features']}, "
                             f"layer is {lin.out_features} x {lin.in_features}")
        if d.get("bias") is not None or lin.bias is not None:
            raise ValueError(f"{name}: BitLinear bias is not on the reference hot path")
        dev = lin.weight.device
        lin.__dict__["_b200_int2"] = ops.packed_from_int2(torch.as_tensor(d["packed_weight"]),
                                                          torch.as_tensor(d["weight_scale"]), lin.in_features, dev)
        n += 1
    return n


def clear_int2_weights(model: torch.nn.Module) -> None:
    """Return every BitLinear to its latent weight."""
    for _, lin in _bitlinears(model):
        lin.__dict__.pop("_b200_int2", None)


def save_int2_model(model: torch.nn.Module, path: str) -> None:
    torch.save(export_model_to_int2(model), path)


def load_int2_model(model: torch.nn.Module, path: str) -> int:
    return load_int2_weights_to_model(model, torch.load(path, weights_only=False))
