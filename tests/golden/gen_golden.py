"""Generate golden vectors by running the reference torch backend.

Run where the reference package is importable (``TESM_REFERENCE`` points at the
project root; default: a ``reference`` directory beside this repository):

    python tests/golden/gen_golden.py

Every case seeds weights with ``torch.manual_seed(0)`` before constructing the
reference module (the b200 mirror modules reproduce the same parameters from the
same seed; ``tests/test_oracle_golden.py`` checks that here) and draws inputs from
``torch.Generator().manual_seed(1)``.  Modules run in ``.eval()`` under
``torch.no_grad()`` with ``kernel_backend="torch"`` in float32 -- the reference's
torch path raises for bfloat16 SISO/MIMO modules (tesm.py:944 einsum dtype
mismatch), so module parity is pinned in float32.  The saved ``.npz`` files hold
inputs' seeds/shapes, outputs, and a SHA-256 of the reference state_dict.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("TESM_REFERENCE") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))), "reference")
sys.path.insert(0, REF)

from tesm_ssm.modules.tesm import BitLinear, TESM_SISO  # noqa: E402
from tesm_ssm.modules.tesm_mimo import TESMMIMO_Optimized  # noqa: E402
from tesm_ssm.models.config_tesm import TESMConfig  # noqa: E402
from tesm_ssm.models.mixer_seq_simple import TESMLMHeadModel  # noqa: E402
from tesm_ssm.utils.int2_quantization import export_model_to_int2, pack_int2_to_uint8  # noqa: E402

import cases  # noqa: E402  (shared case table; no reference import inside)


def sd_hash(module):
    h = hashlib.sha256()
    for k, v in module.state_dict().items():
        h.update(k.encode())
        h.update(v.detach().cpu().contiguous().numpy().tobytes())
    return h.hexdigest()


def randn(shape, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


def save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    print("wrote", path, os.path.getsize(path), "bytes")


def t2n(t):
    return t.detach().cpu().numpy().copy()  # copy: reference caches alias their inputs


def gen_bitlinear():
    for c in cases.BITLINEAR:
        torch.manual_seed(0)
        dt = getattr(torch, c["dtype"])
        lay = BitLinear(c["K"], c["N"], kernel_backend="torch")
        with torch.no_grad():
            lay.weight.copy_(randn((c["N"], c["K"]), 3) * c["wstd"])
        lay = lay.to(dt).eval()
        x = randn(c["xshape"], 1, dt)
        with torch.no_grad():
            y = lay(x)
            qw = lay.quantized_weight()
            scale = 1.0 / lay.weight.abs().mean().clamp_min(lay.bit_eps)
            t = (lay.weight * scale).round().clamp(-1, 1).to(torch.int8)
            sx = 127 / x.abs().max(dim=-1, keepdim=True).values.clamp_min(lay.bit_eps)
            codes = (x * sx).round().clamp(-128, 127).to(torch.int8)
            acc = codes.reshape(-1, c["K"]).int() @ t.int().T
            packed, pscale = pack_int2_to_uint8(lay.weight.float())
        save("bitlinear_" + c["name"], y=t2n(y.float()), t=t2n(t), scale=t2n(scale.float()),
             deq=t2n(qw.float().abs().max()), codes=t2n(codes), sx=t2n(sx.float()), acc=t2n(acc),
             packed=t2n(packed), pscale=t2n(pscale.float()))


def run_siso(c):
    torch.manual_seed(0)
    m = TESM_SISO(kernel_backend="torch", **c["kw"]).eval()
    out = {"sd_sha256": sd_hash(m)}
    B, L = c["B"], c["L"]
    x = randn((B, L, c["kw"]["d_model"]), 1)
    cross = randn((B, L, c["kw"]["d_state"]), 2) if c.get("cross") else None
    prev = randn((B, c["kw"]["d_state"]), 4).double() if c.get("prev") else None
    ip = {"state_cache": m.allocate_inference_cache(B, c["kw"]["max_seq_len"])} if c.get("decode") else None
    with torch.no_grad():
        y, fs = m(x, inference_params=({"state_cache": ip["state_cache"]} if ip else None),
                  cross_layer_state=cross, prev_state=prev)
        out.update(y=t2n(y), final=t2n(fs), states=t2n(m._last_cross_layer_state))
        for s in range(c.get("decode", 0)):
            xt = randn((B, 1, c["kw"]["d_model"]), 10 + s)
            ct = randn((B, c["kw"]["d_state"]), 20 + s) if c.get("cross") else None
            yt, st = m(xt, inference_params={"state_cache": ip["state_cache"]}, cross_layer_state=ct)
            out[f"dec{s}_y"] = t2n(yt)
            out[f"dec{s}_state"] = t2n(st)
        if ip:
            ch = ip["state_cache"]
            out.update(cache_k=t2n(ch["ent_k_cache"]), cache_v=t2n(ch["ent_v_cache"]),
                       cache_idx=np.int64(ch["cache_idx"]), cache_pos=np.int64(ch["seq_pos"]))
    save("siso_" + c["name"], **out)


def run_mimo(c):
    torch.manual_seed(0)
    m = TESMMIMO_Optimized(kernel_backend="torch", **c["kw"]).eval()
    out = {"sd_sha256": sd_hash(m)}
    B, L = c["B"], c["L"]
    H, D = c["kw"]["n_heads"], c["kw"]["d_state"]
    x = randn((B, L, c["kw"]["d_model"]), 1)
    ip = {"state_cache": m.allocate_inference_cache(B, c["kw"]["max_seq_len"])} if c.get("decode") else None
    with torch.no_grad():
        y, fs = m(x, inference_params=({"state_cache": ip["state_cache"]} if ip else None))
        out.update(y=t2n(y), final=t2n(fs), cross=t2n(m._last_cross_layer_state))
        for s in range(c.get("decode", 0)):
            xt = randn((B, 1, c["kw"]["d_model"]), 10 + s)
            ct = randn((B, H, D), 20 + s) if c.get("cross") else None
            yt, st = m(xt, inference_params={"state_cache": ip["state_cache"]}, cross_layer_state=ct)
            out[f"dec{s}_y"] = t2n(yt)
            out[f"dec{s}_state"] = t2n(st)
    save("mimo_" + c["name"], **out)


def run_model(c):
    torch.manual_seed(0)
    cfg = TESMConfig(kernel_backend="torch", **c["cfg"])
    m = TESMLMHeadModel(cfg).eval()
    out = {"sd_sha256": sd_hash(m)}
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (c["B"], c["L"]), generator=g)
    out["ids"] = t2n(ids)
    with torch.no_grad():
        o, _ = m(ids)
        out["logits"] = t2n(o.logits)
        if c.get("decode"):
            ip = {"state_cache": m.backbone.allocate_inference_cache(c["B"], cfg.max_seq_len)}
            o, _ = m(ids, inference_params=ip)
            out["prefill_logits"] = t2n(o.logits)
            for s in range(c["decode"]):
                nt = torch.randint(0, cfg.vocab_size, (c["B"], 1), generator=g)
                o, _ = m(nt, inference_params=ip)
                out[f"dec{s}_ids"] = t2n(nt)
                out[f"dec{s}_logits"] = t2n(o.logits)
    save("model_" + c["name"], **out)


def gen_int2_export():
    """The reference's on-disk INT2 export (export_model_to_int2, int2_quantization.py:196-217) of
    the tiny SISO model of cases.MODEL: per BitLinear its packed bytes and weight_scale."""
    c = cases.MODEL[0]
    torch.manual_seed(0)
    cfg = TESMConfig(kernel_backend="torch", **c["cfg"])
    m = TESMLMHeadModel(cfg).eval()
    ex = export_model_to_int2(m)
    out = {"sd_sha256": sd_hash(m), "names": np.array(sorted(ex))}
    for name, d in ex.items():
        out[name + "/packed"] = t2n(d["packed_weight"])
        out[name + "/scale"] = np.asarray(float(d["weight_scale"]), np.float32)
        out[name + "/shape"] = np.array([d["out_features"], d["in_features"]])
    save("int2_export_tiny", **out)


def gen_scan_rope():
    """Two pieces of the SISO prefill in isolation, at inputs where their fp details show:

    * ``_parallel_state_scan`` (tesm.py:1091-1164) with small decays a = sigmoid(N(0, 1.5) - 1)
      (the in-chunk cumulative product often drops below the 1e-12 clamp) and with the
      module's usual decays (a = sigmoid(N(0,1) + 3));
    * ``_apply_rope`` (tesm.py:783-793) at positions 8000.. for widths 64 and 48, where a
      one-ulp difference in 1/base^(2i/D) moves theta by ~1e-3 rad.
    """
    torch.manual_seed(0)
    m = TESM_SISO(d_model=64, d_state=32, ent_rank=16, entanglement_window=8, max_seq_len=64,
                  kernel_backend="torch").eval()
    out = {}
    B, L, D = 2, 100, 32
    with torch.no_grad():
        for name, shift, sd in (("small", -1.0, 1.5), ("usual", 3.0, 1.0)):
            a = torch.sigmoid(randn((B, L, D), 30) * sd + shift)
            u = randn((B, L, D), 31) * 0.5
            st = m._parallel_state_scan(a, u)
            out[f"scan_{name}_a"] = t2n(a)
            out[f"scan_{name}_u"] = t2n(u)
            out[f"scan_{name}_states"] = t2n(st)
            out[f"scan_{name}_final"] = t2n(m._last_scan_state_f64)
        for R in (64, 48):
            x = randn((1, 24, R), 32 + R)
            out[f"rope{R}_x"] = t2n(x)
            out[f"rope{R}_y"] = t2n(m._apply_rope(x, pos_offset=8000))
    save("scan_rope", **out)


if __name__ == "__main__":
    torch.set_num_threads(8)
    if len(sys.argv) > 1:  # regenerate selected groups only, e.g. "scan_rope"
        for name in sys.argv[1:]:
            globals()["gen_" + name]()
        sys.exit(0)
    gen_scan_rope()
    gen_bitlinear()
    for c in cases.SISO:
        run_siso(c)
    for c in cases.MIMO:
        run_mimo(c)
    for c in cases.MODEL:
        run_model(c)
    gen_int2_export()
