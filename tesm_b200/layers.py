"""Forward paths of the b200 backend, shared by the mirror modules and by the
patch that adds the "b200" rung to the reference classes (integration.py).

Functions read the reference's attribute names off the module they are given,
so the same code serves ``tesm_b200.modules.TESM_SISO`` and the reference's
``tesm_ssm.modules.tesm.TESM_SISO``.
"""
from __future__ import annotations

import torch

from . import ops
from ._lib import TesmError

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


# ------------------------------------------------------------------ BitLinear
def packed_weight(lin) -> ops.PackedWeight:
    """Device ternary weight of a BitLinear, rebuilt whenever the weight changes
    (mirrors the eval-mode cache keyed on weight._version, tesm.py:226-236)."""
    w = lin.weight
    key = (w.data_ptr(), w._version, w.dtype, tuple(w.shape))
    cache = getattr(lin, "_b200", None)
    if cache is None or cache[0] != key:
        wc = w.detach()
        if wc.stride(1) != 1:
            wc = wc.contiguous()
        pw = ops.pack_weight(wc, lin.bit_eps, per_row=False, with_tern=False)
        cache = (key, pw, wc)
        lin._b200 = cache
    return cache[1]


def _pw_for_m(lin, M):
    pw = packed_weight(lin)
    if M > ops.GEMV_MAX_M:
        ops.ensure_tern(pw, lin._b200[2])
    return pw


def bitlinear_2d(lin, x2d, out_dtype=None, out=None):
    pw = _pw_for_m(lin, x2d.shape[0])
    if x2d.stride(1) != 1:
        x2d = x2d.contiguous()
    y = ops.bitlinear_2d(x2d, pw, lin.bit_eps, out_dtype or x2d.dtype, out)
    if lin.bias is not None:
        raise TesmError("tesm_b200: BitLinear with bias is not on the reference hot path (bias=False everywhere)")
    return y


def bitlinear_forward(lin, x):
    """``BitLinear.forward`` (tesm.py:287-290): output in the input dtype."""
    shp = x.shape
    x2d = x.reshape(-1, shp[-1])
    y = bitlinear_2d(lin, x2d)
    return y.reshape(*shp[:-1], lin.out_features)


# ------------------------------------------------------------------ placeholders
def _todo(*a, **k):
    raise NotImplementedError("tesm_b200: path not built yet")


siso_alloc_cache = mimo_alloc_cache = siso_prefill = siso_decode = mimo_prefill = mimo_decode = _todo
rmsnorm = block_forward = ffn_forward = mixer_model_forward = lm_forward = generate = _todo
