"""The "b200" rung inside the reference's own classes.

``install()`` patches the forward methods of an imported ``tesm_ssm`` package so that a module
whose ``kernel_backend`` is ``"b200"`` runs this library's path, and every other backend string
keeps the reference's behaviour unchanged.  The reference's classes accept any backend string
and fall through to their "backend not available" RuntimeError for unknown ones
(tesm.py:279-285); the rung is checked first, as in the reference's dispatch ladders
(BitLinear._project_quantized tesm.py:238, TESM_SISO.forward :1175, TESMMIMO_Optimized.forward
tesm_mimo.py:914).  The patch is a subclass-free method swap, reversible with ``uninstall()``;
the reference's files are not modified.

The b200 functions read the reference's attribute names, so the same code serves the mirror
classes of :mod:`tesm_b200.modules` / :mod:`tesm_b200.models` and the reference instances.
"""
from __future__ import annotations

import importlib
from typing import Dict, Tuple

from . import models as _models
from . import modules as _modules

B200 = "b200"
_ORIG: Dict[Tuple[str, str], object] = {}


def _backend_of(obj) -> str:
    """The kernel_backend governing a reference module instance."""
    for path in (("kernel_backend",), ("mixer", "kernel_backend"), ("gate_proj", "kernel_backend"),
                 ("config", "kernel_backend"), ("tesm_config", "kernel_backend")):
        o = obj
        for a in path:
            o = getattr(o, a, None)
            if o is None:
                break
        if isinstance(o, str):
            return o
    return ""


def _wrap(orig, mirror):
    def forward(self, *args, **kwargs):
        if _backend_of(self) == B200:
            return mirror(self, *args, **kwargs)
        return orig(self, *args, **kwargs)
    forward.__wrapped__ = orig
    forward.__doc__ = orig.__doc__
    return forward


# (module path, class name, mirror forward, extra methods to route)
_TARGETS = [
    ("tesm_ssm.modules.tesm", "BitLinear", _modules.BitLinear.forward),
    ("tesm_ssm.modules.tesm", "TESM_SISO", _modules.TESM_SISO.forward),
    ("tesm_ssm.modules.tesm_mimo", "TESMMIMO_Optimized", _modules.TESMMIMO_Optimized.forward),
    ("tesm_ssm.modules.block", "Block", _modules.Block.forward),
    ("tesm_ssm.models.mixer_seq_simple", "FeedForward", _models.FeedForward.forward),
    ("tesm_ssm.models.mixer_seq_simple", "MixerModel", _models.MixerModel.forward),
    ("tesm_ssm.models.mixer_seq_simple", "TESMLMHeadModel", _models.TESMLMHeadModel.forward),
]


def install() -> int:
    """Patch the imported reference package; returns the number of forwards routed.  Classes
    missing from the installed reference version are skipped."""
    n = 0
    for mod_name, cls_name, mirror in _TARGETS:
        try:
            cls = getattr(importlib.import_module(mod_name), cls_name)
        except (ImportError, AttributeError):
            continue
        key = (mod_name, cls_name)
        if key in _ORIG:
            continue
        _ORIG[key] = cls.forward
        cls.forward = _wrap(cls.forward, mirror)
        n += 1
    return n


def uninstall() -> None:
    for (mod_name, cls_name), orig in list(_ORIG.items()):
        cls = getattr(importlib.import_module(mod_name), cls_name)
        cls.forward = orig
        del _ORIG[(mod_name, cls_name)]
