"""tesm_b200: B200-native (sm_100a) inference hot path for TESM.

Registers as ``kernel_backend="b200"`` behind the reference's module API
(BitLinear, TESM_SISO, TESMMIMO_Optimized, TESMLMHeadModel).  Two ways in:

* the mirror classes in :mod:`tesm_b200.modules` / :mod:`tesm_b200.models`
  (same signatures, parameter names and seeded init as the reference);
* :func:`tesm_b200.integration.install`, which adds a "b200" rung to the
  reference's own classes when the reference package is importable.
"""
from .modules import BitLinear, Block, RMSNorm, TESM, TESM_SISO, TESMMIMO_Optimized  # noqa: F401
from .models import FeedForward, MixerModel, TESMCausalLMOutput, TESMConfig, TESMLMHeadModel  # noqa: F401

__version__ = "0.1.0"
