"""The "b200" rung patched into the reference's own classes (tesm_b200.integration).

Runs where the reference package is importable (``TESM_REFERENCE`` names its project root,
default: a ``reference`` directory beside this repository); skipped elsewhere.  Without a GPU the rung must raise the reference-style "backend not
available" error for kernel_backend="b200" (no CPU fallback), leave every other backend on
the reference's own path, and be reversible."""
import importlib
import os
import sys

import pytest
import torch

REF = os.environ.get("TESM_REFERENCE") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")
if os.path.isdir(REF) and REF not in sys.path:
    sys.path.insert(0, REF)
try:
    importlib.import_module("tesm_ssm.modules.tesm")
    HAVE_REF = True
except Exception:
    HAVE_REF = False

pytestmark = pytest.mark.skipif(not HAVE_REF, reason="reference package (tesm_ssm) not importable")


@pytest.fixture
def installed():
    from tesm_b200 import integration
    n = integration.install()
    yield n
    integration.uninstall()


def test_install_routes_every_forward(installed):
    assert installed >= 6


def test_bitlinear_b200_rung_is_strict(installed):
    from tesm_ssm.modules.tesm import BitLinear
    torch.manual_seed(0)
    lin = BitLinear(64, 32, kernel_backend="b200").eval()
    with torch.no_grad(), pytest.raises(RuntimeError, match="kernel_backend='b200' specified but BitLinear kernel"):
        lin(torch.randn(2, 64))


def test_other_backends_untouched(installed):
    from tesm_ssm.modules.tesm import BitLinear
    torch.manual_seed(0)
    lin = BitLinear(64, 32, kernel_backend="torch").eval()
    x = torch.randn(2, 64)
    with torch.no_grad():
        y = lin(x)
    from tesm_b200 import integration
    integration.uninstall()
    with torch.no_grad():
        y0 = lin(x)
    integration.install()
    assert torch.equal(y, y0)


def test_model_rung_is_strict(installed):
    from tesm_ssm.models.config_tesm import TESMConfig
    from tesm_ssm.models.mixer_seq_simple import TESMLMHeadModel
    torch.manual_seed(0)
    cfg = TESMConfig(n_layer=1, d_model=64, d_state=16, ent_rank=8, vocab_size=64, d_intermediate=128,
                     max_seq_len=32, kernel_backend="b200")
    m = TESMLMHeadModel(cfg).eval()
    with torch.no_grad(), pytest.raises(RuntimeError, match="kernel_backend='b200' specified but"):
        m(torch.randint(0, 64, (1, 8)))


def test_uninstall_restores():
    from tesm_b200 import integration
    from tesm_ssm.modules.tesm import TESM_SISO
    orig = TESM_SISO.forward
    integration.install()
    assert TESM_SISO.forward is not orig
    integration.uninstall()
    assert TESM_SISO.forward is orig
