"""Host-side decode-step conventions that need no GPU."""
import torch

from tesm_b200 import layers


def test_state_out_is_a_snapshot():
    """A decode step returns its new fp64 state as a tensor of its own (the reference rebinds
    cache['state'] each step, tesm.py:1385-1400), while the cache here is updated in place."""
    cache = {"state": torch.arange(6, dtype=torch.float64).view(2, 3)}
    out = layers._state_out(cache)
    assert torch.equal(out, cache["state"]) and out.data_ptr() != cache["state"].data_ptr()
    cache["state"].add_(1.0)  # the next step's in-place update must not reach the returned state
    assert torch.equal(out, torch.arange(6, dtype=torch.float64).view(2, 3))


def test_state_out_skipped_for_discarding_callers():
    """Captured decode graphs and generate() mark the caches: no snapshot is made."""
    cache = {"state": torch.zeros(2, 3, dtype=torch.float64), "_b200_no_state_out": True}
    assert layers._state_out(cache) is None
