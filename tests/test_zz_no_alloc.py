"""The allocation-free scan entry point against the workspace one (GPU).

tesm_b200_siso_scan_noalloc serves callers that cannot allocate device memory: it keeps
the look-back scratch in a fixed array inside the library instead of a caller workspace.
Both entry points are called through the C ABI on the same inputs, twice in a row with
different inputs (the shared array keeps the previous call's contents, which must not
leak), with fp32 projections (shared-memory kernel) and bf16 ones (register-resident
kernel, whose carry words start from an all-ones "not yet written" pattern inside the
array), and must agree within the scan tolerance (max-rel 1e-5).  This file is collected
last so a failing run that stops at the first failure has run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import max_rel, randn

pytestmark = pytest.mark.gpu


def _scan_both(lib, seed, B, L, D, h0, dtype):
    from tesm_b200 import _lib, ops
    Dm, R = 32, 16
    N = 2 * Dm + 3 * D + 2 * R  # even, so bf16 rows keep 4-byte aligned channel pairs
    proj = (randn((B * L, N), seed)).to(dtype).cuda()
    db = (torch.full((D,), 3.0) + randn((D,), seed + 1) * 0.5).cuda()
    prev = randn((B, D), seed + 2).double().cuda() if h0 else None
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for variant in ("workspace", "noalloc"):
        states = torch.full((B * L, D), float("nan"), device="cuda")
        f32 = torch.empty(B, D, device="cuda")
        f64 = torch.empty(B, D, device="cuda", dtype=torch.float64)
        args = [proj.data_ptr(), ops.dtype_code(dtype), proj.stride(0), B, L, Dm, D, R, 16, db.data_ptr(),
                prev.data_ptr() if prev is not None else None, states.data_ptr(), f32.data_ptr(), f64.data_ptr()]
        if variant == "workspace":
            n = ctypes.c_int64(0)
            assert lib.tesm_b200_scan_workspace(B, L, D, 1, ctypes.addressof(n)) == 0
            ws = torch.empty(n.value, device="cuda", dtype=torch.uint8)
            rc = lib.tesm_b200_siso_scan(*args, ws.data_ptr(), ws.numel(), st)
        else:
            rc = lib.tesm_b200_siso_scan_noalloc(*args, st)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        outs.append((states.cpu().numpy(), f64.cpu().numpy()))
    return outs


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_noalloc_matches_workspace_scan_twice(lib, dtype):
    # two calls in a row with different shapes and inputs
    for seed, (B, L, D, h0) in [(100, (2, 1000, 256, True)), (200, (3, 300, 96, False))]:
        (s_ws, f_ws), (s_na, f_na) = _scan_both(lib, seed, B, L, D, h0, dtype)
        assert np.isfinite(s_na).all()
        assert max_rel(s_na, s_ws) <= 1e-5
        assert max_rel(f_na, f_ws) <= 1e-5


def test_noalloc_rejects_oversized_shapes(lib):
    from tesm_b200 import _lib
    # 64 x 8192 positions x d_state 256 needs ~100 MiB of scratch, above the fixed 8 MiB.  No
    # device pointers are passed: the size check answers first, and if it ever stopped doing
    # so the scan's own null-pointer check would refuse the call before any launch.
    rc = lib.tesm_b200_siso_scan_noalloc(None, 0, 2000, 64, 8192, 16, 256, 16, 16, None, None, None, None, None,
                                         None)
    assert rc == 5 and "above the fixed" in _lib.last_error()
