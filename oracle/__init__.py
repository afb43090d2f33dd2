"""CPU oracle for the TESM inference hot path (test infrastructure only).

This package restates, in numpy, the arithmetic of the reference's torch
backend (WANGLILIN360/tesm, ``tesm_ssm/modules/tesm.py``,
``tesm_ssm/modules/tesm_mimo.py``, ``tesm_ssm/models/mixer_seq_simple.py``,
``tesm_ssm/utils/int2_quantization.py``).  It is the checker for the CUDA
library, never part of the product: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` import it.

Parity pin: the restatement is checked against golden vectors produced by
running the reference itself (``tests/golden/gen_golden.py``) in a container
where the reference is importable; the committed ``tests/golden/*.npz`` carry
those outputs to machines that lack the reference.
"""
from .tesm_oracle import *  # noqa: F401,F403
