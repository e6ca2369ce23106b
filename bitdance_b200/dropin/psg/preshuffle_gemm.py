"""``psg.preshuffle_gemm.compile_preshuffle_gemm_a8``: this library's operator
(``bitdance_b200.psg``), which keeps the reference's signature, argument order, buffer sizes
and exceptions (psg_preshuffle_gemm.py:251-277, 3211-3253)."""
import os
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from bitdance_b200.psg import compile_preshuffle_gemm_a8  # noqa: E402,F401
