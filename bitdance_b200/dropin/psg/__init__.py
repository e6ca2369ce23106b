"""``psg``: the reference's package name for its preshuffle GEMM (psg_preshuffle_gemm.py)."""
