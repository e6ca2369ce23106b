"""Drop-in module tree for the reference's operator scripts.

kernel/verify_w4a6.py and kernel/bench_sweep.py (scimg/bitdance) import ``flydsl.compiler``,
``flydsl.expr``, ``flydsl.compiler.jit_argument.from_c_void_p``,
``psg.preshuffle_gemm.compile_preshuffle_gemm_a8`` and (verify_w4a6.py only)
``kernel.nvfp4_mxfp6_gemm_tiled.build_LUT12``. With this directory on PYTHONPATH those imports
resolve to the modules here, which route every launch to this library's sm_100a GEMM through
``bitdance_b200.psg``:

    PYTHONPATH=<repo>/bitdance_b200/dropin python kernel/verify_w4a6.py --dtype w6a6_tc \\
        --a_uniform_byte --a_val 3.25

This directory is not itself a package the library imports; nothing in ``bitdance_b200``
depends on it.
"""
