"""``kernel``: the reference's module directory; only ``nvfp4_mxfp6_gemm_tiled`` is provided."""
