"""bitdance_b200 -- B200-native (sm_100a) W4A6 GEMM: MXFP6 activations times NVFP4 weights
transcoded on chip to MXFP6, block-scaled tcgen05 tensor-core MMAs, bf16 output.

The compute lives in ``libbitdance_b200.so`` (C ABI: include/bitdance_b200.h); this package
is its Python host side. ``psg`` mirrors the reference operator ``compile_preshuffle_gemm_a8``.
"""
from ._lib import BitdanceError, load  # noqa: F401
from .ops import (PackedActivations, PackedWeights, Workspace, device_error,  # noqa: F401
                  mma_peak_tflops,
                  pack_activations, pack_weights, quantize_activations, quantize_mxfp6,
                  quantize_nvfp4, quantize_weights, query_workspace, tensor_scale_of,
                  transcode, w4a6_gemm, w4a6_gemm_noalloc, w4a6_linear)

__version__ = "0.1.0"
