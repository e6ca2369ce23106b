"""The device quantisers against fixtures written by the REFERENCE's own code
(tests/golden/make_golden.py): the direct-MXFP6 activation quantiser vq.quantize(x, E8M0, E2M3)
(vector_quant_error.py:305, :389) on activations with an outlier channel, and the two-level
per-16 NVFP4 encode (remote/quant_real_weights.py:273-287 + encode_nvfp4,
kernel/nvfp4_codec.py:34-63). Bit-exact on the GPU, like the oracle in tests/test_oracle.py."""
import os

import numpy as np
import pytest

import w4a6_oracle as o

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


@pytest.mark.parametrize("dtype", [torch.float32])
def test_activation_quantiser_matches_reference_fixture(dtype):
    import bitdance_b200 as bd
    g = golden("amxfp6.npz")
    codes, e8 = bd.quantize_mxfp6(torch.from_numpy(g["x"]).to(dtype).cuda())
    codes, e8 = codes.cpu().numpy(), e8.cpu().numpy()
    assert np.array_equal(e8.reshape(-1).astype(np.int64) - 127, g["exp"])
    val = np.where((codes >> 5) & 1, -1.0, 1.0) * o.E2M3_POS[codes & 31]
    assert np.array_equal(np.abs(val), np.abs(g["data"]))
    assert np.array_equal(val[g["data"] != 0], g["data"][g["data"] != 0])
    assert not np.any(((codes & 31) == 0) & (((codes >> 5) & 1) == 1))  # no negative zeros


def test_weight_quantiser_matches_reference_fixture():
    import bitdance_b200 as bd
    g = golden("encode16.npz")
    codes, scales, tstat = bd.quantize_nvfp4(torch.from_numpy(g["w"]).cuda())
    assert np.float32(bd.tensor_scale_of(tstat)) == g["s_t"][0]
    assert np.array_equal(scales.cpu().numpy().reshape(-1), g["scales"])
    assert np.array_equal(o.unpack_nibbles(codes.cpu().numpy()).reshape(-1, 16), g["codes"])
    assert bd.device_error() == 0
