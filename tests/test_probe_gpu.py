"""The tensor-core peak probe (bd_probe_mma_peak): back-to-back block-scaled
tcgen05.mma.kind::mxf8f6f4 MMAs, one CTA per SM, end without a device error and give a rate in
the range a B200 can reach (the dense FP8/FP6 peak is 4.5 PFLOP/s nominal)."""
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("a_from_tmem", [False, True])
def test_probe_rate_is_sane(a_from_tmem):
    import bitdance_b200 as bd
    tf = bd.mma_peak_tflops(n_cols=256, a_from_tmem=a_from_tmem, mmas_per_cta=1 << 15)
    assert 1000.0 < tf < 5000.0, tf
    assert bd.device_error() == 0


def test_pair_probe_rate_is_sane():
    """The CTA-pair form (cta_group::2, M = 256 over a cluster of two CTAs): ends without a
    device error, at a rate per SM in the same range as the single-CTA form."""
    import bitdance_b200 as bd
    tf = bd.mma_peak_tflops(pair=True, mmas_per_cta=1 << 15)
    assert 1000.0 < tf < 5000.0, tf
    assert bd.device_error() == 0


def test_probe_narrow_n_is_no_faster_per_instruction():
    """An MMA of N = 64 columns does a quarter of the work of N = 256; it must not take longer
    per instruction than the wide one (the rate per column is what the GEMM's layout relies on:
    the weights are the MMA's 256-wide N operand)."""
    import bitdance_b200 as bd
    wide = bd.mma_peak_tflops(n_cols=256, mmas_per_cta=1 << 15)
    narrow = bd.mma_peak_tflops(n_cols=64, mmas_per_cta=1 << 15)
    # time per instruction = flops / rate: narrow's must not exceed wide's
    assert 64 / narrow <= 256 / wide * 1.05, (wide, narrow)


def test_probe_rejects_bad_arguments():
    import bitdance_b200 as bd
    from bitdance_b200 import BitdanceError, _lib
    from bitdance_b200._lib import call
    for n_mma, n_cols, form in ((0, 256, 0), (1 << 22, 256, 0), (1024, 24, 0), (1024, 272, 0),
                                (1024, 128, 2), (1024, 256, 3), (1024, 256, -1)):
        with pytest.raises(BitdanceError) as e:
            call("bd_probe_mma_peak", n_mma, n_cols, form, None)
        assert e.value.status == _lib.BD_ERR_INVALID_ARG
    assert bd.device_error() == 0
