"""BLAS flag normalisation (the reference's trnblas/_flags.py semantics)."""

import pytest

from trnblas_b200._flags import diag_flag, side_flag, trans_flag, uplo_flag


def test_words_and_letters():
    assert uplo_flag("U") == uplo_flag("upper") == uplo_flag(" Upper ") == "upper"
    assert uplo_flag("l") == "lower"
    assert side_flag("R") == "right" and side_flag("left") == "left"
    assert diag_flag("U") == "unit" and diag_flag("non-unit") == diag_flag("N") == "nonunit"
    assert trans_flag("N") is False and trans_flag("t") is True
    assert trans_flag(1) is True and trans_flag(0) is False


@pytest.mark.parametrize("fn,bad", [(uplo_flag, "x"), (side_flag, "up"), (diag_flag, 3), (uplo_flag, None)])
def test_bad_words_raise(fn, bad):
    with pytest.raises(ValueError):
        fn(bad)


def test_conjugate_transpose_rejected():
    with pytest.raises(ValueError):
        trans_flag("C", "transA")


def test_public_api_validates_flags_before_any_device_work():
    import torch

    import trnblas_b200 as tb

    with pytest.raises(ValueError):
        tb.gemm(1.0, torch.ones(2, 2), torch.ones(2, 2), transA="C")
    with pytest.raises(ValueError):
        tb.syrk(1.0, torch.ones(2, 2), uplo="middle")
    with pytest.raises(TypeError):
        tb.gemm_fp64(torch.ones(2, 2), torch.ones(2, 2), slices=True)
    with pytest.raises(ValueError):
        tb.gemm_fp64(torch.ones(2, 2), torch.ones(2, 2), slices=0)
    with pytest.raises(ValueError):
        tb.set_backend("tpu")
    tb.set_backend("pytorch")
    assert tb.get_backend() == "pytorch"
    tb.set_backend("auto")
