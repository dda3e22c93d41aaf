"""Host-side logic of the drop-in API (no GPU needed)."""
import numpy as np
import pytest
import torch

import metalfaiss_b200 as mf
from metalfaiss_b200 import FlatIndex, IVFFlatIndex, MetricType, SearchRangeResult, SearchResult
from metalfaiss_b200.errors import CudaError, ErrorCode, InvalidArgumentError, check_error


def test_metric_values_are_faiss_integers():
    """python/metalfaiss/unittest/test_metric_type.py:29-40."""
    assert MetricType.INNER_PRODUCT == 0 and MetricType.L2 == 1 and MetricType.L1 == 2
    assert MetricType.LINF == 3 and MetricType.LP == 4
    assert MetricType.CANBERRA == 20 and MetricType.BRAY_CURTIS == 21
    assert MetricType.JENSEN_SHANNON == 22 and MetricType.JACCARD == 23
    assert MetricType.Linf is MetricType.LINF


def test_metric_coercion():
    assert MetricType.coerce("l2") is MetricType.L2
    assert MetricType.coerce("Linf") is MetricType.LINF
    assert MetricType.coerce("inner_product") is MetricType.INNER_PRODUCT
    assert MetricType.coerce(1) is MetricType.L2

    class Foreign:  # a member of one of the reference's other enums
        name = "INNER_PRODUCT"
        value = "inner_product"

    assert MetricType.coerce(Foreign()) is MetricType.INNER_PRODUCT
    with pytest.raises(ValueError):
        MetricType.from_string("cosine")


def test_unsupported_metric_raises_not_implemented():
    with pytest.raises(NotImplementedError):
        FlatIndex(8, MetricType.CANBERRA)


def test_search_result_contract():
    d = torch.zeros((3, 4))
    i = torch.zeros((3, 4), dtype=torch.int64)
    r = SearchResult(d, i)
    D, I = r
    assert D is d and I is i and r.labels is i and len(r) == 3
    with pytest.raises(ValueError):
        SearchResult(torch.zeros((3, 4)), torch.zeros((3, 5), dtype=torch.int64))
    rr = SearchRangeResult(torch.tensor([1.0, 2.0, 3.0]), torch.tensor([4, 5, 6]),
                           torch.tensor([0, 2, 2, 3]))
    assert len(rr) == 3 and rr.get_total_size() == 3
    dq, iq = rr[0]
    assert iq.tolist() == [4, 5]


def test_error_mapping():
    with pytest.raises(ValueError) as e:
        check_error(int(ErrorCode.INVALID_ARGS), "bad")
    assert e.value.code == ErrorCode.INVALID_ARGS
    with pytest.raises(RuntimeError):
        check_error(int(ErrorCode.BAD_STATE), "state")
    with pytest.raises(TimeoutError):
        check_error(int(ErrorCode.TIMEOUT), "late")
    assert mf.get_last_error() is not None
    mf.clear_last_error()
    assert mf.get_last_error() is None


def test_ivf_constructor_forms_and_nprobe():
    q = FlatIndex(16)
    a = IVFFlatIndex(q, 16, 8)  # reference signature (ivf_flat_index.py:24)
    b = IVFFlatIndex(16, 8)  # test signature (test_mlx_index.py:54)
    c = IVFFlatIndex(16, 8, quantizer=q)  # test signature (test_mlx_index.py:84)
    for idx in (a, b, c):
        assert idx.nlist == 8 and idx.nprobe == 1 and not idx.is_trained and idx.ntotal == 0
    with pytest.raises(ValueError):
        a.nprobe = 0
    a.nprobe = 5
    assert a.nprobe == 5
    with pytest.raises(RuntimeError):
        b.add(np.zeros((2, 16), np.float32))  # untrained (ivf_flat_index.py:81-82)
    with pytest.raises(ValueError):
        IVFFlatIndex(FlatIndex(8), 16, 4)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
    idx = FlatIndex(8)
    with pytest.raises(CudaError):
        idx.add(np.zeros((2, 8), np.float32))


def test_dimension_checks_before_device_work():
    from metalfaiss_b200._tensors import as_matrix, padded_dim

    assert padded_dim(1) == 4 and padded_dim(64) == 64 and padded_dim(65) == 68
    t = as_matrix(np.ones((2, 5), np.float32), 5, torch.device("cpu"))
    assert t.shape == (2, 8) and float(t[:, 5:].abs().sum()) == 0.0
    with pytest.raises(InvalidArgumentError):
        as_matrix(np.ones((2, 6), np.float32), 5, torch.device("cpu"))
