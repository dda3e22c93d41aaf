"""Host-side parts of the FAISS-style facade: factory strings, normalize_L2."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import faiss_compat as fc
from metalfaiss_b200.errors import InvalidArgumentError


@pytest.mark.parametrize("s", ["HNSW32,Flat", "IVF,Flat", "PQ8", "IVF16,SQ8", ""])
def test_unsupported_factory_strings(s):
    with pytest.raises(InvalidArgumentError):
        fc.index_factory(8, s)


def test_normalize_l2_numpy_and_torch():
    x = np.array([[3.0, 4.0], [0.0, 0.0]], np.float32)
    out = fc.normalize_L2(x)
    assert out is x
    np.testing.assert_allclose(x, [[0.6, 0.8], [0.0, 0.0]])
    t = torch.tensor([[0.0, 2.0], [1.0, 1.0]])
    fc.normalize_L2(t)
    torch.testing.assert_close(t, torch.tensor([[0.0, 1.0], [2 ** -0.5, 2 ** -0.5]]))
