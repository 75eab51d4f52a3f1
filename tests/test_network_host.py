"""contract_network's label validation (host only, no GPU needed)."""

from __future__ import annotations

import numpy as np
import pytest


def _t(ndt, *shape):
    return ndt.TensorF64.from_numpy(np.zeros(shape))


def test_network_rejects_bad_labels(ndt):
    a, b = _t(ndt, 2, 3), _t(ndt, 3, 4)
    with pytest.raises(ValueError, match="labels for a rank"):
        ndt.contract_network([a, b], [[1, -1, 5], [-1, 2]])
    with pytest.raises(ValueError, match="extents"):
        ndt.contract_network([a, _t(ndt, 4, 4)], [[1, -1], [-1, 2]])
    with pytest.raises(ValueError, match="exactly 2"):
        ndt.contract_network([a, b, _t(ndt, 3)], [[1, -1], [-1, 2], [-1]])
    with pytest.raises(ValueError, match="open label"):
        ndt.contract_network([a, _t(ndt, 3, 2)], [[1, -1], [-1, 1]])
    with pytest.raises(ValueError, match="repeated"):
        ndt.contract_network([_t(ndt, 3, 3)], [[-1, -1]])
    with pytest.raises(ValueError, match="label 0"):
        ndt.contract_network([a, b], [[0, -1], [-1, 2]])
    with pytest.raises(ValueError, match="one label list"):
        ndt.contract_network([a, b], [[1, -1]])
