"""The row-softmax oracle against the reference's own CPU softmax and autograd (CPU)."""
import numpy as np
import pytest

from conftest import REPO
from oracle import softmax as S

GOLDEN = np.load(REPO / "tests" / "golden" / "softmax.npz")
CASES = {"plain": {}, "masked": {"mask": GOLDEN["masked_mask"]},
         "causal": {"causal": True, "offset": int(GOLDEN["causal_offset"])},
         # NaN / +inf in the blocked positions: the reference fills them with -inf first
         "causal_poisoned": {"causal": True, "offset": int(GOLDEN["causal_offset"])}}


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_matches_reference_bit_for_bit(name):
    y, status = S.forward(GOLDEN[f"{name}_x"], **CASES[name])
    np.testing.assert_array_equal(y, GOLDEN[f"{name}_y"])
    np.testing.assert_array_equal(S.backward(y, GOLDEN[f"{name}_g"], **CASES[name]), GOLDEN[f"{name}_dx"])
    assert not status.any()


def test_mask_rows_follow_reference_broadcast_rules():
    assert S.mask_rows((40,), (2, 3, 5, 40)) == 1                 # one row shared by all
    assert S.mask_rows((1, 1), (4, 8)) == 0
    assert S.mask_rows((5, 40), (2, 3, 5, 40)) == 5
    assert S.mask_rows((3, 5, 40), (2, 3, 5, 40)) == 15
    assert S.mask_rows((2, 1, 5, 40), (2, 3, 5, 40)) is None      # a hole in the broadcast
    assert S.mask_rows((5, 1), (2, 3, 5, 40)) is None             # the column dimension must match


def test_empty_and_invalid_rows():
    x = np.array([[1.0, 2.0, 3.0], [-np.inf, -np.inf, -np.inf], [1.0, np.nan, 0.0], [np.inf, 0.0, 1.0]],
                 np.float32)
    y, status = S.forward(x)
    assert status.tolist() == [0, 1, 2, 2]
    assert np.all(y[1] == 0) and np.all(np.isnan(y[2])) and np.all(np.isnan(y[3]))
