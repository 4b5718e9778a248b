"""The oracle against its committed fixtures (tests/golden/golden.npz,
written by tests/golden/make_golden.py): the crate's demo model, its
kernel.rs test programs, the MLP workload and a small f32 block.  Indices
must be equal; values within 1e-6 relative, max-abs normalised (the fixtures
are fp32 results of the same code, so only a libm's last bit may move)."""
import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import make_golden  # noqa: E402

GOLDEN = np.load(HERE / "golden" / "golden.npz")


@pytest.fixture(scope="module")
def fresh():
    return make_golden.compute()


def test_fixture_keys(fresh):
    assert sorted(fresh) == sorted(GOLDEN.files)


@pytest.mark.parametrize("key", sorted(GOLDEN.files))
def test_oracle_reproduces_fixture(fresh, key):
    got, want = np.asarray(fresh[key]), GOLDEN[key]
    assert got.shape == want.shape, key
    if want.dtype.kind in "iu":
        assert np.array_equal(got, want), key
        return
    scale = max(float(np.abs(want).max()), 1e-30)
    assert float(np.abs(got.astype(np.float64) - want).max()) / scale <= 1e-6, key


def test_demo_loss_is_a_cross_entropy_over_32_tokens():
    """The demo's initial loss is near ln(vocab) (a nearly uniform head)."""
    assert abs(float(GOLDEN["demo_loss"]) - np.log(32.0)) < 0.5
