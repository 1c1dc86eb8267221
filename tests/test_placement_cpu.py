"""Expert placement for expert parallelism (host-only parts, no GPU):
hf_ep_balanced_placement and the argument checks of hf_moe_set_placement."""
import ctypes

import numpy as np
import pytest

from hummingflight_b200 import _lib
from hummingflight_b200.moe import HfError, balanced_placement


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_balanced_placement_is_an_even_permutation(world):
    rng = np.random.default_rng(world)
    load = rng.zipf(1.3, 256).clip(max=5000) + 128
    order = balanced_placement(load, world)
    assert sorted(order.tolist()) == list(range(256))
    per = order.reshape(world, -1)
    assert all(np.all(np.diff(r) > 0) for r in per)  # ascending ids inside a rank
    sums = np.array([load[r].sum() for r in per])
    # greedy longest-first: no rank above the mean by more than the largest load
    assert sums.max() - sums.mean() <= load.max()


def test_balanced_placement_beats_contiguous_ranges():
    rng = np.random.default_rng(7)
    load = np.zeros(256, np.int64)
    load[:32] = 2000            # the hot experts all in rank 0's contiguous range
    load[32:] = rng.integers(0, 400, 224)
    contiguous = load.reshape(8, -1).sum(1)
    placed = np.array([load[r].sum() for r in balanced_placement(load, 8).reshape(8, -1)])
    assert placed.max() / placed.mean() < 1.05 < contiguous.max() / contiguous.mean()


def test_balanced_placement_rejects_bad_arguments():
    with pytest.raises(HfError):
        balanced_placement(np.ones(10, np.int64), 4)   # 10 experts over 4 ranks


def test_set_placement_checks_the_permutation_before_any_device_call():
    L = _lib.lib()
    # a null context is an argument error, whatever the order
    order = (ctypes.c_int32 * 4)(0, 1, 2, 3)
    assert L.hf_moe_set_placement(None, 0, order) == _lib.HF_ERR_ARG
