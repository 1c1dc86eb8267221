"""Workload definitions (CPU): the Zipf target shape and config 4's calibration."""
import numpy as np

from hummingflight_b200.configs import (WORKLOADS, ZIPF_BETA, zipf_bias, zipf_ranks,
                                        zipf_stats, zipf_target_shares)


def test_zipf_target_shape_is_capped_and_normalised():
    t = zipf_target_shares(256, 8)
    assert abs(t.sum() - 1.0) < 1e-9
    assert t.max() <= 1 / 8 + 1e-12
    assert np.all(np.diff(t) <= 0)
    # below the cap the shares fall as r^-1.1
    r = np.arange(1, 257)
    free = t < 1 / 8 - 1e-9
    ratio = t[free] * r[free] ** 1.1
    assert np.allclose(ratio, ratio[0])


def test_zipf_bias_follows_the_ranking():
    b = zipf_bias(256, 20)
    ranks = zipf_ranks(256, 20)
    assert b[ranks == 1][0] == 0.0
    assert np.all(np.diff(b[np.argsort(ranks)]) < 0)


def test_config4_beta_is_the_calibrated_value():
    import zipf_calibration as Z
    beta, st = Z.calibrate(WORKLOADS[4], iters=16)
    assert abs(beta - ZIPF_BETA) < 2e-3, beta
    assert abs(st["top_decile_share"] - st["target_top_decile_share"]) < 0.01
    assert st["hottest_share"] <= 1 / 8
    assert st["zero_experts"] > 0


def test_zipf_stats_on_a_perfect_shape():
    t = zipf_target_shares(256, 8)
    ranks = zipf_ranks(256, 3)
    counts = np.round(t[ranks - 1] * 1e7)
    st = zipf_stats(counts, 3, 8)
    assert st["l1_to_target"] < 1e-5
    assert st["zero_experts"] == 0
