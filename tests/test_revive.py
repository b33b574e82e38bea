"""FT unit revival (crates/cuda_cpp/src/ft_revive.rs): the host-side selection
and calibration on CPU (the reference's tests saturation_is_per_unit_and_
includes_threshold and unobserved_bucket_mean_uses_global_mean), and the
device-state edits on the GPU (gpu_reset_and_mean_compensation_preserve_other_
columns, revive_one_saturated_unit_preserves_partner, gpu_shared_and_virtual_
columns), with the random rows checked against the revival stream."""
import numpy as np
import pytest

from bulletou_b200 import revive as rv
from bulletou_b200._lib import CudaCppError
from bulletou_b200.state_bin import RevivalRng


def test_saturation_is_per_unit_and_includes_threshold():
    assert rv.saturated_units([99, 100, 98, 0], 100, 0.99) == [0, 1]
    with pytest.raises(CudaCppError):
        rv.saturated_units([0], 0, 0.99)
    with pytest.raises(CudaCppError):
        rv.saturated_units([101], 100, 0.99)
    with pytest.raises(CudaCppError):
        rv.saturated_units([1], 100, 0.0)


def test_unobserved_bucket_mean_uses_global_mean():
    c = rv.FtCalibration(2, 2)
    c.add([0, 0], [0.2, 0.4, 0.6, 0.8], [1.0, 1.0])
    c.finish_means()
    assert abs(c.means[2] - 0.4) < 1e-6 and abs(c.means[3] - 0.6) < 1e-6
    assert abs(c.means[0] - 0.4) < 1e-6 and c.counts.tolist() == [2, 0]


def test_calibration_mask_and_errors():
    c = rv.FtCalibration(2, 3)
    c.add([1, 2, 1], [1, 2, 3, 4, 5, 6], [1.0, 0.0, 2.0])
    c.finish_means()
    assert c.counts.tolist() == [0, 2, 0]
    assert c.means[2:4].tolist() == [3.0, 4.0]
    for args in (([0], [1.0, np.nan], [1.0]), ([3], [1.0, 2.0], [1.0]), ([0], [1.0, 2.0], [-1.0]),
                 ([0], [1.0], [1.0])):
        with pytest.raises(CudaCppError):
            rv.FtCalibration(2, 3).add(*args)


def test_revival_draws_are_the_xorshift_stream():
    """The FT row values: round(u * bound * 127) / 127 in f32 with u the
    stream's signed uniforms (revive_ft_units, ft_revive.rs:78-83)."""
    r = RevivalRng()
    u = r.signed_uniform_array(5)
    s = RevivalRng()
    assert u.tolist() == [s.signed_uniform() for _ in range(5)]
    bound = max(np.float32(np.sqrt(np.float32(6.0) / np.float32(100 + 12))), np.float32(1 / 127))
    v = rv._round_half_away(u * bound * np.float32(127.0)) / np.float32(127.0)
    assert np.all(np.abs(v) <= bound + 1 / 127) and v.dtype == np.float32
    assert rv._round_half_away(np.array([0.5, -0.5, 1.5, -2.5, 0.49999997], np.float32)).tolist() == [1, -1, 2, -3, 0]


# ------------------------------------------------------------------ L1 revival statistics
def test_contribution_mad_normalization_and_strict_boundary():
    c = rv.Contribution(4, 2)
    for i in range(1024):
        c.add(0, [1.0, float(i % 2), 0.0, float(i % 2)])
        c.add(1, [0.0, 1.0, 0.0, 1.0])
    c.finish([1.0] * 8, 1, 2, 0.01)
    assert c.utility.tolist() == [0.0, 1.0, 0.0, 0.0]
    assert c.relative.tolist() == [0.0, 1.0, 0.0, 0.0]
    assert c.selected([1024, 1024], 2) == [0, 2, 3]
    assert c.selected([1024, 1023], 2) == [0]
    c.relative = np.array([0.009999, 0.01, 0.010001, 0.0])
    assert c.selected([1024, 1024], 2) == [0, 3]


def test_contribution_uses_outgoing_weights_and_rejects_invalid_values():
    c = rv.Contribution(3, 1)
    c.add(0, [0.0, 0.0, 0.25])
    c.add(0, [1.0, 1.0, 0.75])
    c.finish([0.0, -2.0, 1.0], 1, 1, 0.01)
    assert c.utility.tolist() == [0.0, 1.0, 0.25]
    assert c.means.tolist() == [0.5] * 3
    for bad in (0.0, -0.1, 1.01, float("nan"), float("inf")):
        with pytest.raises(CudaCppError):
            rv.Contribution(1, 1).finish([1.0], 1, 1, bad)


def test_configurable_thresholds_and_zero_classification():
    c = rv.L1Calibration(1, 4, 1)
    c.counts[0] = 10000
    c.upper[:] = [9900, 9899, 0, 0]
    c.lower[:] = [0, 0, 9900, 9899]
    assert c.candidates_for(True, True) == [0, 2]
    assert not c.is_upper(2, True)
    assert c.candidates_for(False, False) == []
    c.set_thresholds(1.0, 1.0)
    assert c.candidates_for(True, True) == []
    c.set_thresholds(0.98, 0.995)
    assert c.candidates_for(True, True) == [0, 1]
    for bad in (0.0, -0.1, 1.01, float("nan"), float("inf")):
        with pytest.raises(CudaCppError):
            c.set_thresholds(bad, 0.99)
        with pytest.raises(CudaCppError):
            c.set_thresholds(0.99, bad)
    c.set_thresholds(0.99, 0.99)
    c.counts[0] = 5331
    c.upper[0], c.upper[1] = 5323, 0
    c.lower[:] = 0
    assert c.candidates_for(True, False) == [0]


def test_l1_calibration_statistics():
    c = rv.L1Calibration(2, 2, 2)
    x = np.array([[1, 2], [3, 4], [5, 6]], np.float32)
    y = np.array([[1, 0, 1, 0], [0, 0, 0, 0], [2, 0.5, 3, 0]], np.float32)
    c.add([0, 1, 0], x, y, [1.0, 1.0, 0.0])
    assert c.counts.tolist() == [1, 1]
    assert c.sums.tolist() == [1, 2, 3, 4]
    assert c.branch_sums[:4].tolist() == [1, 0, 1, 0]
    assert c.upper.tolist() == [1, 0, 0, 0] and c.lower.tolist() == [0, 1, 1, 1]
    with pytest.raises(CudaCppError):
        c.add([2], x[:1], y[:1])


def test_l2_calibration_thresholds_and_statistics():
    c = rv.L2Calibration(1, 4, 1)
    c.counts[0] = 10000
    c.upper[:] = [9900, 9899, 0, 0]
    c.lower[:] = [0, 0, 9900, 9899]
    assert c.candidates_for(True, True) == [0, 2] and c.candidates() == [0]
    c.set_thresholds(0.98, 0.995)
    assert c.candidates_for(True, True) == [0, 1]
    d = rv.L2Calibration(2, 2, 2)
    d.add([1, 1, 0], [[1, 2], [3, 4], [5, 6]], [[1.0, 0.0], [0.5, 0.0], [2.0, -1.0]], [1.0, 1.0, 0.0])
    assert d.counts.tolist() == [0, 2] and d.sums.tolist() == [0, 0, 1.5, 0]
    assert d.upper.tolist() == [0, 0, 1, 0] and d.lower.tolist() == [0, 0, 0, 2]
    assert len(d.inputs[1]) == 2 and d.inputs[1][1].tolist() == [3, 4]
    with pytest.raises(CudaCppError):
        d.add([0], [1, 2], [1.0])
