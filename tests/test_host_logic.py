"""CPU: host-side logic of the Python mirror of the reference crate
(crates/cuda_cpp/src/lib.rs): RAdam step scale, Ranger parameter validation,
loss-kind mapping, synthetic data properties."""
import numpy as np
import pytest

from bulletou_b200 import CudaCppError, RAdamUpdateParams, RangerUpdateParams, ScalarLossKind, synthetic
from oracle import oracle


@pytest.mark.parametrize("step", [1, 2, 3, 4, 5, 6, 7, 8, 12, 50, 100, 1000, 100000])
def test_step_scale_matches_oracle_bitwise(step):
    a = RAdamUpdateParams(step=step).step_scale()
    ss, ud = oracle.radam_step_scale(step)
    assert a.use_denom == ud
    assert np.float32(a.step_size).tobytes() == np.float32(ss).tobytes()


def test_step_scale_reference_points():
    s1 = RAdamUpdateParams(step=1).step_scale()
    assert not s1.use_denom and abs(s1.step_size - 10.0) < 1e-5
    s6 = RAdamUpdateParams(step=6).step_scale()
    assert np.isfinite(s6.step_size) and s6.step_size > 0


@pytest.mark.parametrize("kwargs,msg", [
    ({"step": 0}, "step must be greater than zero"),
    ({"beta1": 1.0}, "beta1"),
    ({"beta2": -0.1}, "beta2"),
    ({"epsilon": 0.0}, "epsilon"),
    ({"learning_rate": -1.0}, "learning_rate"),
    ({"min_weight": 1.0, "max_weight": -1.0}, "clamp range"),
])
def test_radam_validation_errors(kwargs, msg):
    with pytest.raises(CudaCppError, match=msg):
        RAdamUpdateParams(**kwargs).validate()


def test_ranger_validation_and_lookahead_schedule():
    with pytest.raises(CudaCppError, match="lookahead_alpha"):
        RangerUpdateParams(lookahead_alpha=1.5).validate()
    with pytest.raises(CudaCppError, match="lookahead_period"):
        RangerUpdateParams(lookahead_period=0).validate()
    with pytest.raises(CudaCppError, match="SGD momentum"):
        RangerUpdateParams(sgd_momentum=1.0).validate()
    sched = [RangerUpdateParams(radam=RAdamUpdateParams(step=s)).should_lookahead() for s in range(1, 13)]
    assert sched == [s % 6 == 0 for s in range(1, 13)]


def test_ranger_ffi_step_carries_scale():
    p = RangerUpdateParams(radam=RAdamUpdateParams(step=6, learning_rate=0.01, min_weight=-1.98, max_weight=1.98))
    s = p.ffi_step()
    sc = p.radam.step_scale()
    assert s.step_size == pytest.approx(sc.step_size) and s.use_denom == int(sc.use_denom)
    assert s.do_lookahead == 1 and s.clip_after_lookahead == 1
    assert s.min_weight == pytest.approx(-1.98)


def test_norm_loss_rate_zero_by_default():
    assert RangerUpdateParams().norm_loss_rate() == 0.0
    r = RangerUpdateParams(norm_loss_strength=0.1, norm_loss_before=True,
                           radam=RAdamUpdateParams(learning_rate=0.01)).norm_loss_rate()
    assert r == pytest.approx(2 * 0.1 * 0.01)


def test_loss_kind_ffi_mapping():
    assert ScalarLossKind.SigmoidPow(2.0).as_ffi() == 0
    assert ScalarLossKind.WinRateModel(2.5, 0.3).as_ffi() == 1
    assert ScalarLossKind.WinRateModel(2.5, 0.3).loss_param() == 0.3
    assert ScalarLossKind.BceWithLogits().as_ffi() == 2
    assert ScalarLossKind.BceWithLogits().loss_pow_exp() == 2.0
    assert ScalarLossKind.BceErrorWeighted(1.5).loss_param() == 1.5


def test_synthetic_halfkp_properties():
    b = synthetic.halfkp_batch(7, 300)
    stm, nstm = b["stm"].reshape(300, 38), b["nstm"].reshape(300, 38)
    for v in (stm, nstm):
        assert v.min() >= 0 and v.max() < synthetic.HALFKP_INPUTS
        kings = v // synthetic.HALFKP_PIECES
        assert np.all(kings == kings[:, :1])  # one king per perspective
        assert all(len(set(row)) == 38 for row in v)  # distinct pieces
    assert np.all((b["targets"] >= 0) & (b["targets"] <= 1))
    again = synthetic.halfkp_batch(7, 300)
    assert np.array_equal(again["stm"], b["stm"])  # seeded
    other = synthetic.halfkp_batch(7, 300, rank=1)
    assert not np.array_equal(other["stm"], b["stm"])  # one stream per rank


def test_synthetic_kpp_pairs():
    rng = synthetic.rng_for(1)
    stm, nstm, n, a = synthetic.kppt_indices(rng, 4, "kpp")
    assert a == 703 and n == 81 * 1548 * 1548
    v = stm.reshape(4, 703).astype(np.int64)
    rest = v % (1548 * 1548)
    lo, hi = rest // 1548, rest % 1548
    assert np.all(lo < hi)
    assert all(len(set(r)) == 703 for r in v)
    assert v.max() < n


def _round_to_f32(x):
    """Nearest float32 (ties to even) of a rational, exactly."""
    import math
    from fractions import Fraction

    if x == 0:
        return 0.0
    a = abs(x)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    ulp = Fraction(2) ** (e - 23)
    m = a / ulp
    fl = math.floor(m)
    r = m - fl
    if r > Fraction(1, 2) or (r == Fraction(1, 2) and fl % 2 == 1):
        fl += 1
    return float(fl * ulp) * (1 if x > 0 else -1)


def test_div127_two_term_reciprocal_is_the_ieee_quotient():
    """sfnn.cu's div127: fma(q, rh, RN(q * rl)) equals RN(q / 127) for every
    q of the i16 range (the QAT fake-quantisation's clamp range)."""
    from fractions import Fraction
    from pathlib import Path

    src = (Path(__file__).resolve().parents[1] / "bulletou_b200" / "csrc" / "sfnn.cu").read_text()
    assert "__fmaf_rn(q, 0x1.020408p-7f, __fmul_rn(q, 0x1.020408p-35f))" in src
    rh, rl = float.fromhex("0x1.020408p-7"), float.fromhex("0x1.020408p-35")
    assert np.float32(rh) == rh and np.float32(rl) == rl
    assert rh == _round_to_f32(Fraction(1, 127)) and rl == _round_to_f32(Fraction(1, 127) - Fraction(rh))
    for q in range(-32768, 32768):
        t = float(np.float32(q) * np.float32(rl))  # the f32 product, correctly rounded
        got = _round_to_f32(Fraction(q) * Fraction(rh) + Fraction(t))
        assert got == _round_to_f32(Fraction(q, 127)), q
