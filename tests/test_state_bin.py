"""state.bin record streams and numbered checkpoint directories on CPU: the
record layout of write_model_weights_bin / parse_model_weights_bin
(crates/bulletou_lib/src/value/yaneuraou_kppt.rs:110-352 and its tests
:655-720), the cuda-cpp state writers (examples/bulletou.rs:25634-25968 and
the test at :35841-35930), the exact 16-bit-limb counters and RevivalRng
(crates/cuda_cpp/src/revival_rng.rs tests), and the checkpoint directory
rules (bulletou.rs:21071-21125, 28100-28170)."""
import struct

import numpy as np
import pytest

from bulletou_b200 import state_bin as sb
from bulletou_b200._lib import CudaCppError


def test_parse_round_trip_minimal():
    buf = b"hello\n" + struct.pack("<Q", 2) + struct.pack("<f", 1.5) + struct.pack("<f", -2.25)
    m = sb.parse_model_weights_bin(buf)
    assert list(m) == ["hello"] and m["hello"].tolist() == [1.5, -2.25]


def test_select_and_rename_records():
    buf = sb.model_weights_bin_bytes([("nnue/weights/l0w", [1.0, 2.0]), ("nnue/momentum/l0w", [3.0, 4.0]),
                                      ("nnue/velocity/l0w", [5.0, 6.0])])
    m = sb.parse_model_weights_bin(buf, lambda i: i[len("nnue/weights/"):] if i.startswith("nnue/weights/") else None)
    assert list(m) == ["l0w"] and m["l0w"].tolist() == [1.0, 2.0]


def test_stream_bytes_and_empty_record(tmp_path):
    recs = [("nnue/weights/l0w", np.array([1.0, -2.5, 3.25], np.float32)), ("nnue/weights/l0b", np.zeros(0)),
            ("nnue/step_ranger/l0w", [1234.0])]
    b = sb.model_weights_bin_bytes(recs)
    assert b[:17] == b"nnue/weights/l0w\n" and struct.unpack("<Q", b[17:25])[0] == 3
    assert len(b) == sum(len(i) + 1 + 8 + 4 * np.asarray(v).size for i, v in recs)
    p = tmp_path / "s.bin"
    p.write_bytes(b)
    m = sb.parse_model_weights_bin(p)
    assert m["nnue/weights/l0w"].tolist() == [1.0, -2.5, 3.25] and m["nnue/weights/l0b"].size == 0
    assert m["nnue/step_ranger/l0w"].tolist() == [1234.0]


def test_later_record_replaces_earlier():
    m = sb.parse_model_weights_bin(sb.model_weights_bin_bytes([("a", [1.0]), ("a", [2.0, 3.0])]))
    assert m["a"].tolist() == [2.0, 3.0]


@pytest.mark.parametrize("cut,msg", [(3, "EOF inside id"), (10, "EOF inside length"), (19, "EOF inside values")])
def test_truncated_streams_fail(cut, msg):
    b = sb.model_weights_bin_bytes([("abcdef", [1.0, 2.0])])
    with pytest.raises(CudaCppError, match=msg):
        sb.parse_model_weights_bin(b[:cut])


def test_state_backend_marker_and_sections(tmp_path):
    p = tmp_path / "state.bin"
    sb.write_state_bin_atomic(p, [("nnue/weights/l0w", [1.0, 2.0]), ("nnue/weights/l0b", [3.0])], "cuda-oxide")
    raw = p.read_bytes()
    assert raw.startswith(b"meta/state_backend/cuda-oxide\n" + struct.pack("<Q", 1) + struct.pack("<f", 1.0))
    m = sb.parse_model_weights_bin(raw)
    assert sb.detect_state_backend(m) == "cuda-oxide"
    w = sb.extract_component_section(m, "nnue", "weights")
    assert sorted(w) == ["l0b", "l0w"] and w["l0w"].tolist() == [1.0, 2.0]
    assert not (tmp_path / "state.bin.tmp").exists()


def test_exact_step_limbs():
    for v in (0, 1, 1234, 65535, 65536, (1 << 40) + 5, (1 << 64) - 1):
        enc = sb.encode_exact_step(v)
        assert enc.dtype == np.float32 and sb.decode_exact_step("x", enc) == v
    assert sb.encode_exact_step(1234).tolist() == [1234.0, 0.0, 0.0, 0.0]
    for bad in ([], [0.0] * 3, [1.5, 0, 0, 0], [65536.0, 0, 0, 0], [np.nan] * 4, [-1.0] * 4):
        with pytest.raises(CudaCppError):
            sb.decode_exact_step("x", bad)


def _xorshift(state, n):
    out = []
    for _ in range(n):
        state ^= (state << 13) % (1 << 64)
        state ^= state >> 7
        state ^= (state << 17) % (1 << 64)
        out.append(float(np.float32(2.0 * ((state >> 40) / 16777216.0) - 1.0)))
    return out


def test_revival_rng_serialisation():
    """revival_rng_continues_exactly_after_serialization and
    revival_rng_validates_lossless_limbs."""
    rng = sb.RevivalRng()
    first = [rng.signed_uniform() for _ in range(64)]
    assert first == _xorshift(0x9E3779B97F4A7C15, 64)
    restored = sb.RevivalRng.decode(rng.encode())
    second = [rng.signed_uniform() for _ in range(64)]
    assert first != second and second == [restored.signed_uniform() for _ in range(64)]
    big = sb.RevivalRng((1 << 64) - 1)
    assert sb.RevivalRng.decode(big.encode()) == big
    for bad in ([], [0.0] * 4, [1.5] * 4, [65536.0] * 4, [np.nan] * 4, [-1.0] * 4):
        with pytest.raises(CudaCppError):
            sb.RevivalRng.decode(bad)


def _group(base):
    return {"momentum": np.array([base], np.float32), "velocity": np.array([base + 0.25], np.float32),
            "slow_params": np.array([base + 0.5], np.float32)}


def _sfnn_state():
    names = ["l0w", "l0b", "l1w", "l1b", "l1fw", "l1fb", "l2w", "l2b", "l2fw", "l2fb", "l3w", "l3b", "l3fw", "l3fb"]
    weights = {n: np.array([10.0 + k], np.float32) for k, n in enumerate(names)}
    opt_base = {"l0w": 1, "l0b": 2, "l1w": 3, "l1b": 4, "l1fw": 5, "l1fb": 6, "l2w": 7, "l2b": 8, "l2fw": 9,
                "l2fb": 10, "l3w": 11, "l3b": 12, "l3fw": 13, "l3fb": 14}
    rng = sb.RevivalRng()
    for _ in range(137):
        rng.signed_uniform()
    return sb.SfnnTrainState(weights, {n: _group(float(b)) for n, b in opt_base.items()}, 1234, 11, (0.5, 0.75),
                             (), True, 3, 3, rng)


def test_sfnn_state_records_full_ranger_state(tmp_path):
    """cuda_cpp_sfnn_weights_bin_writes_full_ranger_state, on the records this
    backend writes (no axis factorizers, batch norm or progress records)."""
    st = _sfnn_state()
    p = tmp_path / "state.bin"
    sb.write_state_bin_atomic(p, sb.sfnn_state_records(st))
    r = sb.parse_model_weights_bin(p)
    assert sb.detect_state_backend(r) == "cuda-cpp"
    assert r["nnue/train/optimizer_kind"].tolist() == [1.0]
    assert r["nnue/train/shared_coefficients"].tolist() == [0.5, 0.75]
    assert sb.decode_exact_step("c", r["nnue/train/completed_steps_u16"]) == 1234
    assert sb.decode_exact_step("o", r["nnue/train/optimizer_steps_u16"]) == 11
    assert r["nnue/train/axis_coefficients"].size == 0
    assert r["nnue/weights/l1_revival_flags"].tolist() == [3.0] and r["nnue/weights/l2_revival_flags"].tolist() == [3.0]
    assert sb.RevivalRng.decode(r["nnue/weights/revival_rng"]) == st.revival_rng
    assert r["nnue/weights/l1fw"].tolist() == [14.0] and r["nnue/weights/l2fw"].tolist() == [18.0]
    assert r["nnue/weights/l3fb"].tolist() == [23.0]
    assert r["nnue/momentum/l1fw"].tolist() == [5.0] and r["nnue/velocity/l3b"].tolist() == [12.25]
    assert r["nnue/slow/l2w"].tolist() == [7.5] and r["nnue/momentum/l3fw"].tolist() == [13.0]
    assert r["nnue/train/completed_steps"].tolist() == [1234.0]
    for n in ("l0w", "l1fb", "l2fb", "l3fw"):
        assert r[f"nnue/step_ranger/{n}"].tolist() == [11.0]
    # record order of the reference writer
    ids = list(r)
    assert ids[:6] == ["meta/state_backend/cuda-cpp", "nnue/train/optimizer_kind", "nnue/train/completed_steps",
                       "nnue/train/completed_steps_u16", "nnue/train/optimizer_steps_u16",
                       "nnue/train/shared_coefficients"]
    mom = [i[len("nnue/momentum/"):] for i in ids if i.startswith("nnue/momentum/")]
    assert mom == ["l0w", "l0b", "l1w", "l1b", "l1fw", "l1fb", "l2w", "l2b", "l2fw", "l2fb", "l3w", "l3b", "l3fw", "l3fb"]


def test_sfnn_state_load_round_trip_and_errors(tmp_path):
    st = _sfnn_state()
    recs = sb.parse_model_weights_bin(sb.model_weights_bin_bytes(sb.sfnn_state_records(st)))
    sizes = {n: 1 for n in st.weights}
    got = sb.load_sfnn_state(recs, sizes)
    assert (got.completed_steps, got.optimizer_steps, got.shared_coefficients, got.sgd) == (1234, 11, (0.5, 0.75), True)
    assert got.revival_rng == st.revival_rng and (got.l1_revival_flags, got.l2_revival_flags) == (3, 3)
    for n in st.weights:
        assert got.weights[n].tolist() == st.weights[n].tolist()
        for k in ("momentum", "velocity", "slow_params"):
            assert got.optimizer[n][k].tolist() == st.optimizer[n][k].tolist()
    # wrong length
    with pytest.raises(CudaCppError, match="has 1 values, expected 2"):
        sb.load_sfnn_state(recs, dict(sizes, l2w=2))
    # partial optimizer state
    part = {k: v for k, v in recs.items() if not k.startswith("nnue/slow/")}
    with pytest.raises(CudaCppError, match="optimizer state is partial"):
        sb.load_sfnn_state(part, sizes)
    # factorizer moments absent: zero moments, slow = the weights (load_or_zero)
    nof = {k: v for k, v in recs.items() if not (k.endswith("/l2fw") and "/weights/" not in k)}
    got = sb.load_sfnn_state(nof, sizes)
    assert got.optimizer["l2fw"]["momentum"].tolist() == [0.0] and got.optimizer["l2fw"]["slow_params"].tolist() == [18.0]
    # a core tensor missing its moments is an error
    nocore = {k: v for k, v in recs.items() if k != "nnue/velocity/l1w"}
    with pytest.raises(CudaCppError, match="missing nnue/velocity/l1w"):
        sb.load_sfnn_state(nocore, sizes)
    # half a factorizer pair
    half = {k: v for k, v in recs.items() if k != "nnue/weights/l1fb"}
    with pytest.raises(CudaCppError, match="partial l1f"):
        sb.load_sfnn_state(half, sizes)
    # older files: counters from the step records
    old = {k: v for k, v in recs.items() if not k.startswith("nnue/train/")}
    got = sb.load_sfnn_state(old, sizes)
    assert (got.completed_steps, got.optimizer_steps) == (11, 11)


def test_halfkp_state_records_and_load():
    names = sb.HALFKP_NAMES
    w = {n: np.arange(k + 1, dtype=np.float32) for k, n in enumerate(names)}
    opt = {n: {"momentum": w[n] + 1, "velocity": w[n] + 2, "slow_params": w[n] + 3} for n in names}
    recs = sb.halfkp_state_records(w, opt, 77)
    ids = [i for i, _ in recs]
    assert ids[:8] == [f"nnue/weights/{n}" for n in names]
    assert ids[8:11] == ["nnue/momentum/l0w", "nnue/velocity/l0w", "nnue/slow/l0w"]
    assert ids[-8:] == [f"nnue/step_ranger/{n}" for n in names]
    parsed = sb.parse_model_weights_bin(sb.model_weights_bin_bytes(recs))
    gw, gopt, done = sb.load_halfkp_state(parsed, {n: w[n].size for n in names})
    assert done == 77
    for n in names:
        np.testing.assert_array_equal(gw[n], w[n])
        np.testing.assert_array_equal(gopt[n]["slow_params"], opt[n]["slow_params"])


def test_checkpoint_dir_names():
    assert sb.checkpoint_dir_name(3, 12) == "0003-0012sb"
    assert sb.parse_checkpoint_dir_name("0003-0012sb") == (3, 12)
    assert sb.parse_checkpoint_dir_name("12345-00001sb") == (12345, 1)
    for bad in ("003-0012sb", "0003-012sb", "0003_0012sb", "0003-0012", "000a-0012sb"):
        assert sb.parse_checkpoint_dir_name(bad) is None


def _log(epoch, sbn, **kw):
    return sb.CheckpointLog(epoch, sbn, curr_batch=5, positions=1000, lr_start=0.001, lr_end=0.0005, lambda_=1.0, **kw)


def test_checkpoint_dir_write_latest_and_refusals(tmp_path):
    def payload(d):
        (d / "nn.bin").write_bytes(b"n")
        (d / "state.bin").write_bytes(b"s")

    a = sb.write_checkpoint_dir(tmp_path, _log(1, 2, dataloader_byte_offset=4000, dataloader_plies=100), payload)
    assert a.name == "0001-0002sb" and sb.is_complete_checkpoint_dir(a)
    assert (a / "dataloader_pos.txt").read_text() == "4000,100\n"
    learn = (a / "learn.log").read_text().splitlines()
    assert learn[0] == sb.LEARN_LOG_HEADER
    assert learn[1] == "SFNN_halfkahm2-1536x15x32,1,2,5,-,-,-,-,0.001000,0.000500,1.000000,1000,-"
    b = sb.write_checkpoint_dir(tmp_path, _log(1, 10, test_accuracy=0.75, test_loss=0.0123, teacher="a,b"), payload)
    assert (b / "learn.log").read_text().splitlines()[1].endswith(",0.750000,0.012300,-,-,0.001000,0.000500,1.000000,1000,\"a,b\"")
    assert sb.latest_complete_checkpoint_dir(tmp_path) == b
    with pytest.raises(CudaCppError, match="refusing to overwrite"):
        sb.write_checkpoint_dir(tmp_path, _log(1, 2), payload)
    # an incomplete directory is archived, then replaced
    inc = tmp_path / "0002-0001sb"
    inc.mkdir()
    (inc / "nn.bin").write_bytes(b"partial")
    c = sb.write_checkpoint_dir(tmp_path, _log(2, 1), payload)
    assert sb.is_complete_checkpoint_dir(c) and any(p.name.startswith("0002-0001sb.failed-") for p in tmp_path.iterdir())
    assert sb.latest_complete_checkpoint_dir(tmp_path) == c
    # a payload that fails leaves no directory behind
    def broken(d):
        (d / "nn.bin").write_bytes(b"n")
        raise OSError("disk full")

    with pytest.raises(OSError):
        sb.write_checkpoint_dir(tmp_path, _log(3, 1), broken)
    assert not any(p.name.startswith("0003-0001sb") for p in tmp_path.iterdir())
    # legacy numbered dirs rank by their learn.log position
    leg = tmp_path / "0007"
    leg.mkdir()
    for f in ("state.bin", "dataloader_pos.txt"):
        (leg / f).write_text("x")
    (leg / "learn.log").write_text(sb.LEARN_LOG_HEADER + "\nx,2,5,0\nx,1,9,0\n")
    assert sb.latest_complete_checkpoint_dir(tmp_path) == leg
