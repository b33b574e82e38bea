"""Training state on disk: ``state.bin`` record streams and numbered checkpoint
directories, so a run can be resumed from the reference's checkpoints and the
reference can resume from ours.

Record stream (crates/bulletou_lib/src/value/yaneuraou_kppt.rs): each record is
the id in ASCII, ``\\n``, the value count as a little-endian u64, then that many
little-endian f32 (write_model_weights_bin_writer :294-320, parse :110-225;
a later record with the same id replaces the earlier one).  The cuda-cpp
backend opens its files with the ``meta/state_backend/cuda-cpp`` = [1.0]
marker (write_cuda_cpp_state_records_atomic, examples/bulletou.rs:27476-27510)
and writes the weights, then per parameter the Ranger momentum / velocity /
slow records, then the step records, in the order of
write_cuda_cpp_halfkp_weights_bin (bulletou.rs:25634-25683) and
write_cuda_cpp_sfnn_weights_bin (bulletou.rs:25745-25968).  Counters that must
survive f32 are four exact 16-bit limbs (encode_sfnn_exact_step,
bulletou.rs:24983-24996; RevivalRng, crates/cuda_cpp/src/revival_rng.rs).

Checkpoint directories (bulletou.rs:21009-21125, 28100-28170) are named
``EEEE-SSSSsb``, written into ``<name>.tmp-<pid>-<n>`` and renamed into place;
a directory is complete when it holds ``state.bin``, ``learn.log`` and
``dataloader_pos.txt``.
"""
from __future__ import annotations

import io
import os
import struct
import time
from dataclasses import dataclass
from pathlib import Path
from typing import BinaryIO, Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from ._lib import CudaCppError

STATE_BACKEND_RECORD_PREFIX = "meta/state_backend/"
STATE_BACKEND_MARKER_VALUE = 1.0
STATE_BACKEND = "cuda-cpp"
LEARN_LOG_HEADER = ("eval,epoch,superbatch,curr_batch,test_value_accuracy,test_value_loss,quantized_value_accuracy,"
                    "quantized_value_loss,lr_start,lr_end,lambda,positions,teacher")
_CHUNK_VALUES = 1 << 20

Record = Tuple[str, np.ndarray]


# ------------------------------------------------------------------ record stream
def write_records(f: BinaryIO, records: Iterable[Record]) -> None:
    for rid, values in records:
        v = np.ascontiguousarray(values, dtype="<f4").reshape(-1)
        f.write(rid.encode("ascii") + b"\n" + struct.pack("<Q", v.size))
        for start in range(0, v.size, _CHUNK_VALUES):
            f.write(v[start:start + _CHUNK_VALUES].tobytes())


def model_weights_bin_bytes(records: Iterable[Record]) -> bytes:
    buf = io.BytesIO()
    write_records(buf, records)
    return buf.getvalue()


def parse_model_weights_bin(data, select: Optional[Callable[[str], Optional[str]]] = None) -> Dict[str, np.ndarray]:
    """Records of a byte stream (bytes, or a path).  ``select`` maps an id to
    the key to store it under, or None to skip it, as
    parse_model_weights_bin_reader_select_map does."""
    if isinstance(data, (str, os.PathLike)):
        data = Path(data).read_bytes()
    data = bytes(data)
    out: Dict[str, np.ndarray] = {}
    off, total = 0, len(data)
    while off < total:
        nl = data.find(b"\n", off)
        if nl < 0:
            raise CudaCppError("raw.bin: EOF inside id")
        rid = data[off:nl].decode("latin-1")
        off = nl + 1
        if off + 8 > total:
            raise CudaCppError(f"raw.bin: EOF inside length (id={rid!r}, offset={off}, total={total})")
        n = struct.unpack_from("<Q", data, off)[0]
        off += 8
        if n * 4 > total - off:
            raise CudaCppError(f"raw.bin: EOF inside values (id={rid!r}, len={n}, need={n * 4} bytes, "
                               f"have={total - off} bytes)")
        key = rid if select is None else select(rid)
        if key is not None:
            out[key] = np.frombuffer(data, "<f4", n, off).astype(np.float32)
        off += n * 4
    return out


def state_backend_record_id(backend: str) -> str:
    return STATE_BACKEND_RECORD_PREFIX + backend


def state_backend_marker(backend: str = STATE_BACKEND) -> Record:
    return state_backend_record_id(backend), np.array([STATE_BACKEND_MARKER_VALUE], np.float32)


def detect_state_backend(records: Dict[str, np.ndarray]) -> Optional[str]:
    for rid in sorted(records):
        v = records[rid]
        if rid.startswith(STATE_BACKEND_RECORD_PREFIX) and v.size == 1 and v[0] == STATE_BACKEND_MARKER_VALUE:
            name = rid[len(STATE_BACKEND_RECORD_PREFIX):]
            if name:
                return name
    return None


def extract_component_section(records: Dict[str, np.ndarray], component: str, section: str) -> Dict[str, np.ndarray]:
    prefix = f"{component}/{section}/"
    return {k[len(prefix):]: v for k, v in records.items() if k.startswith(prefix)}


def write_state_bin_atomic(path, records: Iterable[Record], backend: str = STATE_BACKEND) -> None:
    """Marker first, then the records, into ``<name>.tmp`` renamed over ``path``."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    try:
        with open(tmp, "wb", buffering=8 << 20) as f:
            write_records(f, [state_backend_marker(backend)])
            write_records(f, records)
        os.replace(tmp, path)
    except BaseException:
        tmp.unlink(missing_ok=True)
        raise


# ------------------------------------------------------------------ exact counters
def encode_exact_step(value: int) -> np.ndarray:
    return np.array([(int(value) >> (16 * i)) & 0xFFFF for i in range(4)], np.float32)


def decode_exact_step(label: str, values) -> int:
    v = np.asarray(values, np.float32)
    if v.size != 4 or not np.all(np.isfinite(v)) or np.any(v < 0) or np.any(v > 65535) or np.any(v != np.floor(v)):
        raise CudaCppError(f"invalid SFNN exact step record {label}")
    return sum(int(x) << (16 * i) for i, x in enumerate(v))


@dataclass
class RevivalRng:
    """The revival xorshift stream (revival_rng.rs): state persisted as four
    16-bit limbs; the zero state is rejected."""

    state: int = 0x9E3779B97F4A7C15

    def signed_uniform(self) -> float:
        s = self.state
        s ^= (s << 13) & 0xFFFFFFFFFFFFFFFF
        s ^= s >> 7
        s ^= (s << 17) & 0xFFFFFFFFFFFFFFFF
        self.state = s
        return float(np.float32(2.0) * (np.float32(s >> 40) / np.float32(16777216.0)) - np.float32(1.0))

    def signed_uniform_array(self, n: int) -> np.ndarray:
        """n consecutive draws (the same values as n calls of signed_uniform)."""
        s, m = self.state, 0xFFFFFFFFFFFFFFFF
        top = np.empty(n, np.float32)
        for i in range(n):
            s ^= (s << 13) & m
            s ^= s >> 7
            s ^= (s << 17) & m
            top[i] = s >> 40
        self.state = s
        return np.float32(2.0) * (top / np.float32(16777216.0)) - np.float32(1.0)

    def encode(self) -> np.ndarray:
        return encode_exact_step(self.state)

    @staticmethod
    def decode(values) -> "RevivalRng":
        v = np.asarray(values, np.float32)
        if v.size != 4 or not np.all(np.isfinite(v)) or np.any(v < 0) or np.any(v > 65535) or np.any(v != np.floor(v)):
            raise CudaCppError("invalid revival RNG checkpoint state (expected four u16 limbs)")
        state = sum(int(x) << (16 * i) for i, x in enumerate(v))
        if state == 0:
            raise CudaCppError("invalid zero revival RNG checkpoint state")
        return RevivalRng(state)


# ------------------------------------------------------------------ HalfKP state
HALFKP_NAMES = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "outw", "outb")


def _group_records(names: Sequence[str], optimizer: Dict[str, dict]) -> List[Record]:
    out: List[Record] = []
    for n in names:
        st = optimizer[n]
        out += [(f"nnue/momentum/{n}", st["momentum"]), (f"nnue/velocity/{n}", st["velocity"]),
                (f"nnue/slow/{n}", st["slow_params"])]
    return out


def halfkp_state_records(weights: Dict[str, np.ndarray], optimizer: Dict[str, dict], completed_steps: int) -> List[Record]:
    """write_cuda_cpp_halfkp_weights_bin without batch-norm records."""
    steps = np.array([completed_steps], np.float32)
    recs: List[Record] = [(f"nnue/weights/{n}", weights[n]) for n in HALFKP_NAMES]
    recs += _group_records(HALFKP_NAMES, optimizer)
    recs += [(f"nnue/step_ranger/{n}", steps) for n in HALFKP_NAMES]
    return recs


# ------------------------------------------------------------------ SFNN state
SFNN_CORE = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "l3w", "l3b")
SFNN_PAIRS = (("l1fw", "l1fb"), ("l2fw", "l2fb"), ("l3fw", "l3fb"))


@dataclass
class SfnnTrainState:
    """The host side of an SFNN state.bin: weights, Ranger states and counters."""

    weights: Dict[str, np.ndarray]
    optimizer: Optional[Dict[str, dict]]
    completed_steps: int
    optimizer_steps: int
    shared_coefficients: Tuple[float, float] = (1.0, 0.0)
    axis_coefficients: Tuple[float, ...] = ()
    sgd: bool = False
    l1_revival_flags: int = 0
    l2_revival_flags: int = 0
    revival_rng: RevivalRng = None

    def __post_init__(self):
        if self.revival_rng is None:
            self.revival_rng = RevivalRng()


def _present_pairs(weights: Dict[str, Optional[np.ndarray]], what: str) -> List[str]:
    names = []
    for w, b in SFNN_PAIRS:
        has_w, has_b = weights.get(w) is not None, weights.get(b) is not None
        if has_w != has_b:
            raise CudaCppError(f"cuda-cpp SFNN {what} have partial {w[:3]} state")
        if has_w:
            names += [w, b]
    return names


def sfnn_state_records(state: SfnnTrainState) -> List[Record]:
    """write_cuda_cpp_sfnn_weights_bin (no batch norm, no progress axis, no
    bucket-axis factorizers: this backend trains none of them)."""
    w = state.weights
    pairs = _present_pairs(w, "weights")
    opt_steps = np.array([state.optimizer_steps], np.float32)
    recs: List[Record] = [
        ("nnue/train/optimizer_kind", np.array([1.0 if state.sgd else 0.0], np.float32)),
        ("nnue/train/completed_steps", np.array([state.completed_steps], np.float32)),
        ("nnue/train/completed_steps_u16", encode_exact_step(state.completed_steps)),
        ("nnue/train/optimizer_steps_u16", encode_exact_step(state.optimizer_steps)),
        ("nnue/train/shared_coefficients", np.array(state.shared_coefficients, np.float32)),
    ]
    recs += [(f"nnue/weights/{n}", w[n]) for n in SFNN_CORE]
    recs.append(("nnue/train/axis_coefficients", np.array(state.axis_coefficients, np.float32)))
    recs.append(("nnue/weights/l1_revival_flags", np.array([state.l1_revival_flags], np.float32)))
    recs.append(("nnue/weights/l2_revival_flags", np.array([state.l2_revival_flags], np.float32)))
    recs.append(("nnue/weights/revival_rng", state.revival_rng.encode()))
    recs += [(f"nnue/weights/{n}", w[n]) for n in pairs]
    if state.optimizer is None:
        raise CudaCppError("cuda-cpp SFNN state.bin needs the optimizer states")
    order = ["l0w", "l0b", "l1w", "l1b"] + [n for n in pairs if n.startswith("l1")] + ["l2w", "l2b"] + \
        [n for n in pairs if n.startswith("l2")] + ["l3w", "l3b"] + [n for n in pairs if n.startswith("l3")]
    recs += _group_records(order, state.optimizer)
    recs += [(f"nnue/step_ranger/{n}", opt_steps) for n in SFNN_CORE + tuple(pairs)]
    return recs


def _check_len(label: str, section: str, name: str, values: np.ndarray, expected: int) -> np.ndarray:
    if values.size != expected:
        raise CudaCppError(f"cuda-cpp {label} {section} record nnue/{section}/{name} has {values.size} values, "
                           f"expected {expected}")
    return values


def _optimizer_from_sections(label: str, names: Sequence[str], optional: Sequence[str], sizes: Dict[str, int],
                             records: Dict[str, np.ndarray]) -> Optional[Dict[str, dict]]:
    sec = {s: extract_component_section(records, "nnue", s) for s in ("momentum", "velocity", "slow")}
    if not any(sec.values()):
        return None
    if not all(sec.values()):
        raise CudaCppError(f"cuda-cpp {label} optimizer state is partial: expected nnue/{{momentum,velocity,slow}}/* "
                           "records")
    out = {}
    for n in list(names) + list(optional):
        if n in optional and not any(n in sec[s] for s in sec):
            continue  # load_or_zero: zero moments; slow = the loaded weights (filled by the caller)
        st = {}
        for s, key in (("momentum", "momentum"), ("velocity", "velocity"), ("slow", "slow_params")):
            if n not in sec[s]:
                raise CudaCppError(f"cuda-cpp {label} optimizer state missing nnue/{s}/{n}")
            st[key] = _check_len(label, s, n, sec[s][n], sizes[n])
        out[n] = st
    return out


def load_sfnn_state(path_or_records, sizes: Dict[str, int]) -> SfnnTrainState:
    """The state of an SFNN state.bin for a network whose tensors have the
    element counts ``sizes`` (the factorizer tensors only when present)."""
    records = path_or_records if isinstance(path_or_records, dict) else parse_model_weights_bin(path_or_records)
    w = extract_component_section(records, "nnue", "weights")
    train = extract_component_section(records, "nnue", "train")
    steps = extract_component_section(records, "nnue", "step_ranger")
    weights = {}
    for n in SFNN_CORE + tuple(x for p in SFNN_PAIRS for x in p):
        if n not in sizes:
            continue
        if n not in w:
            if n in SFNN_CORE:
                raise CudaCppError(f"cuda-cpp SFNN state missing nnue/weights/{n}")
            continue
        weights[n] = _check_len("SFNN", "weights", n, w[n], sizes[n])
    pairs = _present_pairs(weights, "weights")
    opt = _optimizer_from_sections("SFNN", SFNN_CORE, pairs, sizes, records)
    if opt is not None:
        for n in pairs:
            opt.setdefault(n, {"momentum": np.zeros(sizes[n], np.float32), "velocity": np.zeros(sizes[n], np.float32),
                               "slow_params": weights[n].copy()})
    if "optimizer_steps_u16" in train:
        optimizer_steps = decode_exact_step("optimizer_steps_u16", train["optimizer_steps_u16"])
    else:
        optimizer_steps = _single_step(steps.get("l0w"), "nnue/step_ranger/l0w") if "l0w" in steps else 0
    if "completed_steps_u16" in train:
        completed = decode_exact_step("completed_steps_u16", train["completed_steps_u16"])
    elif "completed_steps" in train:
        completed = _single_step(train["completed_steps"], "nnue/train/completed_steps")
    else:
        completed = optimizer_steps
    sc = train.get("shared_coefficients")
    rng = RevivalRng.decode(w["revival_rng"]) if "revival_rng" in w else RevivalRng()
    return SfnnTrainState(weights, opt, completed, optimizer_steps,
                          (1.0, 0.0) if sc is None else (float(sc[0]), float(sc[1])),
                          tuple(float(x) for x in train.get("axis_coefficients", ())),
                          bool(train.get("optimizer_kind", [0.0])[0] == 1.0),
                          int(w.get("l1_revival_flags", [0])[0]), int(w.get("l2_revival_flags", [0])[0]), rng)


def load_halfkp_state(path_or_records, sizes: Dict[str, int]) -> Tuple[Dict[str, np.ndarray], Optional[Dict[str, dict]], int]:
    records = path_or_records if isinstance(path_or_records, dict) else parse_model_weights_bin(path_or_records)
    w = extract_component_section(records, "nnue", "weights")
    weights = {}
    for n in HALFKP_NAMES:
        if n not in w:
            raise CudaCppError(f"cuda-cpp HalfKP state missing nnue/weights/{n}")
        weights[n] = _check_len("HalfKP", "weights", n, w[n], sizes[n])
    opt = _optimizer_from_sections("HalfKP", HALFKP_NAMES, (), sizes, records)
    steps = extract_component_section(records, "nnue", "step_ranger")
    done = _single_step(steps["l0w"], "nnue/step_ranger/l0w") if "l0w" in steps else 0
    return weights, opt, done


def _single_step(values, label: str) -> int:
    v = np.asarray(values, np.float32)
    if v.size != 1 or not np.isfinite(v[0]) or v[0] < 0 or v[0] != np.floor(v[0]):
        raise CudaCppError(f"invalid step record {label}")
    return int(v[0])


# ------------------------------------------------------------------ checkpoint dirs
def checkpoint_dir_name(epoch: int, superbatch: int) -> str:
    return f"{epoch:04d}-{superbatch:04d}sb"


def parse_checkpoint_dir_name(name: str) -> Optional[Tuple[int, int]]:
    if not name.endswith("sb") or "-" not in name:
        return None
    epoch, sb = name[:-2].split("-", 1)
    if len(epoch) < 4 or len(sb) < 4 or not (epoch.isdigit() and sb.isdigit()) or not (epoch.isascii() and sb.isascii()):
        return None
    return int(epoch), int(sb)


def is_complete_checkpoint_dir(d) -> bool:
    d = Path(d)
    return (d / "state.bin").is_file() and (d / "learn.log").is_file() and (d / "dataloader_pos.txt").is_file()


def read_checkpoint_epoch_superbatch(d) -> Optional[Tuple[int, int]]:
    """The latest (epoch, superbatch) row of a legacy numbered dir's learn.log."""
    try:
        text = (Path(d) / "learn.log").read_text()
    except OSError:
        return None
    latest = None
    for line in text.splitlines():
        line = line.strip()
        if not line or line.startswith("#") or line.startswith("eval,"):
            continue
        parts = line.split(",", 3)
        if len(parts) < 3 or not (parts[1].isdigit() and parts[2].isdigit()):
            continue
        pos = (int(parts[1]), int(parts[2]))
        latest = pos if latest is None else max(latest, pos)
    return latest


def latest_complete_checkpoint_dir(output_dir) -> Optional[Path]:
    out = Path(output_dir)
    if not out.is_dir():
        return None
    named, legacy = [], []
    for p in out.iterdir():
        if not is_complete_checkpoint_dir(p):
            continue
        pos = parse_checkpoint_dir_name(p.name)
        if pos is not None:
            named.append((pos, p))
        elif p.name.isdigit():
            legacy.append((int(p.name), p))
    cands = []
    if named:
        cands.append(max(named, key=lambda x: x[0]))
    if legacy:
        _, p = max(legacy, key=lambda x: x[0])
        pos = read_checkpoint_epoch_superbatch(p)
        if pos is not None:
            cands.append((pos, p))
    return max(cands, key=lambda x: x[0])[1] if cands else None


@dataclass
class CheckpointLog:
    """The learn.log row (cuda_cpp_direct_learn_log_row, bulletou.rs:21127-21150)
    and the data-loader position of one checkpoint."""

    epoch: int
    superbatch: int
    curr_batch: int
    positions: int
    lr_start: float
    lr_end: float
    lambda_: float
    eval_name: str = "SFNN_halfkahm2-1536x15x32"
    teacher: str = "-"
    test_accuracy: Optional[float] = None
    test_loss: Optional[float] = None
    dataloader_byte_offset: int = 0
    dataloader_plies: int = 0

    def row(self) -> str:
        acc = "-" if self.test_accuracy is None else f"{self.test_accuracy:.6f}"
        loss = "-" if self.test_loss is None else f"{self.test_loss:.6f}"
        teacher = f'"{self.teacher}"' if ("," in self.teacher or '"' in self.teacher) else self.teacher
        return (f"{self.eval_name},{self.epoch},{self.superbatch},{self.curr_batch},{acc},{loss},-,-,"
                f"{self.lr_start:.6f},{self.lr_end:.6f},{self.lambda_:.6f},{self.positions},{teacher}\n")


def _archive_incomplete(d: Path) -> None:
    ts = int(time.time())
    for attempt in range(1000):
        failed = d.with_name(f"{d.name}.failed-{ts}" + ("" if attempt == 0 else f"-{attempt}"))
        if not failed.exists():
            d.rename(failed)
            return
    raise CudaCppError(f"failed to archive incomplete checkpoint {d}")


def write_checkpoint_dir(output_dir, log: CheckpointLog, write_payload: Callable[[Path], None]) -> Path:
    """prepare / write / commit of a numbered checkpoint: an existing complete
    directory is never overwritten, an incomplete one is archived as
    ``<name>.failed-<time>``; ``write_payload(tmp)`` writes nn.bin and
    state.bin into the temporary directory before the metadata files."""
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    name = checkpoint_dir_name(log.epoch, log.superbatch)
    final = out / name
    if final.exists():
        if is_complete_checkpoint_dir(final):
            raise CudaCppError(f"refusing to overwrite existing numbered checkpoint {final}")
        _archive_incomplete(final)
    tmp = None
    for attempt in range(1000):
        cand = out / f"{name}.tmp-{os.getpid()}-{attempt}"
        if not cand.exists():
            cand.mkdir()
            tmp = cand
            break
    if tmp is None:
        raise CudaCppError(f"failed to choose temporary checkpoint directory for {final}")
    try:
        write_payload(tmp)
        (tmp / "dataloader_pos.txt").write_text(f"{log.dataloader_byte_offset},{log.dataloader_plies}\n")
        (tmp / "learn.log").write_text(LEARN_LOG_HEADER + "\n" + log.row())
        if final.exists():
            raise CudaCppError(f"refusing to overwrite existing numbered checkpoint {final}")
        tmp.rename(final)
    except BaseException:
        for p in sorted(tmp.glob("*")):
            p.unlink()
        tmp.rmdir()
        raise
    return final


# ------------------------------------------------------------------ runners
def _upload_group(ctx, st, host: dict) -> None:
    st.momentum.upload(host["momentum"], ctx)
    st.velocity.upload(host["velocity"], ctx)
    st.slow_params.upload(host["slow_params"], ctx)


def sfnn_runner_state(ctx, runner, completed_steps: int, optimizer_steps: int) -> SfnnTrainState:
    """Download an SfnnTrainStepRunner's weights and Ranger states."""
    a = runner.alpha
    rng = getattr(runner, "revival_rng", None)
    return SfnnTrainState(runner.read_weights(ctx), runner.read_optimizer_states(ctx), int(completed_steps),
                          int(optimizer_steps), (a.ft, a.shared if runner.present.get("l1fw") else 0.0),
                          l1_revival_flags=getattr(runner, "l1_revival_flags", 0),
                          l2_revival_flags=getattr(runner, "l2_revival_flags", 0),
                          revival_rng=None if rng is None else RevivalRng(rng.state))


def sfnn_runner_sizes(runner) -> Dict[str, int]:
    return {n: w.length for n, w in runner.weights.items() if w is not None}


def restore_sfnn_runner(ctx, runner, state: SfnnTrainState) -> None:
    """Upload a loaded state into the runner's device buffers; every tensor the
    runner trains must be in the state (the factorizer pairs included)."""
    for n, buf in runner.weights.items():
        if buf is None:
            continue
        if n not in state.weights:
            raise CudaCppError(f"cuda-cpp SFNN state missing nnue/weights/{n}")
        buf.upload(state.weights[n], ctx)
        st = runner.optimizer_states[n]
        if state.optimizer is None:
            st.momentum.fill(0.0, ctx)
            st.velocity.fill(0.0, ctx)
            st.slow_params.upload(state.weights[n], ctx)
        else:
            _upload_group(ctx, st, state.optimizer[n])
    runner.revival_rng = RevivalRng(state.revival_rng.state)
    runner.l1_revival_flags = state.l1_revival_flags
    runner.l2_revival_flags = state.l2_revival_flags


def write_sfnn_state_bin(path, ctx, runner, completed_steps: int, optimizer_steps: int) -> SfnnTrainState:
    state = sfnn_runner_state(ctx, runner, completed_steps, optimizer_steps)
    write_state_bin_atomic(path, sfnn_state_records(state))
    return state


def halfkp_runner_sizes(runner) -> Dict[str, int]:
    return {n: w.length for n, w in zip(HALFKP_NAMES, runner.weights)}


def write_halfkp_state_bin(path, ctx, runner, completed_steps: int) -> None:
    write_state_bin_atomic(path, halfkp_state_records(runner.read_weights(ctx), runner.read_optimizer_states(ctx),
                                                      completed_steps))


def restore_halfkp_runner(ctx, runner, weights: Dict[str, np.ndarray], optimizer: Optional[Dict[str, dict]]) -> None:
    for n, buf, st in zip(HALFKP_NAMES, runner.weights, runner.optimizer_states):
        buf.upload(weights[n], ctx)
        if optimizer is None:
            st.momentum.fill(0.0, ctx)
            st.velocity.fill(0.0, ctx)
            st.slow_params.upload(weights[n], ctx)
        else:
            _upload_group(ctx, st, optimizer[n])


def write_sfnn_checkpoint(output_dir, ctx, runner, log: CheckpointLog, completed_steps: int, optimizer_steps: int,
                          quantized=None, feature_set: str = "halfka_hm2") -> Path:
    """A numbered SFNN checkpoint: nn.bin from the device quantisation of the
    runner's weights (when ``quantized``, a QuantizedSfnnDeviceWeights, is
    given), state.bin, dataloader_pos.txt and learn.log."""
    from .nn_bin import write_sfnn_nn_bin
    from .sfnn import sfnn_quantize_device

    def payload(tmp: Path) -> None:
        if quantized is not None:
            sfnn_quantize_device(ctx, runner.shape, runner.weights, quantized, runner.alpha)
            write_sfnn_nn_bin(tmp / "nn.bin", ctx, quantized, feature_set)
        write_sfnn_state_bin(tmp / "state.bin", ctx, runner, completed_steps, optimizer_steps)

    return write_checkpoint_dir(output_dir, log, payload)


def write_halfkp_checkpoint(output_dir, ctx, runner, log: CheckpointLog, completed_steps: int, quantized=None,
                            feature_set: str = "halfkp") -> Path:
    """A numbered HalfKP checkpoint (write_cuda_cpp_nnue_numbered_checkpoint,
    examples/bulletou.rs:20925-20948): nn.bin from the device quantisation of
    the runner's weights (when ``quantized``, a QuantizedNnueDeviceWeights, is
    given), state.bin, dataloader_pos.txt and learn.log."""
    from .nn_bin import write_nnue_nn_bin
    from .nnue_quant import nnue_quantize_device

    def payload(tmp: Path) -> None:
        if quantized is not None:
            nnue_quantize_device(ctx, dict(zip(HALFKP_NAMES, runner.weights)), quantized)
            write_nnue_nn_bin(tmp / "nn.bin", ctx, quantized, feature_set)
        write_halfkp_state_bin(tmp / "state.bin", ctx, runner, completed_steps)

    return write_checkpoint_dir(output_dir, log, payload)
