"""Engine nn.bin files from the device's quantised weights.

The HalfKP 256x2-32-32 writer of the reference (write_cuda_cpp_nnue_nn_bin,
examples/bulletou.rs:26309-26375) with the header and hash helpers of
crates/bulletou_lib/src/value/nnue_save.rs:1-222: the version, the network
hash (the FC-chain hash of compute_fc_hash xor the feature-transformer hash),
the architecture description string, the FT hash, then FT biases / weights as
i16, the FC hash, and per dense layer the i32 biases and the i8 weights
(output-major, inputs padded to 32).  The tensors come from
``bulletou_b200_nnue_quantize_device`` already in that layout, so writing is a
download and a concatenation; a value that does not fit its integer type
fails the write, as the reference's quantisation does.
"""
from __future__ import annotations

import struct
from pathlib import Path
from typing import Optional

import numpy as np

from ._lib import CudaCppError
from .cuda_cpp import Context
from .nnue_quant import QuantizedNnueDeviceWeights

NNUE_VERSION = 0x7AF32F16
# feature hashes (Side::kFriend): game/inputs/shogi_halfkp.rs:25, shogi_halfka_hm2.rs:30
FEATURE_HASHES = {"halfkp": 0x5D69D5B8, "halfka_hm2": 0x7F234CB8}
DISPLAY_NAMES = {"halfkp": "HalfKP(Friend)", "halfka_hm2": "HalfKA_hm2(Friend)"}
INPUT_SIZES = {"halfkp": 125_388, "halfka_hm2": 73_305}
M32 = 0xFFFFFFFF


def compute_fc_hash(l1: int, l2: int, l3: int) -> int:
    """compute_fc_hash (nnue_save.rs:93-108): the AffineTransform / ClippedReLU chain."""
    prev = (0xEC42E90D ^ (l1 * 2)) & M32
    for i, out in enumerate((l2, l3, 1)):
        h = (0xCC03DAE4 + out) & M32
        h ^= prev >> 1
        h ^= (prev << 31) & M32
        if i < 2:
            h = (h + 0x538D24C7) & M32
        prev = h
    return prev


def ft_hash(feature_set: str, l1: int) -> int:
    return (FEATURE_HASHES[feature_set] ^ (l1 * 2)) & M32


def network_hash(feature_set: str, l1: int, l2: int, l3: int) -> int:
    return (compute_fc_hash(l1, l2, l3) ^ FEATURE_HASHES[feature_set] ^ (l1 * 2)) & M32


def description(feature_set: str, l1: int, l2: int, l3: int) -> str:
    """The architecture string of nnue_save.rs:114-131."""
    return (f"Features={DISPLAY_NAMES[feature_set]}[{INPUT_SIZES[feature_set]}->{l1}x2],"
            f"Network=AffineTransform[1<-{l3}](ClippedReLU[{l3}](AffineTransform[{l3}<-{l2}](ClippedReLU[{l2}]"
            f"(AffineTransformSparseInput[{l2}<-{l1 * 2}](InputSlice[{l1 * 2}(0:{l1 * 2})])))))")


def header_bytes(feature_set: str, l1: int, l2: int, l3: int) -> bytes:
    desc = description(feature_set, l1, l2, l3).encode()
    return struct.pack("<III", NNUE_VERSION, network_hash(feature_set, l1, l2, l3), len(desc)) + desc


def nnue_nn_bin_bytes(q: dict, l1: int, l2: int, l3: int, feature_set: str = "halfkp") -> bytes:
    """The file from the quantised tensors (NNUE_QUANT_NAMES arrays in the
    engine layout, as QuantizedNnueDeviceWeights.download returns them)."""
    parts = [header_bytes(feature_set, l1, l2, l3), struct.pack("<I", ft_hash(feature_set, l1)),
             np.ascontiguousarray(q["l0b"], np.int16).tobytes(), np.ascontiguousarray(q["l0w"], np.int16).tobytes(),
             struct.pack("<I", compute_fc_hash(l1, l2, l3))]
    for b, w in (("l1b", "l1w"), ("l2b", "l2w"), ("outb", "outw")):
        parts.append(np.ascontiguousarray(q[b], np.int32).tobytes())
        parts.append(np.ascontiguousarray(q[w], np.int8).tobytes())
    return b"".join(parts)


def write_nnue_nn_bin(path, ctx: Context, q: QuantizedNnueDeviceWeights, feature_set: str = "halfkp",
                      data: Optional[dict] = None) -> int:
    """Writes the quantised HalfKP net to `path`; returns the byte count.
    Raises when a parameter fell outside its integer type during the device
    quantisation (write_quantized_i8/i16/i32, bulletou.rs:26520-26575)."""
    arrays = data if data is not None else q.download(ctx)
    if arrays.get("errors", 0):
        raise CudaCppError(f"failed to quantize NNUE nn.bin: {arrays['errors']} value(s) outside their integer type")
    _, l1, l2, l3 = q.dims
    blob = nnue_nn_bin_bytes(arrays, l1, l2, l3, feature_set)
    Path(path).write_bytes(blob)
    return len(blob)


# ------------------------------------------------------------------ SFNN nn.bin
# SFNNwithoutPSQT files (write_cuda_cpp_sfnn_nn_bin_format, examples/bulletou.rs:
# 25998-26300; constants crates/bulletou_lib/src/value/nnue_save_sfnn1536.rs:
# 59-67): header with the SFNN kHash and the "ModelType=SFNNWithoutPsqt..."
# string, the FT hash, FT biases and weights as signed-LEB128 i16 blocks
# ("COMPRESSED_LEB128" + payload length + payload), then per LayerStack the
# network hash, L1 (i32 biases, i8 weights [out][pad32(ft)]), L2 and L3.
SFNN_KHASH = 0x3C203B32
SFNN_FT_HASH = 0x5F134AB8
SFNN_NETWORK_HASH = 0x6333718A
LEB128_MAGIC = b"COMPRESSED_LEB128"


def signed_leb128_i16(values, chunk: int = 1 << 22) -> bytes:
    """push_sfnn_signed_leb128_i16 (bulletou.rs:26466-26478) over an array:
    7 bits a byte, low first, continuation bit 0x80, stop once the rest is
    the sign extension of bit 6 (1 to 3 bytes for an i16)."""
    v = np.asarray(values).reshape(-1)
    if v.size and (v.min() < -32768 or v.max() > 32767):
        raise ValueError("signed LEB128: value outside i16")
    pieces = []
    for start in range(0, v.size, chunk):
        rest = v[start:start + chunk].astype(np.int32)
        out = np.zeros((rest.size, 3), np.uint8)
        length = np.zeros(rest.size, np.int8)
        active = np.ones(rest.size, bool)
        for k in range(3):
            byte = (rest & 0x7F).astype(np.uint8)
            rest = rest >> 7
            sign = (byte & 0x40) != 0
            done = ((rest == 0) & ~sign) | ((rest == -1) & sign)
            out[:, k] = np.where(done | ~active, byte, byte | 0x80)
            length[active] = k + 1
            active &= ~done
        pieces.append(out[np.arange(3)[None, :] < length[:, None]].tobytes())
    return b"".join(pieces)


def leb128_block(values) -> bytes:
    payload = signed_leb128_i16(values)
    return LEB128_MAGIC + struct.pack("<I", len(payload)) + payload


def sfnn_architecture(feature_set: str, ft: int, stacks: int) -> str:
    return (f"ModelType=SFNNWithoutPsqt;Features={DISPLAY_NAMES[feature_set]}[{INPUT_SIZES[feature_set]}->{ft}x2],"
            f"Network=SFNN-{ft}{{LayerStack={stacks}}}")


def sfnn_nn_bin_bytes(q: dict, ft: int, l1_out: int, l2: int, l2_in: int, stacks: int,
                      feature_set: str = "halfka_hm2") -> bytes:
    """The file from the quantised SFNN tensors (SFNN_QUANT_NAMES in the engine
    layout: FT i16 folded, dense i8 [stack][out][pad32(in)], i32 biases)."""
    arch = sfnn_architecture(feature_set, ft, stacks).encode()
    parts = [struct.pack("<III", NNUE_VERSION, SFNN_KHASH, len(arch)), arch, struct.pack("<I", SFNN_FT_HASH),
             leb128_block(q["l0b"]), leb128_block(q["l0w"])]
    p1, p2, p3 = (ft + 31) // 32 * 32, (l2_in + 31) // 32 * 32, (l2 + 31) // 32 * 32
    l1w = np.asarray(q["l1w"], np.int8).reshape(stacks, l1_out * p1)
    l1b = np.asarray(q["l1b"], np.int32).reshape(stacks, l1_out)
    l2w = np.asarray(q["l2w"], np.int8).reshape(stacks, l2 * p2)
    l2b = np.asarray(q["l2b"], np.int32).reshape(stacks, l2)
    l3w = np.asarray(q["l3w"], np.int8).reshape(stacks, p3)
    l3b = np.asarray(q["l3b"], np.int32).reshape(stacks)
    for s in range(stacks):
        parts += [struct.pack("<I", SFNN_NETWORK_HASH), l1b[s].tobytes(), l1w[s].tobytes(), l2b[s].tobytes(),
                  l2w[s].tobytes(), l3b[s:s + 1].tobytes(), l3w[s].tobytes()]
    return b"".join(parts)


def write_sfnn_nn_bin(path, ctx: Context, q, feature_set: str = "halfka_hm2", data: Optional[dict] = None) -> int:
    """Writes a QuantizedSfnnDeviceWeights (bulletou_b200_sfnn_quantize_device,
    which folds the factorizers and rounds like the writer) as nn.bin; returns
    the byte count."""
    sh = q.shape
    arrays = data if data is not None else q.download(ctx)
    blob = sfnn_nn_bin_bytes(arrays, sh.ft_size, sh.l1_out, sh.l2_size, sh.l2_in, sh.num_stacks, feature_set)
    Path(path).write_bytes(blob)
    return len(blob)


# ------------------------------------------------------------------ readers
def _pad32(n: int) -> int:
    return (n + 31) // 32 * 32


class _Reader:
    def __init__(self, blob: bytes, what: str):
        self.b, self.off, self.what = blob, 0, what

    def u32(self) -> int:
        if self.off + 4 > len(self.b):
            raise CudaCppError(f"{self.what}: truncated file")
        v = struct.unpack_from("<I", self.b, self.off)[0]
        self.off += 4
        return v

    def array(self, dtype, n: int) -> np.ndarray:
        nbytes = np.dtype(dtype).itemsize * n
        if self.off + nbytes > len(self.b):
            raise CudaCppError(f"{self.what}: truncated file")
        a = np.frombuffer(self.b, dtype, n, self.off).copy()
        self.off += nbytes
        return a

    def bytes(self, n: int) -> bytes:
        if self.off + n > len(self.b):
            raise CudaCppError(f"{self.what}: truncated file")
        v = self.b[self.off:self.off + n]
        self.off += n
        return v

    def expect(self, value: int, label: str) -> None:
        got = self.u32()
        if got != value:
            raise CudaCppError(f"{self.what}: {label} mismatch: expected 0x{value:08X}, got 0x{got:08X}")

    def end(self) -> None:
        if self.off != len(self.b):
            raise CudaCppError(f"{self.what}: {len(self.b) - self.off} trailing bytes")


def parse_nnue_nn_bin(blob: bytes, rows: int, l1: int = 256, l2: int = 32, l3: int = 32,
                      feature_set: str = "halfkp") -> dict:
    """The quantised tensors of a HalfKP nn.bin (the engine's layout, as
    written by nnue_nn_bin_bytes); header, hashes and sizes are checked."""
    r = _Reader(bytes(blob), "nn.bin")
    r.expect(NNUE_VERSION, "version")
    r.expect(network_hash(feature_set, l1, l2, l3), "network hash")
    desc = r.bytes(r.u32())
    if desc != description(feature_set, l1, l2, l3).encode():
        raise CudaCppError("nn.bin: architecture description mismatch")
    r.expect(ft_hash(feature_set, l1), "feature transformer hash")
    out = {"l0b": r.array("<i2", l1), "l0w": r.array("<i2", rows * l1)}
    r.expect(compute_fc_hash(l1, l2, l3), "network hash of the dense layers")
    for b, w, n_out, n_in in (("l1b", "l1w", l2, 2 * l1), ("l2b", "l2w", l3, l2), ("outb", "outw", 1, l3)):
        out[b] = r.array("<i4", n_out)
        out[w] = r.array("i1", n_out * _pad32(n_in))
    r.end()
    return out


def read_signed_leb128_i16(data: bytes, count: int) -> tuple:
    """count signed-LEB128 values from the start of data; returns (values,
    bytes consumed)."""
    b = np.frombuffer(data, np.uint8)
    ends = np.flatnonzero((b & 0x80) == 0)
    if ends.size < count:
        raise CudaCppError("nn.bin: truncated COMPRESSED_LEB128 block")
    if count == 0:
        return np.zeros(0, np.int16), 0
    ends = ends[:count]
    starts = np.concatenate(([0], ends[:-1] + 1))
    lengths = ends - starts + 1
    if lengths.max() > 3:
        raise CudaCppError("nn.bin: LEB128 value longer than an i16")
    val = np.zeros(count, np.int64)
    for k in range(3):
        has = lengths > k
        val[has] |= (b[starts[has] + k].astype(np.int64) & 0x7F) << (7 * k)
    neg = (b[ends] & 0x40) != 0
    val[neg] -= np.left_shift(np.int64(1), 7 * lengths[neg])
    if val.min() < -32768 or val.max() > 32767:
        raise CudaCppError("nn.bin: LEB128 value outside i16")
    return val.astype(np.int16), int(ends[-1] + 1)


def parse_sfnn_nn_bin(blob: bytes, rows: int, ft: int, l1_out: int, l2: int, l2_in: int, stacks: int,
                      feature_set: str = "halfka_hm2") -> dict:
    """The quantised tensors of an SFNN nn.bin (as written by
    sfnn_nn_bin_bytes), in the engine layout QuantizedSfnnDeviceWeights holds."""
    r = _Reader(bytes(blob), "SFNN nn.bin")
    r.expect(NNUE_VERSION, "version")
    r.expect(SFNN_KHASH, "kHash")
    arch = r.bytes(r.u32())
    if arch != sfnn_architecture(feature_set, ft, stacks).encode():
        raise CudaCppError(f"SFNN nn.bin: architecture mismatch: {arch!r}")
    r.expect(SFNN_FT_HASH, "feature transformer hash")
    out = {}
    for name, n in (("l0b", ft), ("l0w", rows * ft)):
        if r.bytes(len(LEB128_MAGIC)) != LEB128_MAGIC:
            raise CudaCppError(f"SFNN nn.bin: {name} is not a COMPRESSED_LEB128 block")
        size = r.u32()
        payload = r.bytes(size)
        vals, used = read_signed_leb128_i16(payload, n)
        if used != size:
            raise CudaCppError(f"SFNN nn.bin: {name} block holds {size - used} extra bytes")
        out[name] = vals
    parts = {k: [] for k in ("l1b", "l1w", "l2b", "l2w", "l3b", "l3w")}
    for _ in range(stacks):
        r.expect(SFNN_NETWORK_HASH, "stack network hash")
        parts["l1b"].append(r.array("<i4", l1_out))
        parts["l1w"].append(r.array("i1", l1_out * _pad32(ft)))
        parts["l2b"].append(r.array("<i4", l2))
        parts["l2w"].append(r.array("i1", l2 * _pad32(l2_in)))
        parts["l3b"].append(r.array("<i4", 1))
        parts["l3w"].append(r.array("i1", _pad32(l2)))
    r.end()
    out.update({k: np.concatenate(v) for k, v in parts.items()})
    return out


def read_nnue_nn_bin(path, ctx: Context, q: QuantizedNnueDeviceWeights, feature_set: str = "halfkp") -> None:
    """Loads a HalfKP nn.bin into the device tensors of ``q`` (its dims give
    the expected layout)."""
    _, l1, l2, l3 = q.dims
    q.upload(parse_nnue_nn_bin(Path(path).read_bytes(), q.rows, l1, l2, l3, feature_set), ctx)


def read_sfnn_nn_bin(path, ctx: Context, q, feature_set: str = "halfka_hm2") -> None:
    """Loads an SFNN nn.bin into a QuantizedSfnnDeviceWeights."""
    sh = q.shape
    q.upload(parse_sfnn_nn_bin(Path(path).read_bytes(), q.rows, sh.ft_size, sh.l1_out, sh.l2_size, sh.l2_in,
                               sh.num_stacks, feature_set), ctx)
