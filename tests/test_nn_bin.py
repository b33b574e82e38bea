"""nn.bin writer: header, hashes and section layout of the reference's HalfKP
writer (write_cuda_cpp_nnue_nn_bin, examples/bulletou.rs:26309-26375; helpers
crates/bulletou_lib/src/value/nnue_save.rs:1-222), on CPU from the oracle's
quantisation, and on the GPU from the device quantisation (marked gpu)."""
import struct

import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import nn_bin as nb
from bulletou_b200 import synthetic
from oracle import oracle

SHAPE = (125388, 256, 32, 32)


def test_header_known_answers():
    """header_length_matches_components (nnue_save.rs:266-272), the HalfKP
    feature hash (shogi_halfkp.rs:25); the network hash of halfkp_256x2-32-32
    is the value the engine checks when it loads such a file."""
    h = nb.header_bytes("halfkp", 256, 32, 32)
    desc = nb.description("halfkp", 256, 32, 32)
    assert len(h) == 12 + len(desc)
    assert h[0:4] == struct.pack("<I", nb.NNUE_VERSION) and nb.NNUE_VERSION == 0x7AF32F16
    assert struct.unpack("<I", h[8:12])[0] == len(desc) and h[12:].decode() == desc
    assert nb.FEATURE_HASHES["halfkp"] == 0x5D69D5B8 and nb.FEATURE_HASHES["halfka_hm2"] == 0x7F234CB8
    assert struct.unpack("<I", h[4:8])[0] == nb.network_hash("halfkp", 256, 32, 32) == 0x3E5AA6EE
    assert desc.startswith("Features=HalfKP(Friend)[125388->256x2],Network=AffineTransform[1<-32]")


def _parse(blob, l1=256, l2=32, l3=32):
    """Section boundaries in the writer's order."""
    off = 12 + struct.unpack("<I", blob[8:12])[0]
    out = {"ft_hash": struct.unpack("<I", blob[off:off + 4])[0]}
    off += 4
    rows = 125388

    def take(name, dtype, n):
        nonlocal off
        a = np.frombuffer(blob, dtype, n, off)
        out[name] = a
        off += a.nbytes

    take("l0b", np.int16, l1)
    take("l0w", np.int16, rows * l1)
    out["fc_hash"] = struct.unpack("<I", blob[off:off + 4])[0]
    off += 4
    take("l1b", np.int32, l2)
    take("l1w", np.int8, l2 * ((2 * l1 + 31) // 32 * 32))
    take("l2b", np.int32, l3)
    take("l2w", np.int8, l3 * ((l2 + 31) // 32 * 32))
    take("outb", np.int32, 1)
    take("outw", np.int8, (l3 + 31) // 32 * 32)
    out["end"] = off
    return out


@pytest.mark.parametrize("factorized", [False, True])
def test_sections_from_the_oracle_quantisation(factorized):
    shape = (SHAPE[0] + 1548 if factorized else SHAPE[0],) + SHAPE[1:]
    w = synthetic.halfkp_weights(synthetic.rng_for(3), input_size=shape[0], std=0.05)
    q = oracle.nnue_quantize(shape, w)
    blob = nb.nnue_nn_bin_bytes(q, 256, 32, 32)
    p = _parse(blob)
    assert p["end"] == len(blob)
    assert p["ft_hash"] == nb.ft_hash("halfkp", 256) and p["fc_hash"] == nb.compute_fc_hash(256, 32, 32)
    for k in oracle.NNUE_QUANT_NAMES:
        np.testing.assert_array_equal(p[k], np.asarray(q[k]).reshape(-1), err_msg=k)


@pytest.mark.gpu
def test_device_quantised_file_matches_the_oracle_bytes(ctx, tmp_path):
    shape = (SHAPE[0] + 1548,) + SHAPE[1:]
    w = synthetic.halfkp_weights(synthetic.rng_for(4), input_size=shape[0], std=0.05)
    dw = {n: bo.F32Buffer.from_host(ctx, w[n]) for n in oracle.NNUE_QUANT_NAMES}
    dq = bo.QuantizedNnueDeviceWeights(ctx, *shape)
    bo.nnue_quantize_device(ctx, dw, dq)
    n = nb.write_nnue_nn_bin(tmp_path / "nn.bin", ctx, dq)
    want = nb.nnue_nn_bin_bytes(oracle.nnue_quantize(shape, w), 256, 32, 32)
    got = (tmp_path / "nn.bin").read_bytes()
    assert n == len(got) == len(want) and got == want
    w["l1w"][0] = 10.0                                   # 640 is outside i8: the write fails
    dw["l1w"].upload(w["l1w"])
    bo.nnue_quantize_device(ctx, dw, dq)
    with pytest.raises(bo.CudaCppError, match="outside their integer type"):
        nb.write_nnue_nn_bin(tmp_path / "bad.bin", ctx, dq)


# ------------------------------------------------------------------ SFNN
def test_signed_leb128_known_answers():
    """Signed LEB128 as push_sfnn_signed_leb128_i16 (bulletou.rs:26466-26478)
    writes it, and the reader's round trip (read_sfnn_signed_leb128_i16,
    bulletou.rs:7671-7696, restated below)."""
    cases = {0: [0x00], 1: [0x01], -1: [0x7F], 63: [0x3F], 64: [0xC0, 0x00], -64: [0x40], -65: [0xBF, 0x7F],
             127: [0xFF, 0x00], 8191: [0xFF, 0x3F], 8192: [0x80, 0xC0, 0x00], 32767: [0xFF, 0xFF, 0x01],
             -32768: [0x80, 0x80, 0x7E]}
    for v, b in cases.items():
        assert list(nb.signed_leb128_i16([v])) == b, v
    vals = np.random.default_rng(1).integers(-32768, 32768, 5000)
    data = nb.signed_leb128_i16(vals)
    got, pos = [], 0
    while pos < len(data):
        result, shift = 0, 0
        while True:
            byte = data[pos]
            pos += 1
            result |= (byte & 0x7F) << shift
            shift += 7
            if not byte & 0x80:
                if byte & 0x40:
                    result -= 1 << shift
                break
        got.append(result)
    assert got == vals.tolist()


def _sfnn_shape():
    from bulletou_b200 import sfnn as bs

    return bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 256, 15, True, 32, 9)


def test_sfnn_sections_from_the_oracle_quantisation():
    sh = _sfnn_shape()
    w = synthetic.sfnn_weights(synthetic.rng_for(5), sh.input_size, sh.ft_size, sh.l1_hidden, sh.l1_skip,
                               sh.l2_size, sh.num_stacks, True, True, 0.05)
    q = oracle.sfnn_quantize(sh.as_tuple(), w)
    blob = nb.sfnn_nn_bin_bytes(q, sh.ft_size, sh.l1_out, sh.l2_size, sh.l2_in, sh.num_stacks)
    arch = nb.sfnn_architecture("halfka_hm2", 256, 9)
    assert arch == "ModelType=SFNNWithoutPsqt;Features=HalfKA_hm2(Friend)[73305->256x2],Network=SFNN-256{LayerStack=9}"
    assert struct.unpack("<III", blob[:12]) == (0x7AF32F16, 0x3C203B32, len(arch)) and blob[12:12 + len(arch)] == arch.encode()
    off = 12 + len(arch)
    assert struct.unpack("<I", blob[off:off + 4])[0] == 0x5F134AB8
    off += 4
    for name in ("l0b", "l0w"):
        assert blob[off:off + 17] == b"COMPRESSED_LEB128"
        n = struct.unpack("<I", blob[off + 17:off + 21])[0]
        assert blob[off + 21:off + 21 + n] == nb.signed_leb128_i16(q[name])
        off += 21 + n
    per_stack = 4 + 4 * 16 + 16 * 256 + 4 * 32 + 32 * 32 + 4 + 32
    assert len(blob) - off == 9 * per_stack
    for s in range(9):
        assert struct.unpack("<I", blob[off:off + 4])[0] == 0x6333718A
        l1b = np.frombuffer(blob, np.int32, 16, off + 4)
        np.testing.assert_array_equal(l1b, q["l1b"][s * 16:(s + 1) * 16])
        off += per_stack


@pytest.mark.gpu
def test_sfnn_device_quantised_file_matches_the_oracle_bytes(ctx, tmp_path):
    """The production 1536x2-15-32 LayerStack=9 net with factorizer rows: the
    file written from bulletou_b200_sfnn_quantize_device equals the one built
    from the oracle's quantisation, byte for byte."""
    from bulletou_b200 import sfnn as bs

    sh = bs.SFNN_HALFKA_HM2_1536_15_32_K3K3
    w = synthetic.sfnn_weights(synthetic.rng_for(6), sh.input_size, sh.ft_size, sh.l1_hidden, sh.l1_skip,
                               sh.l2_size, sh.num_stacks, True, False, 0.05)
    dw = {n: (None if w.get(n) is None else bo.F32Buffer.from_host(ctx, w[n])) for n in bs.SFNN_WEIGHT_NAMES}
    dq = bs.QuantizedSfnnDeviceWeights(ctx, sh)
    bs.sfnn_quantize_device(ctx, sh, dw, dq)
    n = nb.write_sfnn_nn_bin(tmp_path / "nn.bin", ctx, dq)
    want = nb.sfnn_nn_bin_bytes(oracle.sfnn_quantize(sh.as_tuple(), w), sh.ft_size, sh.l1_out, sh.l2_size,
                                sh.l2_in, sh.num_stacks)
    got = (tmp_path / "nn.bin").read_bytes()
    assert n == len(want) and got == want


# ------------------------------------------------------------------ readers
def test_halfkp_read_round_trip_and_checks():
    shape = (SHAPE[0] + 1548,) + SHAPE[1:]
    w = synthetic.halfkp_weights(synthetic.rng_for(7), input_size=shape[0], std=0.05)
    q = oracle.nnue_quantize(shape, w)
    blob = nb.nnue_nn_bin_bytes(q, 256, 32, 32)
    got = nb.parse_nnue_nn_bin(blob, SHAPE[0])
    for k in oracle.NNUE_QUANT_NAMES:
        np.testing.assert_array_equal(got[k], np.asarray(q[k]).reshape(-1), err_msg=k)
    assert nb.nnue_nn_bin_bytes(got, 256, 32, 32) == blob
    bad = bytearray(blob)
    bad[4] ^= 1
    with pytest.raises(bo.CudaCppError, match="network hash mismatch"):
        nb.parse_nnue_nn_bin(bytes(bad), SHAPE[0])
    with pytest.raises(bo.CudaCppError, match="truncated"):
        nb.parse_nnue_nn_bin(blob[:-1], SHAPE[0])
    with pytest.raises(bo.CudaCppError, match="trailing"):
        nb.parse_nnue_nn_bin(blob + b"\0", SHAPE[0])


def test_leb128_reader():
    vals = np.random.default_rng(2).integers(-32768, 32768, 10000).astype(np.int16)
    vals[:4] = [0, -1, 32767, -32768]
    data = nb.signed_leb128_i16(vals)
    got, used = nb.read_signed_leb128_i16(data + b"\x05", vals.size)
    assert used == len(data)
    np.testing.assert_array_equal(got, vals)
    with pytest.raises(bo.CudaCppError, match="truncated"):
        nb.read_signed_leb128_i16(data[:-1], vals.size)


def test_sfnn_read_round_trip_and_checks():
    sh = _sfnn_shape()
    w = synthetic.sfnn_weights(synthetic.rng_for(8), sh.input_size, sh.ft_size, sh.l1_hidden, sh.l1_skip,
                               sh.l2_size, sh.num_stacks, True, True, 0.05)
    q = oracle.sfnn_quantize(sh.as_tuple(), w)
    args = (sh.ft_size, sh.l1_out, sh.l2_size, sh.l2_in, sh.num_stacks)
    blob = nb.sfnn_nn_bin_bytes(q, *args)
    rows = sh.factorized_base()
    got = nb.parse_sfnn_nn_bin(blob, rows, *args)
    for k in q:
        np.testing.assert_array_equal(got[k], np.asarray(q[k]).reshape(-1), err_msg=k)
    assert nb.sfnn_nn_bin_bytes(got, *args) == blob
    with pytest.raises(bo.CudaCppError, match="architecture mismatch"):
        nb.parse_sfnn_nn_bin(blob, rows, 512, *args[1:])
    with pytest.raises(bo.CudaCppError):
        nb.parse_sfnn_nn_bin(blob[:-3], rows, *args)


@pytest.mark.gpu
def test_read_files_into_device_weights(ctx, tmp_path):
    """A file written from the device quantisation loads back into fresh
    device tensors unchanged (HalfKP and SFNN)."""
    from bulletou_b200 import sfnn as bs

    shape = (SHAPE[0] + 1548,) + SHAPE[1:]
    w = synthetic.halfkp_weights(synthetic.rng_for(9), input_size=shape[0], std=0.05)
    dq = bo.QuantizedNnueDeviceWeights(ctx, *shape)
    bo.nnue_quantize_device(ctx, {n: bo.F32Buffer.from_host(ctx, w[n]) for n in oracle.NNUE_QUANT_NAMES}, dq)
    nb.write_nnue_nn_bin(tmp_path / "a.bin", ctx, dq)
    back = bo.QuantizedNnueDeviceWeights(ctx, *shape)
    nb.read_nnue_nn_bin(tmp_path / "a.bin", ctx, back)
    a, b = dq.download(ctx), back.download(ctx)
    for k in oracle.NNUE_QUANT_NAMES:
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)
    sh = _sfnn_shape()
    sw = synthetic.sfnn_weights(synthetic.rng_for(10), sh.input_size, sh.ft_size, sh.l1_hidden, sh.l1_skip,
                                sh.l2_size, sh.num_stacks, True, False, 0.05)
    sq = bs.QuantizedSfnnDeviceWeights(ctx, sh)
    bs.sfnn_quantize_device(ctx, sh, {n: (None if sw.get(n) is None else bo.F32Buffer.from_host(ctx, sw[n]))
                                      for n in bs.SFNN_WEIGHT_NAMES}, sq)
    nb.write_sfnn_nn_bin(tmp_path / "s.bin", ctx, sq)
    sback = bs.QuantizedSfnnDeviceWeights(ctx, sh)
    nb.read_sfnn_nn_bin(tmp_path / "s.bin", ctx, sback)
    a, b = sq.download(ctx), sback.download(ctx)
    for k in a:
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)
