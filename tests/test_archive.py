"""The quantized weight archive (NcnnQ8Archive.cs), pinned by the reference's
Qwen35Q8ArchiveTests (Packages/com.aexis/Samples/AIImageApplicationExample/
Editor/Qwen35Q8ArchiveTests.cs:125-197), and its direct GPU upload."""
import io
import math
import struct

import numpy as np
import pytest

from aiimage_b200 import archive, errors


def test_round_trip_tolerance_and_record_boundaries():
    """CaptureRoundTripPreservesRecordBoundariesAndTolerance: 8193 values
    sin(i*0.017)*(1+i%13), block 256, threshold 16 -> max error <= 13/127."""
    vals = np.array([math.sin(i * 0.017) * (1 + i % 13) for i in range(8193)], dtype=np.float32)
    buf = io.BytesIO()
    with archive.ArchiveWriter(buf, vals.nbytes, default_block_size=256, fp32_threshold=16) as w:
        w.write_ncnn_array(vals)
    buf.seek(0)
    r = archive.ArchiveReader(buf)
    assert r.record_count == 1
    restored = r.read_array(vals.size)
    assert np.max(np.abs(restored - vals)) <= 13 / 127 + 1e-6
    assert buf.tell() == len(buf.getvalue())


def test_small_fp32_record_is_bit_exact():
    """SmallFp32RecordIsBitExact: -0, 1.25, -9.5, float.Epsilon."""
    expected = np.array([-0.0, 1.25, -9.5, np.float32(1.4e-45)], dtype=np.float32)
    buf = io.BytesIO()
    with archive.ArchiveWriter(buf, 20, default_block_size=256, fp32_threshold=4096) as w:
        w.write_ncnn_array(expected)
    buf.seek(0)
    got = archive.ArchiveReader(buf).read_array(4)
    assert np.array_equal(got.view(np.uint32), expected.view(np.uint32))


def test_forced_fp32_above_threshold_is_bit_exact():
    """RawLoadTypeConstantRemainsFp32AboveQuantizationThreshold."""
    expected = (np.arange(5000, dtype=np.uint32) + 0x3F000000).view(np.float32)
    buf = io.BytesIO()
    with archive.ArchiveWriter(buf, expected.nbytes, default_block_size=256, fp32_threshold=16) as w:
        w.write_ncnn_array(expected, force_fp32=True)
    buf.seek(0)
    assert np.array_equal(archive.ArchiveReader(buf).read_array(5000, require_raw=True), expected)


def test_packed_row_wise_read_uses_one_scale_per_row(oracle):
    """PackedRowWiseReadUsesOneScalePerRow: rows 3, cols 8 -> 3 scales, 6 words;
    and the packed values equal the per-row quantizer's."""
    rows, cols = 3, 8
    vals = np.array([(r + 1) * (c - 3.5) for r in range(rows) for c in range(cols)], dtype=np.float32)
    buf = io.BytesIO()
    with archive.ArchiveWriter(buf, vals.nbytes, cols, 0) as w:
        w.write_q8(vals, cols)
    buf.seek(0)
    packed, scales, block = archive.ArchiveReader(buf).read_packed_array(vals.size, cols)
    assert scales.size == rows and packed.size == (vals.size + 3) // 4 and block == cols
    p, s = oracle.quantize_rows(8, vals, rows, cols, True)
    assert np.array_equal(packed, p) and np.array_equal(scales, s)


def test_q4_record_matches_quantizer_and_dequant(oracle):
    r = np.random.default_rng(3)
    n, k, g = 16, 64, 16
    vals = r.standard_normal(n * k).astype(np.float32)
    buf = io.BytesIO()
    with archive.ArchiveWriter(buf, vals.nbytes, g, 0, quantization_bits=4) as w:
        w.write_ncnn_array(vals)
    buf.seek(0)
    packed, scales, block = archive.ArchiveReader(buf).read_q4_packed_array(n * k, g)
    # A block is a row of the per-channel quantizer with per_ch = g.
    p, s = oracle.quantize_rows(4, vals, n * k // g, g, True)
    assert np.array_equal(packed, p) and np.array_equal(scales, s)
    buf.seek(0)
    deq = archive.ArchiveReader(buf).read_array(n * k)
    assert np.array_equal(deq, oracle.dequant(4, packed, scales, g, n, k).reshape(-1))


def test_odd_tail_block_and_q4_from_q8(oracle):
    vals = np.linspace(-3, 3, 1001).astype(np.float32)
    for bits in (4, 8):
        buf = io.BytesIO()
        with archive.ArchiveWriter(buf, vals.nbytes, 64, 0, quantization_bits=bits) as w:
            w.write_ncnn_array(vals)
        buf.seek(0)
        got = archive.ArchiveReader(buf).read_array(vals.size)
        assert np.max(np.abs(got - vals)) <= (3 / 7 if bits == 4 else 3 / 127) / 2 + 1e-6
    # WriteQ4FromQ8Rows: per-row Q8 -> Q4 groups of 32.
    rows, cols = 4, 64
    v = np.random.default_rng(5).standard_normal(rows * cols).astype(np.float32)
    p8, s8 = oracle.quantize_rows(8, v, rows, cols, True)
    buf = io.BytesIO()
    with archive.ArchiveWriter(buf, v.nbytes, 32, 0, quantization_bits=4) as w:
        w.write_q4_from_q8_rows(p8, s8, rows, cols, 32)
    buf.seek(0)
    p4, s4, blk = archive.ArchiveReader(buf).read_q4_packed_array(rows * cols, 32)
    assert blk == 32 and s4.size == rows * cols // 32
    deq = oracle.dequant(4, p4, s4, 32, rows, cols)
    assert np.max(np.abs(deq.reshape(-1) - v)) <= np.abs(v).max() / 7 / 2 + np.abs(v).max() / 127


def test_reader_rejects_corruption():
    buf = io.BytesIO()
    with archive.ArchiveWriter(buf, 0, 8, 0) as w:
        w.write_q8(np.ones(16, np.float32), 8)
    data = bytearray(buf.getvalue())
    with pytest.raises(archive.InvalidDataError):
        archive.ArchiveReader(io.BytesIO(b"\0" * 32))
    r = archive.ArchiveReader(io.BytesIO(bytes(data)))
    with pytest.raises(archive.InvalidDataError):
        r.read_packed_array(15)  # element count mismatch
    bad = bytearray(data)
    struct.pack_into("<i", bad, 32 + 16, 999)  # payload bytes
    with pytest.raises(archive.InvalidDataError):
        archive.ArchiveReader(io.BytesIO(bytes(bad))).read_packed_array(16, 8)
    r = archive.ArchiveReader(io.BytesIO(bytes(data)))
    r.read_array(16)
    with pytest.raises(EOFError):
        r.read_array(16)
    with pytest.raises(errors.ArgumentOutOfRangeError):
        archive.ArchiveWriter(io.BytesIO(), 0, quantization_bits=5)


@pytest.mark.gpu
def test_archive_records_upload_and_gemv(ops, oracle):
    """Q8 per-row and Q4 group records go to the GPU with no fp32 round trip;
    the GEMV matches the oracle on the record's packed values."""
    import torch
    r = np.random.default_rng(7)
    n, k = 256, 1024
    w8 = r.standard_normal(n * k).astype(np.float32)
    w4 = r.standard_normal(n * k).astype(np.float32)
    buf = io.BytesIO()
    with archive.ArchiveWriter(buf, 0, 16, 0, quantization_bits=4) as w:
        w.write_q8(w8, k)
        w.write_q4(w4, 16)
    buf.seek(0)
    rd = archive.ArchiveReader(buf)
    h8 = archive.upload_q8_record(ops, rd, n, k)
    h4 = archive.upload_q4_record(ops, rd, n, k)
    buf.seek(0)
    rd2 = archive.ArchiveReader(buf)
    p8, s8, _ = rd2.read_packed_array(n * k, k)
    p4, s4, _ = rd2.read_q4_packed_array(n * k, 16)
    x = np.random.default_rng(8).standard_normal((1, k)).astype(np.float32)
    for h, bits, p, s, g in ((h8, 8, p8, s8, 0), (h4, 4, p4, s4, 16)):
        ops.set_int8_gemm_weights(h if bits == 8 else None)
        ops.set_int4_gemm_weights(h if bits == 4 else None)
        y = torch.zeros((1, n), dtype=torch.float32, device="cuda")
        ops.gemm2d_pack4_linear_texture_a(torch.from_numpy(x).cuda(), None, 1, n, k, output=y)
        torch.cuda.synchronize()
        ref = oracle.gemm(x, bits, p, s, g, n)
        err = np.abs(y.cpu().numpy() - ref)
        assert (err <= 1e-2 * np.abs(ref) + 1e-3 * np.abs(ref).max()).all()
