"""The AIImage quantized weight archive (NcnnQ8Archive) and its direct upload
to libaexis_cuda weight handles.

Format (Packages/com.aexis/Runtime/Ncnn/NcnnCompute/NcnnQ8Archive.cs:24-267),
little-endian:
  header (32 B): u64 magic 0x0038544547535141, u32 version 1, u32 bits (4|8),
                 i32 default block, i32 record count, i64 source bytes
  record (24 B): u32 magic 0x31523851 ("Q8R1"), i32 kind (1 Q8, 2 raw, 3 Q4),
                 i32 element count, i32 block size, i32 payload bytes, i32 0
  payload: raw = float32 values; Q8/Q4 = per block an fp32 scale followed by
           `length` int8 bytes (Q8) or ceil(length/2) bytes of nibbles, low
           nibble = even element (Q4).
Block scale = maxAbs/127 (or /7), 1 when the block is all zero; values
RoundToInt (midpoint to even) and clamped to [-127, 127] (or [-7, 7]).

The reader returns packed arrays in the kernels' layout (four int8 or eight
nibbles per uint32, flat element index, NcnnQ8Archive.cs:341-413), so a record
goes to the GPU with no fp32 round trip.
"""
from __future__ import annotations

import io
import struct

import numpy as np

from . import errors

MAGIC = 0x0038544547535141
VERSION = 1
RECORD_MAGIC = 0x31523851
HEADER_BYTES = 32
RECORD_HEADER_BYTES = 24
RECORD_Q8, RECORD_RAW, RECORD_Q4 = 1, 2, 3


class InvalidDataError(errors.AexisError, ValueError):
    """InvalidDataException of the reference reader."""


def _blocks(values: np.ndarray, block: int):
    n = values.size
    for off in range(0, n, block):
        yield off, values[off:off + block]


def _quantize_block(v: np.ndarray, qmax: float, lim: int):
    max_abs = np.float32(np.abs(v).max()) if v.size else np.float32(0)
    scale = np.float32(max_abs / np.float32(qmax)) if max_abs > 0 else np.float32(1)
    q = np.clip(np.rint((v / scale).astype(np.float32)), -lim, lim).astype(np.int8)
    return scale, q


class ArchiveWriter:
    """NcnnQ8ArchiveWriter (NcnnQ8Archive.cs:24-267)."""

    def __init__(self, stream, source_bytes: int, default_block_size: int = 256, fp32_threshold: int = 4096,
                 quantization_bits: int = 8):
        if stream is None:
            raise errors.ArgumentNullError("stream")
        if default_block_size <= 0:
            raise errors.ArgumentOutOfRangeError("defaultBlockSize")
        if fp32_threshold < 0:
            raise errors.ArgumentOutOfRangeError("fp32Threshold")
        if quantization_bits not in (4, 8):
            raise errors.ArgumentOutOfRangeError("quantizationBits")
        self.stream, self.block, self.threshold, self.bits = stream, default_block_size, fp32_threshold, quantization_bits
        self.records = 0
        self._start = stream.tell()
        stream.write(struct.pack("<QIIiiq", MAGIC, VERSION, quantization_bits, default_block_size, 0, source_bytes))

    def _record(self, kind, count, block, payload):
        self.stream.write(struct.pack("<Iiiiii", RECORD_MAGIC, kind, count, block, payload, 0))
        self.records += 1

    def write_ncnn_array(self, values, block_size: int = 0, force_fp32: bool = False):
        v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        if force_fp32 or v.size <= self.threshold:
            return self.write_float32_array(v)
        bs = block_size if block_size > 0 else self.block
        return self.write_q4(v, bs) if self.bits == 4 else self.write_q8(v, bs)

    def write_q8(self, values, block_size: int):
        v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        if block_size <= 0:
            raise errors.ArgumentOutOfRangeError("blockSize")
        nblocks = (v.size + block_size - 1) // block_size
        self._record(RECORD_Q8, v.size, block_size, v.size + nblocks * 4)
        for _, b in _blocks(v, block_size):
            scale, q = _quantize_block(b, 127.0, 127)
            self.stream.write(struct.pack("<f", scale))
            self.stream.write(q.tobytes())

    @staticmethod
    def _q4_payload(count, block):
        return sum(4 + (min(block, count - off) + 1) // 2 for off in range(0, count, block))

    def write_q4(self, values, block_size: int):
        v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        if block_size <= 0:
            raise errors.ArgumentOutOfRangeError("blockSize")
        self._record(RECORD_Q4, v.size, block_size, self._q4_payload(v.size, block_size))
        for _, b in _blocks(v, block_size):
            scale, q = _quantize_block(b, 7.0, 7)
            self.stream.write(struct.pack("<f", scale))
            self.stream.write(_pack_nibbles(q).tobytes())

    def write_q4_from_q8_rows(self, packed: np.ndarray, scales: np.ndarray, rows: int, row_size: int, group: int):
        """WriteQ4FromQ8Rows (:167-207): re-quantise per-row Q8 to Q4 groups;
        group scale = rowScale * maxAbs(q8) / 7, q4 = RoundToInt(q8 * 7 / maxAbs)."""
        if rows <= 0 or row_size <= 0:
            raise errors.ArgumentError("Q8 row source shape is invalid.")
        scales = np.asarray(scales, dtype=np.float32)
        if scales.size != rows:
            raise InvalidDataError("Q8 row source must contain one scale per embedding row.")
        if group <= 0 or row_size % group != 0:
            raise errors.ArgumentError("Q4 embedding group size must divide the embedding row width.")
        count = rows * row_size
        q8 = np.ascontiguousarray(packed, dtype=np.uint32).view(np.int8)[:count].reshape(rows, row_size // group, group)
        self._record(RECORD_Q4, count, group, self._q4_payload(count, group))
        max_abs = np.abs(q8.astype(np.int32)).max(axis=2)
        for r in range(rows):
            for g in range(row_size // group):
                m = int(max_abs[r, g])
                scale = np.float32(np.float32(scales[r] * np.float32(m)) / np.float32(7)) if m > 0 else np.float32(1)
                if m > 0:
                    q4 = np.clip(np.rint((q8[r, g].astype(np.float32) * np.float32(7)) / np.float32(m)), -7, 7)
                else:
                    q4 = np.zeros(group)
                self.stream.write(struct.pack("<f", scale))
                self.stream.write(_pack_nibbles(q4.astype(np.int8)).tobytes())

    def write_raw(self, data: bytes):
        self._record(RECORD_RAW, len(data), 1, len(data))
        self.stream.write(data)

    def write_float32_array(self, values):
        b = np.ascontiguousarray(values, dtype=np.float32).tobytes()
        self._record(RECORD_RAW, len(b) // 4, 1, len(b))
        self.stream.write(b)

    def close(self):
        end = self.stream.tell()
        self.stream.seek(self._start + 20)
        self.stream.write(struct.pack("<i", self.records))
        self.stream.seek(end)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _pack_nibbles(q: np.ndarray) -> np.ndarray:
    q = (q.astype(np.int8) & 0xF).astype(np.uint8)
    if q.size % 2:
        q = np.concatenate([q, np.zeros(1, np.uint8)])
    return (q[0::2] | (q[1::2] << 4)).astype(np.uint8)


class ArchiveReader:
    """NcnnQ8ArchiveReader (NcnnQ8Archive.cs:269-503)."""

    def __init__(self, stream):
        if stream is None:
            raise errors.ArgumentNullError("stream")
        self.stream = stream
        head = stream.read(HEADER_BYTES)
        if len(head) < HEADER_BYTES:
            raise InvalidDataError("Invalid AIImage Q8 archive magic.")
        magic, version, bits, block, count, _ = struct.unpack("<QIIiiq", head)
        if magic != MAGIC:
            raise InvalidDataError("Invalid AIImage Q8 archive magic.")
        if version != VERSION:
            raise InvalidDataError(f"Unsupported AIImage Q8 archive version: {version}")
        if block <= 0 or count < 0 or bits not in (0, 4, 8):
            raise InvalidDataError("Invalid AIImage quantized archive header.")
        self.bits = 8 if bits == 0 else bits
        self.default_block = block
        self.record_count, self.records_read = count, 0

    def _header(self, expected_count: int):
        if self.records_read >= self.record_count:
            raise EOFError("Q8 archive has no remaining records.")
        pos = self.stream.tell()
        raw = self.stream.read(RECORD_HEADER_BYTES)
        if len(raw) < RECORD_HEADER_BYTES:
            raise EOFError("Unexpected end of Q8 archive source.")
        magic, kind, count, block, payload, _ = struct.unpack("<Iiiiii", raw)
        if magic != RECORD_MAGIC:
            raise InvalidDataError(f"Invalid Q8 record magic at {pos}.")
        self.records_read += 1
        if count != expected_count:
            raise InvalidDataError(f"Q8 record element count mismatch. expected={expected_count} actual={count} "
                                   f"record={self.records_read}.")
        if block <= 0 or payload < 0:
            raise InvalidDataError("Invalid Q8 record header.")
        return kind, count, block, payload

    def _read(self, n: int) -> bytes:
        b = self.stream.read(n)
        if len(b) != n:
            raise EOFError("Unexpected end of Q8 archive source.")
        return b

    def _blocks_payload(self, kind, count, block):
        """Parse all blocks of a Q8/Q4 payload: (scales fp32, values int8)."""
        nblocks = (count + block - 1) // block if count else 0
        per = [min(block, count - i * block) for i in range(nblocks)]
        nbytes = [(l if kind == RECORD_Q8 else (l + 1) // 2) for l in per]
        data = self._read(sum(nbytes) + 4 * nblocks)
        scales = np.empty(nblocks, dtype=np.float32)
        vals = np.empty(count, dtype=np.int8)
        off = 0
        full = block if kind == RECORD_Q8 else (block + 1) // 2
        if nblocks and all(nb == full for nb in nbytes[:-1]):
            # Regular blocks: view the payload as [scale | bytes] rows.
            nreg = nblocks - 1 if nbytes[-1] != full else nblocks
            stride = 4 + full
            reg = np.frombuffer(data, dtype=np.uint8, count=nreg * stride).reshape(nreg, stride)
            scales[:nreg] = reg[:, :4].copy().view(np.float32).reshape(-1)
            body = reg[:, 4:]
            if kind == RECORD_Q8:
                vals[:nreg * block] = body.reshape(-1).view(np.int8)
            else:
                nib = np.empty((nreg, full * 2), dtype=np.uint8)
                nib[:, 0::2], nib[:, 1::2] = body & 0xF, body >> 4
                vals[:nreg * block] = np.where(nib[:, :block] >= 8, nib[:, :block].astype(np.int16) - 16,
                                               nib[:, :block]).astype(np.int8).reshape(-1)
            off = nreg * stride
            start = nreg
        else:
            start = 0
        for b in range(start, nblocks):
            scales[b] = struct.unpack_from("<f", data, off)[0]
            off += 4
            l = per[b]
            raw = np.frombuffer(data, dtype=np.uint8, count=nbytes[b], offset=off)
            off += nbytes[b]
            if kind == RECORD_Q8:
                vals[b * block:b * block + l] = raw.view(np.int8)
            else:
                nib = np.empty(raw.size * 2, dtype=np.uint8)
                nib[0::2], nib[1::2] = raw & 0xF, raw >> 4
                vals[b * block:b * block + l] = np.where(nib[:l] >= 8, nib[:l].astype(np.int16) - 16,
                                                         nib[:l]).astype(np.int8)
        return scales, vals, sum(nbytes) + 4 * nblocks

    def read_array(self, expected_count: int, require_raw: bool = False) -> np.ndarray:
        """ReadArray (:295-339): fp32 values (raw, or dequantised q * scale)."""
        kind, count, block, payload = self._header(expected_count)
        if kind == RECORD_RAW:
            if payload != expected_count * 4:
                raise InvalidDataError("Q8 raw float record size mismatch.")
            return np.frombuffer(self._read(payload), dtype=np.float32).copy()
        if require_raw:
            raise InvalidDataError("Expected a raw FP32 quantized archive record.")
        if kind not in (RECORD_Q8, RECORD_Q4):
            raise InvalidDataError("Expected a quantized array record.")
        scales, vals, consumed = self._blocks_payload(kind, count, block)
        if consumed != payload:
            raise InvalidDataError(f"Q8 payload size mismatch. expected={payload} actual={consumed}.")
        return (vals.astype(np.float32) * np.repeat(scales, block)[:count]).astype(np.float32)

    def _read_packed(self, want_kind, expected_count, expected_block):
        kind, count, block, payload = self._header(expected_count)
        name = "Q8" if want_kind == RECORD_Q8 else "Q4"
        if kind != want_kind:
            raise InvalidDataError(f"Expected a {name} packed array record.")
        if expected_block > 0 and block != expected_block:
            raise InvalidDataError(f"{name} block size mismatch. expected={expected_block} actual={block}")
        scales, vals, consumed = self._blocks_payload(kind, count, block)
        if consumed != payload:
            raise InvalidDataError(f"Q8 payload size mismatch. expected={payload} actual={consumed}.")
        if want_kind == RECORD_Q8:
            words = max(1, (count + 3) // 4)
            buf = np.zeros(words * 4, dtype=np.int8)
            buf[:count] = vals
            return buf.view(np.uint32), scales, block
        words = max(1, (count + 7) // 8)
        nib = np.zeros(words * 8, dtype=np.uint8)
        nib[:count] = vals.view(np.uint8) & 0xF
        packed = (nib[0::2] | (nib[1::2] << 4)).astype(np.uint8)
        return packed.view(np.uint32), scales, block

    def read_packed_array(self, expected_count: int, expected_block: int = 0):
        """ReadPackedArray (:341-367): (packed uint32, block scales fp32, block)."""
        return self._read_packed(RECORD_Q8, expected_count, expected_block)

    def read_q4_packed_array(self, expected_count: int, expected_block: int = 0):
        """ReadQ4PackedArray (:385-413): (packed uint32, block scales fp32, block)."""
        return self._read_packed(RECORD_Q4, expected_count, expected_block)

    def read_raw(self, expected_bytes: int) -> bytes:
        kind, count, block, payload = self._header(expected_bytes)
        if kind != RECORD_RAW or payload != expected_bytes:
            raise InvalidDataError("Q8 raw record mismatch.")
        return self._read(expected_bytes)

    def skip_record(self, expected_count: int):
        kind, count, block, payload = self._header(expected_count)
        self.stream.seek(payload, io.SEEK_CUR)


def upload_q8_record(ops, reader: ArchiveReader, n: int, k: int):
    """A per-row Q8 record (block == k) straight to a device weight handle
    (AexisGemmLayer.LoadLayer -> NewInt8WeightOnlyUpload(direct))."""
    packed, scales, block = reader.read_packed_array(n * k, k)
    return ops.new_int8_weight_only_upload(packed, scales, n, k)


def upload_q4_record(ops, reader: ArchiveReader, n: int, k: int):
    """A Q4 record straight to a device weight handle; the record's block is
    the scale group (it must divide k, as NewInt4WeightOnlyUpload requires)."""
    packed, scales, block = reader.read_q4_packed_array(n * k)
    return ops.new_int4_weight_only_upload(packed, scales, n, k, block)
