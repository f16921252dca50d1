"""Test infrastructure, not product code: a Python/numpy restatement of the reference's WAV reader,
used only by the tests as the checker for the library's host decoder (ge_audio_decode_wav).

It follows WAVDecoder.decode (Sources/GemmaEmbed/Audio/WAVDecoder.swift:29-84), which reads a
RIFF/WAVE file into the float32 samples miniaudio's dr_wav returns for an f32 request:

- the chunk walk (WAVDecoder.swift:36-53) stops at `data`, so `fmt ` must come before it; `fact`
  chunks have their 4-byte count read; other chunks are skipped with their odd-size padding; a
  skip that leaves the file ends the walk;
- the format checks (WAVDecoder.swift:55-60) and the frame size (61-63): bits x channels / 8 for
  whole-byte samples, else the block align;
- a data size that overruns the file is clamped to the bytes present and cut to whole frames
  (WAVDecoder.swift:64-67);
- WAVE_FORMAT_EXTENSIBLE defers to its sub-format tag (WAVDecoder.swift:96, 112-121);
- dr_wav's integer conversions (WAVDecoder.swift:132-173): u8 in two float operations, s16 by
  2^-15 in float, s24 by 2^-23 in double, s32 divided by 2^31 in double, 5-8 byte samples placed
  at the top of an int64 and divided by 2^63 - 1 in double; IEEE float 32 copied bit for bit and
  float 64 rounded to float (WAVDecoder.swift:176-193).

Pinned by the reference's own known answers (AudioDecoderTests.swift:64-160), which the tests
check against this module before using it.
"""
import struct

import numpy as np

PCM, IEEE_FLOAT, EXTENSIBLE = 0x0001, 0x0003, 0xFFFE


class WavError(ValueError):
    """The reason dr_wav (as the reference restates it) refuses a file, prefixed "WAV: "."""

    def __init__(self, reason: str):
        super().__init__("WAV: " + reason)


def is_wav(data: bytes) -> bool:
    """AudioDecoder.isWAV (Audio/AudioDecoder.swift:44-46)."""
    return len(data) >= 12 and data[:4] == b"RIFF" and data[8:12] == b"WAVE"


def _read_format(b: bytes, off: int, size: int):
    """WAVDecoder.readFormat (WAVDecoder.swift:99-125): the format fields and the offset after
    the chunk."""
    n = len(b)
    if n - off < 16:
        raise WavError("fmt chunk is truncated")
    tag, channels, rate, _, block_align, bits = struct.unpack_from("<HHIIHH", b, off)
    off += 16
    sub = 0
    if size > 16:
        if n - off < 2:
            raise WavError("fmt chunk is truncated")
        ext = struct.unpack_from("<H", b, off)[0]
        off += 2
        consumed = 18
        if ext > 0:
            if tag == EXTENSIBLE:
                if ext != 22:
                    raise WavError(f"extensible fmt chunk has a {ext}-byte extension, expected 22")
                if n - off < 22:
                    raise WavError("fmt chunk is truncated")
                sub = struct.unpack_from("<H", b, off + 6)[0]
                off += 22
            else:
                if not 0 <= off + ext <= n:
                    raise WavError("fmt chunk is truncated")
                off += ext
            consumed += ext
        if not 0 <= off + size - consumed <= n:
            raise WavError("fmt chunk is truncated")
        off += size - consumed
    fmt = dict(tag=tag, channels=channels, rate=rate, block_align=block_align, bits=bits, sub=sub)
    return fmt, off


def decode(data: bytes):
    """WAVDecoder.decode: (interleaved float32 samples, sample rate, channel count)."""
    b = bytes(data)
    n = len(b)
    if n < 4 or b[:4] != b"RIFF":
        raise WavError("not a RIFF file")
    if n < 12 or b[8:12] != b"WAVE":
        raise WavError("not a WAVE file")
    off = 12
    fmt = None
    data_at = data_size = None
    while n - off >= 8:
        cid = b[off:off + 4]
        size = struct.unpack_from("<I", b, off + 4)[0]
        off += 8
        pad = size & 1
        if cid == b"fmt ":
            fmt, off = _read_format(b, off, size)
            if off + pad > n:
                break
            off += pad
        elif cid == b"data":
            data_at, data_size = off, size
            break
        elif cid == b"fact":
            if off + 4 > n:
                raise WavError("fact chunk is truncated")
            off += 4
            t = off + size - 4 + pad
            if not 0 <= t <= n:
                break
            off = t
        else:
            if off + size + pad > n:
                break
            off += size + pad
    if fmt is None:
        raise WavError("no fmt chunk before the data chunk")
    if data_at is None:
        raise WavError("no data chunk")
    if not 0 < fmt["rate"] <= 384000:
        raise WavError(f"sample rate {fmt['rate']} is out of range")
    if not 0 < fmt["channels"] <= 256:
        raise WavError(f"channel count {fmt['channels']} is out of range")
    if not 0 < fmt["bits"] <= 64:
        raise WavError(f"{fmt['bits']} bits per sample is out of range")
    if fmt["block_align"] == 0:
        raise WavError("block align is zero")
    ch, bits = fmt["channels"], fmt["bits"]
    frame = bits * ch // 8 if bits % 8 == 0 else fmt["block_align"]
    size = min(data_size, n - data_at)
    size -= size % frame
    count = (size // frame) * ch
    payload = b[data_at:data_at + size]
    tag = fmt["sub"] if fmt["tag"] == EXTENSIBLE else fmt["tag"]
    if tag == PCM:
        bps = frame // ch
        if bps <= 0 or frame % ch != 0:
            raise WavError(f"{bits}-bit PCM frames do not split evenly over {ch} channels")
        out = _pcm(payload, count, bps)
    elif tag == IEEE_FLOAT:
        out = np.zeros(count, np.float32)
        if bits == 32:
            out = np.frombuffer(payload, "<u4", count).view(np.float32).copy()
        elif frame // ch == 8:
            with np.errstate(over="ignore", invalid="ignore"):  # out-of-range doubles round to inf
                out = np.frombuffer(payload, "<f8", count).astype(np.float32)
    else:
        raise WavError(f"format tag 0x{tag:x} is not PCM or IEEE float")
    return out, fmt["rate"], ch


def _pcm(payload: bytes, count: int, bps: int) -> np.ndarray:
    """dr_wav's integer-to-float conversions, one per sample width (WAVDecoder.swift:132-173)."""
    raw = np.frombuffer(payload, np.uint8, count * bps).reshape(count, bps) if count else np.zeros((0, bps), np.uint8)
    if bps == 1:
        x = raw[:, 0].astype(np.float32)
        return (x * np.float32(0.00784313725490196078)) - np.float32(1.0)
    if bps == 2:
        v = raw.copy().view("<i2").reshape(-1)
        return v.astype(np.float32) * np.float32(0.000030517578125)
    if bps == 3:
        u = (raw[:, 0].astype(np.uint32) << 8) | (raw[:, 1].astype(np.uint32) << 16) | (raw[:, 2].astype(np.uint32) << 24)
        v = u.view(np.int32) >> 8
        return (v.astype(np.float64) * 0.00000011920928955078125).astype(np.float32)
    if bps == 4:
        v = raw.copy().view("<i4").reshape(-1)
        return (v.astype(np.float64) / 2147483648.0).astype(np.float32)
    if 5 <= bps <= 8:
        u = np.zeros(count, np.uint64)
        for k in range(bps):
            u |= raw[:, k].astype(np.uint64) << np.uint64(8 * (8 - bps + k))
        return (u.view(np.int64).astype(np.float64) / 9223372036854775807.0).astype(np.float32)
    return np.zeros(count, np.float32)
