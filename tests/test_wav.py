"""WAV bytes to samples (WAVDecoder, Audio/WAVDecoder.swift) on CPU: the oracle restatement
(oracle/wav.py) against the reference's known answers and refusal reasons
(AudioDecoderTests.swift:64-160), the library's host decoder (ge_audio_decode_wav) against the
oracle bit for bit on those and on seeded random files of every sample format, header variant and
truncation, the input forms of AudioDecoder.decode (AudioDecoderTests.swift:208-225), and the
library on the reference's WAV fixtures against digests made by an independent reader
(tests/golden/make_wav_golden.py)."""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

from oracle import binding as B
from oracle import wav as W

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "wav_fixtures.json")
# The reference checkout, when this machine has one (GE_REFERENCE=<path>); the digest test skips otherwise.
FIXTURES = os.path.join(os.environ.get("GE_REFERENCE", ""), "Tests/GemmaEmbedTests/Fixtures/audio")

# (bits, tag) of each sample format the reference's tests build (AudioDecoderTests.swift:10-30).
FORMATS = {"u8": (8, 1), "s16": (16, 1), "s24": (24, 1), "s32": (32, 1), "f32": (32, 3), "f64": (64, 3)}
GUID_TAIL = bytes([0x00, 0x00, 0x00, 0x00, 0x10, 0x00, 0x80, 0x00, 0x00, 0xAA, 0x00, 0x38, 0x9B, 0x71])


def chunk(cid: bytes, payload: bytes) -> bytes:
    return cid + struct.pack("<I", len(payload)) + payload + (b"\0" if len(payload) % 2 else b"")


def make_wav(fmt, channels, rate, samples: bytes, extensible=False, before_data=(), declared=None,
             fmt_after_data=False, bits=None, block_align=None) -> bytes:
    """A RIFF/WAVE file around raw little-endian sample bytes, laid out as the reference's test
    builder lays it out: fmt (16 bytes, or 40 with the extensible extension), any extra chunks,
    then data (padded to even length unless its size is declared)."""
    b, tag = FORMATS[fmt]
    bits = b if bits is None else bits
    align = channels * b // 8 if block_align is None else block_align
    body = struct.pack("<HHIIHH", 0xFFFE if extensible else tag, channels, rate, rate * align, align, bits)
    if extensible:
        body += struct.pack("<HHIH", 22, bits, (1 << channels) - 1 if channels < 32 else 0, tag) + GUID_TAIL
    data = b"data" + struct.pack("<I", len(samples) if declared is None else declared) + samples
    if len(samples) % 2 and declared is None:
        data += b"\0"
    out = b"" if fmt_after_data else chunk(b"fmt ", body)
    for c in before_data:
        out += c
    out += data
    if fmt_after_data:
        out += chunk(b"fmt ", body)
    return b"RIFF" + struct.pack("<I", 4 + len(out)) + b"WAVE" + out


def i16(v):
    return np.asarray(v, "<i2").tobytes()


def i24(v):
    return b"".join(struct.pack("<i", x)[:3] for x in v)


def i32(v):
    return np.asarray(v, "<i4").tobytes()


def f32b(v):
    return np.asarray(v, "<f4").tobytes()


def f64b(v):
    return np.asarray(v, "<f8").tobytes()


def lib_decode(ge, data):
    return ge.decode_wav(data)


def both(ge, data):
    """(samples, rate, channels) from the oracle and from the library, which must agree bit for bit."""
    want = W.decode(data)
    got = ge.decode_wav(data)
    assert (got[1], got[2]) == (want[1], want[2])
    assert np.array_equal(got[0].view(np.uint32), want[0].view(np.uint32))
    return want


def f32(xs):
    return np.array(xs, np.float32)


# ---- the reference's known answers (AudioDecoderTests.swift:64-125) ----------------------------

def test_pcm8_unsigned_dr_wav_scaling(ge):
    x, rate, ch = both(ge, make_wav("u8", 1, 16000, bytes([0, 1, 127, 128, 255])))
    assert (ch, rate) == (1, 16000)
    assert np.array_equal(x, f32([-1.0, -0.9921568632125854, -0.0039215087890625, 0.003921627998352051, 1.0]))


def test_pcm16(ge):
    x, rate, _ = both(ge, make_wav("s16", 1, 44100, i16([32767, -32768, 1, -1, 12345])))
    assert rate == 44100
    assert np.array_equal(x, f32([0.999969482421875, -1.0, 3.0517578125e-05, -3.0517578125e-05, 0.376739501953125]))


def test_pcm24(ge):
    x, _, _ = both(ge, make_wav("s24", 1, 48000, i24([8388607, -8388608, 1, -1, -1234567])))
    assert np.array_equal(x, f32([0.9999998807907104, -1.0, 1.1920928955078125e-07, -1.1920928955078125e-07,
                                  -0.14717185497283936]))


def test_pcm32(ge):
    x, _, _ = both(ge, make_wav("s32", 1, 8000, i32([2147483647, -2147483648, 1, -1, 123456789])))
    assert np.array_equal(x, f32([1.0, -1.0, 4.656612873077393e-10, -4.656612873077393e-10, 0.057489048689603806]))


def test_float32_copied_bit_for_bit(ge):
    vals = np.array([0.1, -0.333333343, 1.5, -2.0, 0, 0], np.float32)
    vals.view(np.uint32)[4:] = [0x3F800001, 0x00000001]
    x, _, _ = both(ge, make_wav("f32", 1, 16000, vals.tobytes()))
    assert np.array_equal(x.view(np.uint32), vals.view(np.uint32))


def test_float64_rounds_to_float(ge):
    vals = [0.1, -0.3333333333333333, 1.0 / 3.0, 0.7, -1e-50, 0.0]
    x, _, ch = both(ge, make_wav("f64", 2, 22050, f64b(vals)))
    assert ch == 2
    assert np.array_equal(x, np.array(vals, np.float64).astype(np.float32))


def test_extensible_uses_the_sub_format(ge):
    x, rate, ch = both(ge, make_wav("s24", 6, 44100, i24([4194304] * 12), extensible=True))
    assert (ch, rate) == (6, 44100)
    assert np.array_equal(x, np.full(12, 0.5, np.float32))
    x, _, _ = both(ge, make_wav("f32", 1, 16000, f32b([0.25, -0.75]), extensible=True))
    assert np.array_equal(x, f32([0.25, -0.75]))


def test_unknown_and_odd_chunks_are_skipped(ge):
    lst = chunk(b"LIST", b"INFOISFT" + struct.pack("<I", 7) + b"gemma\0\0")
    extra = [lst, chunk(b"junk", bytes([1, 2, 3])), chunk(b"fact", struct.pack("<I", 3)), chunk(b"bext", b"\xab" * 5)]
    x, _, _ = both(ge, make_wav("s16", 1, 16000, i16([100, 200, -300]), before_data=extra))
    assert np.array_equal(x, f32([100, 200, -300]) * np.float32(0.000030517578125))


def test_overrunning_data_chunk_is_clamped(ge):
    x, _, ch = both(ge, make_wav("s16", 2, 16000, i16([1, 2, 3, 4, 5]) + b"\x07", declared=1_000_000))
    assert len(x) // ch == 2
    assert np.array_equal(x, f32([1, 2, 3, 4]) * np.float32(0.000030517578125))


REFUSALS = [
    (b"RIFX\0\0\0\0WAVE", "WAV: not a RIFF file"),
    (b"RIFF\0\0\0\0AVI ", "WAV: not a WAVE file"),
    (make_wav("s16", 1, 16000, i16([1]), fmt_after_data=True), "WAV: no fmt chunk before the data chunk"),
    (b"RIFF" + struct.pack("<I", 4) + b"WAVE" + chunk(b"fmt ", bytes(16)), "WAV: no data chunk"),
    (lambda b: b[:20] + b"\x02" + b[21:])(make_wav("s16", 1, 16000, i16([1, 2]))),
    (lambda b: b[:22] + b"\x00" + b[23:])(make_wav("s16", 1, 16000, i16([1, 2]))),
    (b"RIFF" + struct.pack("<I", 4) + b"WAVE" + b"fmt " + struct.pack("<I", 16) + bytes([1, 0]), "WAV: fmt chunk is truncated"),
]
REFUSALS[4] = (REFUSALS[4], "WAV: format tag 0x2 is not PCM or IEEE float")
REFUSALS[5] = (REFUSALS[5], "WAV: channel count 0 is out of range")


@pytest.mark.parametrize("case", range(len(REFUSALS)))
def test_malformed_files_refused_with_the_reason(ge, case):
    """testMalformedFilesAreRejectedWithAReason (AudioDecoderTests.swift:127-160)."""
    data, reason = REFUSALS[case]
    with pytest.raises(W.WavError) as e:
        W.decode(data)
    assert str(e.value) == reason
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.decode_wav(data)
    assert e.value.case == "audioDecoding"
    assert e.value.message == "cannot decode audio: " + reason


def test_other_refusals_agree(ge):
    base = make_wav("s16", 1, 16000, i16([1, 2]))
    cases = {
        "WAV: sample rate 0 is out of range": base[:24] + struct.pack("<I", 0) + base[28:],
        "WAV: sample rate 384001 is out of range": base[:24] + struct.pack("<I", 384001) + base[28:],
        "WAV: channel count 257 is out of range": base[:22] + struct.pack("<H", 257) + base[24:],
        "WAV: 0 bits per sample is out of range": base[:34] + struct.pack("<H", 0) + base[36:],
        "WAV: 65 bits per sample is out of range": base[:34] + struct.pack("<H", 65) + base[36:],
        "WAV: block align is zero": base[:32] + struct.pack("<H", 0) + base[34:],
        "WAV: extensible fmt chunk has a 10-byte extension, expected 22":
            make_wav("s16", 1, 16000, i16([1]), extensible=True).replace(struct.pack("<HH", 22, 16), struct.pack("<HH", 10, 16), 1),
        "WAV: 12-bit PCM frames do not split evenly over 2 channels": make_wav("s16", 2, 16000, i16([1, 2]), bits=12, block_align=3),
    }
    for reason, data in cases.items():
        with pytest.raises(W.WavError) as e:
            W.decode(data)
        assert str(e.value) == reason
        with pytest.raises(ge.GemmaEmbedError) as e:
            ge.decode_wav(data)
        assert e.value.message == "cannot decode audio: " + reason


# ---- the library against the oracle on seeded random files ---------------------------------------

def random_wav(rng):
    """A random, mostly valid file: any sample width 1-8 bytes (PCM) or float 32/64, 1-8
    channels, extensible or plain, extra and odd chunks, fmt extensions, overrunning or short
    data sizes, odd bit depths with their own block align, and cut at a random byte."""
    kind = rng.integers(0, 4)
    ch = int(rng.integers(1, 9))
    rate = int(rng.choice([8000, 11025, 16000, 22050, 44100, 48000, 96000, 384000]))
    if kind == 0:
        bps, tag = int(rng.integers(1, 9)), 1
    elif kind == 1:
        bps, tag = int(rng.choice([4, 8])), 3
    else:
        bps, tag = int(rng.choice([1, 2, 3, 4])), 1
    bits = bps * 8
    align = ch * bps
    if rng.random() < 0.15 and tag == 1:
        bits = bps * 8 - int(rng.integers(1, 8))  # 12-bit in 16, 20-bit in 24 ...
    frames = int(rng.integers(0, 300))
    payload = rng.integers(0, 256, frames * align, dtype=np.uint8).tobytes()
    if tag == 3 and bps == 4:
        payload = rng.uniform(-1.5, 1.5, frames * ch).astype("<f4").tobytes()
    extensible = rng.random() < 0.3
    fmt = struct.pack("<HHIIHH", 0xFFFE if extensible else tag, ch, rate, rate * align, align, bits)
    if extensible:
        fmt += struct.pack("<HHIH", 22, bits, 3, tag) + GUID_TAIL
    elif rng.random() < 0.3:
        ext = int(rng.integers(0, 6))
        fmt += struct.pack("<H", ext) + bytes(ext)
    chunks = []
    for _ in range(int(rng.integers(0, 3))):
        cid = [b"LIST", b"junk", b"fact", b"bext", b"cue "][int(rng.integers(0, 5))]
        chunks.append(chunk(cid, rng.integers(0, 256, int(rng.integers(0, 9)), dtype=np.uint8).tobytes()))
    declared = len(payload)
    r = rng.random()
    if r < 0.15:
        declared += int(rng.integers(1, 5000))
    elif r < 0.25:
        declared = max(0, declared - int(rng.integers(1, 7)))
    body = chunk(b"fmt ", fmt) + b"".join(chunks) + b"data" + struct.pack("<I", declared) + payload
    if rng.random() < 0.2:
        body += chunk(b"LIST", b"tail")
    data = b"RIFF" + struct.pack("<I", 4 + len(body)) + b"WAVE" + body
    if rng.random() < 0.15:
        data = data[:int(rng.integers(0, len(data) + 1))]
    return data


def test_library_equals_oracle_on_random_files(ge):
    rng = np.random.default_rng(20261202)
    decoded = refused = 0
    for i in range(1500):
        data = random_wav(rng)
        try:
            want = W.decode(data)
        except W.WavError as e:
            with pytest.raises(ge.GemmaEmbedError) as g:
                ge.decode_wav(data)
            assert g.value.message == "cannot decode audio: " + str(e), i
            refused += 1
            continue
        got = ge.decode_wav(data)
        assert (got[1], got[2]) == (want[1], want[2]), i
        assert np.array_equal(got[0].view(np.uint32), want[0].view(np.uint32)), i
        decoded += 1
    assert decoded > 1000 and refused > 20


def test_wide_pcm_sits_at_the_top_of_an_int64(ge):
    """5 to 8-byte PCM: the bytes fill an int64 from the top, then / (2^63 - 1) in double."""
    for bps in range(5, 9):
        vals = [(1 << (8 * bps - 1)) - 1, -(1 << (8 * bps - 1)), 1, -1, 12345678901 % (1 << (8 * bps - 1))]
        raw = b"".join(int(v).to_bytes(bps, "little", signed=True) for v in vals)
        data = make_wav("s16", 1, 16000, raw, bits=8 * bps, block_align=bps)
        x, _, _ = both(ge, data)
        want = [np.float32(float(np.int64(v << (64 - 8 * bps))) / 9223372036854775807.0) for v in vals]
        assert np.array_equal(x, np.array(want, np.float32)), bps


# ---- input forms (AudioDecoder.decode, Audio/AudioDecoder.swift:17-41) --------------------------

def lcg_noise(count, seed=1):
    """The reference tests' noise (AudioDecoderTests.swift:154-160): a 32-bit LCG as float / 2^31."""
    out = np.zeros(count, np.float32)
    s = seed
    for i in range(count):
        s = (1664525 * s + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(np.int32(np.uint32(s).view(np.int32))) / np.float32(2147483648.0)
    return out


def test_every_input_form_decodes_alike(ge, tmp_path):
    """testEveryInputFormDecodesAlike (AudioDecoderTests.swift:208-225)."""
    pcm = (lcg_noise(3002) * np.float32(32767)).astype(np.int16)  # Int16(Float) truncates toward zero
    data = make_wav("s16", 2, 22050, pcm.astype("<i2").tobytes())
    path = tmp_path / "clip.wav"
    path.write_bytes(data)
    from_url = ge.audio_to_mono16k(ge.AudioInput.url(path))
    from_data = ge.audio_to_mono16k(ge.AudioInput.data(data))
    x, rate, ch = ge.decode_wav(data)
    from_samples = ge.audio_to_mono16k(ge.AudioInput.samples(x, rate, ch))
    assert len(from_url) == 1089
    assert np.array_equal(from_url.view(np.uint32), from_data.view(np.uint32))
    assert np.array_equal(from_url.view(np.uint32), from_samples.view(np.uint32))
    assert np.array_equal(from_url.view(np.uint32), B.to_mono16k(*W.decode(data)[:1], rate, ch).view(np.uint32))
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.audio_to_mono16k(ge.AudioInput.data(b"not audio at all"))
    assert e.value.case == "audioDecoding"
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.audio_to_mono16k(ge.AudioInput.url("/nonexistent/clip.wav"))
    assert e.value.message == "cannot decode audio: /nonexistent/clip.wav is not readable"
    with pytest.raises(ge.GemmaEmbedError):
        ge.audio_to_mono16k(ge.AudioInput.samples(np.array([0.1, 0.2, 0.3], np.float32), 16000, 2))


def test_url_errors_name_the_path(ge, tmp_path):
    path = tmp_path / "bad.wav"
    path.write_bytes(b"RIFF" + struct.pack("<I", 4) + b"WAVE" + chunk(b"fmt ", bytes(16)))
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.audio_to_mono16k(ge.AudioInput.url(path))
    assert e.value.message == f"cannot decode audio: {path}: WAV: no data chunk"


def test_wav_with_no_frames_has_no_samples(ge):
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.audio_to_mono16k(ge.AudioInput.data(make_wav("s16", 1, 16000, b"")))
    assert e.value.message == "cannot decode audio: audio has no samples"


# ---- the reference's WAV fixtures ---------------------------------------------------------------

def sha(a: np.ndarray) -> str:
    return hashlib.sha256(a.astype("<f4").tobytes()).hexdigest()


def test_fixture_golden_is_consistent():
    """Each fixture's 16 kHz length is the resampled-length rule of its frames, and its rows plus
    the four frame rows are llama-server's prompt_tokens."""
    files = json.load(open(GOLDEN))["files"]
    assert len(files) == 29
    for f in files:
        assert B.frames_after_resampling(f["sample_rate"], f["frames"]) == f["mono16k"], f["file"]
        if f["prompt_tokens"] is not None:
            assert B.audio_token_count(f["mono16k"]) + 4 == f["prompt_tokens"], f["file"]


@pytest.mark.skipif(not os.path.isdir(FIXTURES), reason="the reference's WAV fixtures are not on this machine (set GE_REFERENCE to its checkout)")
def test_library_decodes_the_reference_fixtures(ge):
    files = json.load(open(GOLDEN))["files"]
    for f in files:
        data = open(os.path.join(FIXTURES, f["file"]), "rb").read()
        assert hashlib.sha256(data).hexdigest() == f["sha256"], f["file"]
        x, rate, ch = ge.decode_wav(data)
        assert (ch, rate, len(x) // ch) == (f["channels"], f["sample_rate"], f["frames"]), f["file"]
        assert sha(x) == f["samples_sha256"], f["file"]
        mono = ge.audio_to_mono16k(ge.AudioInput.data(data))
        assert len(mono) == f["mono16k"] and sha(mono) == f["mono16k_sha256"], f["file"]
