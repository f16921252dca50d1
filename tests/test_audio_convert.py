"""Conversion of decoded PCM to 16 kHz mono (MiniaudioConverter, Audio/MiniaudioConverter.swift) on
CPU: the oracle against the reference's known answers (AudioDecoderTests.swift:163-206) and the
fixture clips' llama-server prompt sizes at other rates, against an independent float64
restatement (scipy's Butterworth sections and a numpy linear resampler), and the library's
ge_audio_convert (host code) against the oracle bit for bit."""
import json
import os

import numpy as np
import pytest

from oracle import binding as B

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "audio_counts.json")


def noise(n, seed=0):
    return np.random.default_rng(seed).uniform(-0.9, 0.9, n).astype(np.float32)


def test_resampled_length_known_answers():
    """testResampledLengthRule (AudioDecoderTests.swift:182-195)."""
    cases = [(16000, 5003, 5003), (44100, 13231, 4800), (8000, 2401, 4802), (48000, 14401, 4801),
             (11025, 3308, 4800), (22050, 6616, 4800), (96000, 28801, 4801), (32000, 9601, 4801), (44100, 0, 0)]
    for rate, frames, want in cases:
        assert B.frames_after_resampling(rate, frames) == want, (rate, frames)


def test_downmix_and_passthrough_known_answers():
    """testMono16kPassesThroughBitIdentical, testIdenticalStereoChannelsDownmixToThatChannel,
    testDownmixAveragesChannelsInOrder (AudioDecoderTests.swift:163-180)."""
    s = noise(5003)
    assert np.array_equal(B.to_mono16k(s, 16000).view(np.uint32), s.view(np.uint32))
    mono = noise(4001, 1)
    stereo = np.repeat(mono, 2)
    assert np.array_equal(B.to_mono16k(stereo, 16000, 2).view(np.uint32), mono.view(np.uint32))
    got = B.to_mono16k(np.array([0.5, -0.25, 1.0, 0.75, 0.75, 0.75], np.float32), 16000, 3)
    f = np.float32
    want = [((f(0.5) + f(-0.25)) + f(1.0)) / f(3), ((f(0.75) + f(0.75)) + f(0.75)) / f(3)]
    assert np.array_equal(got, np.array(want, np.float32))


def test_resampler_lengths_and_range():
    """testResamplerProducesTheDeclaredLengthAndNoNaN (AudioDecoderTests.swift:197-206)."""
    for rate in (8000, 11025, 22050, 32000, 44100, 48000, 96000):
        frames = rate * 3 // 10 + 1
        out = B.to_mono16k(noise(frames, rate), rate)
        assert len(out) == B.frames_after_resampling(rate, frames), rate
        assert not np.isnan(out).any() and np.abs(out).max() < 2, rate


def test_fixture_clips_at_other_rates_prompt_tokens():
    """llama-server's prompt_tokens for the fixture clips at 8, 22.05, 44.1 and 48 kHz: the clip's
    rows after resampling to 16 kHz, plus the four frame rows."""
    clips = json.load(open(GOLDEN))["clips"]
    checked = 0
    for c in clips:
        if c["sample_rate"] == 16000:
            continue
        frames = int(round(c["seconds"] * c["sample_rate"]))
        n = B.frames_after_resampling(c["sample_rate"], frames)
        assert B.audio_token_count(n) + 4 == c["prompt_tokens"], c["file"]
        checked += 1
    assert checked == 4


def _float64_restatement(x, rate):
    """An independent float64 restatement: scipy's 4th-order Butterworth low-pass (cut at half
    the lower rate, at the higher of the gcd-reduced rates) and linear interpolation on the
    resampler's fixed-point time grid."""
    from math import gcd
    from scipy import signal
    g = gcd(rate, 16000)
    rin, rout = rate // g, 16000 // g
    sos = signal.butter(4, (min(rin, rout) * 0.5) / (max(rin, rout) / 2), output="sos")
    n_out = B.frames_after_resampling(rate, len(x))
    xin = signal.sosfilt(sos, x.astype(np.float64)) if rin > rout else x.astype(np.float64)
    # output k interpolates between input frames i - 1 and i at fraction f, where the first
    # output sits at input frame 0 (x0 = 0 before the stream) and each step advances rin / rout.
    k = np.arange(n_out, dtype=np.int64)
    pos = k * rin
    i, f = pos // rout, (pos % rout) / rout
    prev = np.where(i >= 1, xin[np.clip(i - 1, 0, len(xin) - 1)], 0.0)
    cur = xin[np.clip(i, 0, len(xin) - 1)]
    y = prev + (cur - prev) * f
    valid = i < len(xin)
    y = np.where(valid, y, 0.0)
    if rin < rout:
        y = signal.sosfilt(sos, y)
    return y.astype(np.float32), valid


@pytest.mark.parametrize("rate", [8000, 22050, 44100, 48000])
def test_resampler_matches_float64_restatement(rate):
    x = (0.5 * np.sin(2 * np.pi * 440 * np.arange(rate) / rate) + 0.05 * noise(rate, 7)).astype(np.float32)
    got = B.to_mono16k(x, rate)
    want, valid = _float64_restatement(x, rate)
    assert got.shape == want.shape
    assert np.abs(got[valid] - want[valid]).max() < 2e-4, rate


@pytest.mark.parametrize("rate,channels,frames", [(16000, 2, 4001), (44100, 1, 13231), (8000, 2, 2401),
                                                  (48000, 4, 14401), (11025, 3, 3308), (22050, 2, 6616),
                                                  (96000, 1, 28801), (32000, 1, 9601), (16000, 1, 777)])
def test_library_conversion_equals_oracle(ge, rate, channels, frames):
    x = noise(frames * channels, rate + channels)
    got = ge.audio_to_mono16k(x, rate, channels)
    want = B.to_mono16k(x, rate, channels)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (rate, channels)


def test_library_conversion_refusals(ge):
    for bad in ((np.zeros(4, np.float32), 0, 1), (np.zeros(4, np.float32), 16000, 0),
                (np.zeros(0, np.float32), 16000, 1)):
        with pytest.raises(ge.GemmaEmbedError) as e:
            ge.audio_to_mono16k(*bad)
        assert e.value.case == "audioDecoding"
