"""Regenerates tests/golden/wav_fixtures.json from the reference's WAV fixtures
(Tests/GemmaEmbedTests/Fixtures/audio/**.wav, the clips behind Fixtures/audio/embeddings.jsonl).

Per file: its size and SHA-256, the format fields, the frame count, the SHA-256 of its samples
as float32 (little-endian, interleaved) and of its 16 kHz mono samples, and llama-server's
`prompt_tokens` for it.  The samples are decoded independently of the library: PCM files through
Python's stdlib `wave` reader with dr_wav's integer-to-float constants applied in numpy
(WAVDecoder.swift:132-173), IEEE float files by reading the canonical 44-byte header and copying
the float32 payload.  The 16 kHz samples come from the C oracle's MiniaudioConverter restatement
(oracle/logmel.c), which the CPU tests pin to the reference's converter known answers.  The WAV
files themselves stay in the reference checkout.

Run here, where the reference checkout exists:
    python tests/golden/make_wav_golden.py [reference root]
"""
import hashlib
import json
import os
import struct
import sys
import wave

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import binding as B  # noqa: E402

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GE_REFERENCE")
if not REF:
    sys.exit("usage: python make_wav_golden.py <reference checkout> (or set GE_REFERENCE to its path)")
FIX = os.path.join(REF, "Tests/GemmaEmbedTests/Fixtures/audio")


def stdlib_decode(data: bytes):
    """(float32 samples, channels, rate) without the library or the oracle's WAV reader."""
    tag = struct.unpack_from("<H", data, 20)[0]
    if tag == 3:  # IEEE float: canonical header, data chunk at byte 36
        assert data[36:40] == b"data"
        ch, rate = struct.unpack_from("<HI", data, 22)
        size = struct.unpack_from("<I", data, 40)[0]
        return np.frombuffer(data[44:44 + size], "<f4").astype(np.float32), ch, rate
    import io
    with wave.open(io.BytesIO(data)) as w:
        ch, width, rate, n = w.getnchannels(), w.getsampwidth(), w.getframerate(), w.getnframes()
        raw = np.frombuffer(w.readframes(n), np.uint8).reshape(-1, width)
    if width == 1:
        x = (raw[:, 0].astype(np.float32) * np.float32(0.00784313725490196078)) - np.float32(1)
    elif width == 2:
        x = raw.copy().view("<i2").reshape(-1).astype(np.float32) * np.float32(2.0 ** -15)
    elif width == 3:
        v = ((raw[:, 0].astype(np.int64) | (raw[:, 1].astype(np.int64) << 8) | (raw[:, 2].astype(np.int64) << 16)) ^ 0x800000) - 0x800000
        x = (v.astype(np.float64) * 2.0 ** -23).astype(np.float32)
    else:
        x = (raw.copy().view("<i4").reshape(-1).astype(np.float64) / 2.0 ** 31).astype(np.float32)
    return x, ch, rate


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


prompt = {}
with open(os.path.join(FIX, "embeddings.jsonl")) as f:
    for line in f:
        d = json.loads(line)
        prompt[d["file"]] = d["prompt_tokens"]
files = []
for sub in sorted(os.listdir(FIX)):
    d = os.path.join(FIX, sub)
    if not os.path.isdir(d):
        continue
    for name in sorted(os.listdir(d)):
        if not name.endswith(".wav"):
            continue
        rel = f"{sub}/{name}"
        data = open(os.path.join(d, name), "rb").read()
        x, ch, rate = stdlib_decode(data)
        mono = B.to_mono16k(x, rate, ch)
        files.append({"file": rel, "bytes": len(data), "sha256": sha(data), "sample_rate": rate, "channels": ch,
                      "frames": len(x) // ch, "samples_sha256": sha(x.astype("<f4").tobytes()),
                      "mono16k": len(mono), "mono16k_sha256": sha(mono.astype("<f4").tobytes()),
                      "prompt_tokens": prompt.get(rel)})
with open(os.path.join(HERE, "wav_fixtures.json"), "w") as f:
    json.dump({"source": "Tests/GemmaEmbedTests/Fixtures/audio (WAV files and embeddings.jsonl)", "files": files},
              f, indent=1)
print(f"{len(files)} files")
