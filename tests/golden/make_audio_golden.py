"""Regenerates tests/golden/audio_counts.json from the reference's audio fixtures.

* `clips`: every clip of Tests/GemmaEmbedTests/Fixtures/audio/embeddings.jsonl with its length,
  sample rate, channel count and llama-server's `prompt_tokens` (the clip's rows plus the four
  frame rows `bos`, `<|audio>`, `<audio|>`, `eos`, AudioEmbedding.swift:5-6).  The embedding
  vectors are left out: they need the real weight files.
* `counts`: the frame and token counts of AudioPreprocessingTests.testFrameAndTokenCounts and
  testChunking (Tests/GemmaEmbedTests/AudioPreprocessingTests.swift:8-33), transcribed.

Run here, where the reference checkout exists; the fixture travels with the repository:
    python tests/golden/make_audio_golden.py [reference root]
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GE_REFERENCE")
if not REF:
    sys.exit("usage: python make_audio_golden.py <reference checkout> (or set GE_REFERENCE to its path)")
SRC = os.path.join(REF, "Tests/GemmaEmbedTests/Fixtures/audio/embeddings.jsonl")

clips = []
with open(SRC) as f:
    for line in f:
        d = json.loads(line)
        clips.append({k: d[k] for k in ("file", "kind", "seconds", "sample_rate", "channels", "format",
                                        "prompt_tokens")})
counts = {
    "frame_count": [[4800, 29], [160, 1], [2, 1], [1, 0]],
    "token_count": [[4800, 8], [16000, 25], [480000, 750], [560000, 875]],
    "chunking": {"samples": 496000, "frames": [2999, 99], "tokens": [750, 25], "total": 775},
    "minimum_samples": 2,
}
with open(os.path.join(HERE, "audio_counts.json"), "w") as f:
    json.dump({"source": "Tests/GemmaEmbedTests/Fixtures/audio/embeddings.jsonl and "
                         "Tests/GemmaEmbedTests/AudioPreprocessingTests.swift:8-33",
               "clips": clips, "counts": counts}, f, indent=1)
print(f"{len(clips)} clips")
