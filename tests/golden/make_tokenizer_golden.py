"""Regenerates tests/golden/tokenizer_cases.json.

* `cases`: texts and their ids under the synthetic gemma4 vocabulary of a 4096-entry file
  (gemma-embed-swift_b200/synthetic.py: tokenizer_vocab), computed by the Hugging Face
  `tokenizers` BPE model wrapped as oracle/hf_bpe.py describes -- an implementation written
  independently of the reference, the oracle and the library.  The texts are edge cases of
  the kinds Tests/GemmaEmbedTests/TokenizerTests.swift covers (empty input, spaces at both
  ends, tabs and newline runs, digits and symbols, accents, CJK, emoji with modifiers, right-
  to-left scripts, zero-width characters, a 3000-character run), seeded synthetic prose, the
  same texts behind the reference's task prefixes, and the inputs of the reference's token
  fixture file.
* `reference_fixtures`: Tests/GemmaEmbedTests/Fixtures/tokens.jsonl as the reference ships it
  (llama-tokenize ids under the real EmbeddingGemma vocabulary), for a run against the real
  weight file when one is available (GEMMA_EMBED_WEIGHTS).

Run here, where the reference checkout exists; the fixture travels with the repository and
the tests never read the reference at run time:
    python tests/golden/make_tokenizer_golden.py [reference root]
"""
import hashlib
import importlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GE_REFERENCE")
if not REF:
    sys.exit("usage: python make_tokenizer_golden.py <reference checkout> (or set GE_REFERENCE to its path)")

synth = importlib.import_module("gemma-embed-swift_b200.synthetic")
from oracle.hf_bpe import HfBpe  # noqa: E402

VOCAB = 4096
PREFIXES = ["title: none | text: ", "task: search result | query: ", "task: clustering | query: ",
            "task: classification | query: ", "task: sentence similarity | query: "]
EXTRA = "ΩλЖ🙂👍🏽🇦🇺ش्ह​﻿é"


def edge_texts():
    return [
        "", " ", "  ", "\n", "\n\n\n\n\n", "\n" * 40, "a\n\nb", " \n ",
        "   padded on both sides   ",
        "col1\tcol2\tcol3\nrow\n\n\nend",
        "digits 0123456789 and marks ~`!@#$%^&*()_+-=[]{}|;:'\",.<>/?",
        "accents: crème brûlée, naïve, façade, Ångström",
        "漢字かなカナ한글 mixed",
        "emoji \U0001F600\U0001F680 with a skin tone \U0001F44D\U0001F3FD and a flag \U0001F1E6\U0001F1FA",
        "right-to-left مرحبا and देवनागरी",
        "zero​width and ﻿mark",
        "literal ▁ marks ▁▁ inside",
        "<bos>not parsed<eos>",
        "<sep><sep><sep>",
        "a" * 3000,
        "gawy " * 200,
    ]


def random_scalar_texts(seed: int, n: int):
    """Strings of random scalars in U+0020..U+2FFF without U+2581 (the space mark, which
    decodes to a space), as the reference's round-trip test draws them."""
    rng = synth.SeededRandom(seed)
    out = []
    for _ in range(n):
        k = 1 + rng.next() % 40
        chars = []
        for _ in range(k):
            c = 0x20 + rng.next() % (0x3000 - 0x20)
            if c != 0x2581:
                chars.append(chr(c))
        out.append("".join(chars))
    return out


def main():
    tokens, types, merges = synth.tokenizer_vocab(VOCAB)
    digest = hashlib.sha256(json.dumps([tokens, types, merges], ensure_ascii=False).encode()).hexdigest()
    hf = HfBpe(tokens, merges)
    fixtures = [json.loads(line) for line in open(os.path.join(REF, "Tests/GemmaEmbedTests/Fixtures/tokens.jsonl"))]
    texts = [("edge", t) for t in edge_texts()]
    texts += [("synthetic", synth.synthetic_text(1000 + s, 20 + 37 * s, EXTRA)) for s in range(24)]
    texts += [("random-scalars", t) for t in random_scalar_texts(43, 20)]
    texts += [("prefixed", p + t) for p in PREFIXES for _, t in texts[:12:3]]
    seen = set()
    for f in fixtures:
        if f["input"] not in seen:
            seen.add(f["input"])
            texts.append(("reference-fixture-input", f["input"]))
    import tokenizers
    cases = [{"kind": k, "text": t, "body": hf.encode_body(t)} for k, t in texts]
    out = {
        "vocab_size": VOCAB,
        "vocab_sha256": digest,
        "bos_id": synth.BOS_ID, "eos_id": synth.EOS_ID,
        "generator": f"tokenizers {tokenizers.__version__} models.BPE(byte_fallback=True)",
        "cases": cases,
        "reference_fixtures": [{"i": f["i"], "input": f["input"], "token_ids": f["token_ids"]} for f in fixtures],
    }
    path = os.path.join(HERE, "tokenizer_cases.json")
    with open(path, "w") as fh:
        json.dump(out, fh, ensure_ascii=False, separators=(",", ":"))
        fh.write("\n")
    print(path, len(cases), "cases", os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
