"""An independent implementation of the tokenizer's merge loop, used to pin the oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/ and tests/golden/make_tokenizer_golden.py.

The reference tokenizer's core (Sources/GemmaEmbed/Tokenizer/Tokenizer.swift:236-282) is
llama.cpp's byte-pair merge: lowest merge rank first, leftmost on ties, with `<0xXX>` byte
fallback.  The `tokenizers` library (Hugging Face, Rust; version printed by
`tokenizers.__version__`) implements the same rule in its `models.BPE` with
`byte_fallback=True`, written independently of both.  This module wraps it with the steps
that surround the merge loop in the reference -- spaces to U+2581 (205-210), newline runs
split from the rest (211-218) and a newline run that is a piece kept whole (236-240) -- so
that, on a vocabulary whose every merge joins two pieces into a third (what `models.BPE`
accepts), its ids are an outside check on `oracle.tokenizer.Tokenizer.encode`.
"""
from __future__ import annotations

import re

SPACE = "▁"


class HfBpe:
    def __init__(self, tokens, merges):
        from tokenizers import models
        self.vocab = {}
        for i, t in enumerate(tokens):
            self.vocab.setdefault(t, i)
        pairs = []
        for m in merges:
            left, right = m[:m.index(" ", 1)], m[m.index(" ", 1) + 1:]
            pairs.append((left, right))
        self.model = models.BPE(vocab=self.vocab, merges=pairs, byte_fallback=True)

    def encode_body(self, text: str) -> list:
        """Ids of `text` without BOS/EOS and without special-token parsing."""
        out = []
        esc = text.replace(" ", SPACE)
        for run in re.findall("\n+|[^\n]+", esc):
            if run[0] == "\n" and run in self.vocab:
                out.append(self.vocab[run])
            else:
                out.extend(t.id for t in self.model.tokenize(run))
        return out
