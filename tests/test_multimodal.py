"""The mixed-input sequence layout (MultimodalSequence, MultimodalEmbedding.swift:43-83) on CPU:
the library's layout against the reference's own known answers
(Tests/GemmaEmbedTests/MultimodalSequenceTests.swift, one id per Unicode scalar standing in for
the tokenizer) and against the oracle's restatement on random inputs."""
import ctypes
from importlib import import_module

import numpy as np
import pytest

from oracle import multimodal as om

IMG, AUD = (900, 901), (800, 801)


def ids(text):
    return [ord(c) for c in text]


def layout(prefix, parts, rows, max_tokens=100):
    """parts: str for text, "I" / "A" objects for image / audio spans (rows in order)."""
    m = import_module("gemma-embed-swift_b200._lib")
    L = m.lib()
    kinds, texts = [], []
    for p in parts:
        if isinstance(p, str):
            kinds.append(0)
            texts.append(p.encode())
        else:
            kinds.append(1 if p is Image else 2)
            texts.append(None)
    n = len(parts)
    k = (ctypes.c_int32 * max(n, 1))(*kinds)
    t = (ctypes.c_char_p * max(n, 1))(*texts)
    r = (ctypes.c_int32 * max(len(rows), 1))(*rows)
    cap = 4096
    out = (ctypes.c_int32 * cap)()
    cnt, tr = ctypes.c_int32(0), ctypes.c_int32(0)
    rc = L.ge_test_multimodal_sequence(prefix.encode(), k, t, n, r, max_tokens, 2, 1, IMG[0], IMG[1], AUD[0], AUD[1],
                                       out, cap, ctypes.byref(cnt), ctypes.byref(tr))
    if rc != 0:
        return None
    return list(out[:cnt.value]), bool(tr.value)


class Image:
    pass


class Audio:
    pass


def test_audio_spans_use_their_own_frame_and_share_row_numbering():
    got, _ = layout("P:", ["a", Image, Audio, "b"], [2, 3])
    assert got == [2] + ids("P:a") + [900, -1, -2, 901, 800, -3, -4, -5, 801] + ids("b") + [1]


def test_lays_out_parts_in_order_inside_image_frames():
    got, cut = layout("P:", ["ab", Image, "c", Image], [2, 3])
    assert got == [2] + ids("P:ab") + [900, -1, -2, 901] + ids("c") + [900, -3, -4, -5, 901, 1]
    assert not cut


def test_prefix_leads_an_input_that_opens_with_an_image():
    got, _ = layout("P", [Image, "a"], [1])
    assert got == [2] + ids("P") + [900, -1, 901] + ids("a") + [1]


def test_truncation_cuts_text_from_the_end_and_keeps_frames():
    got, cut = layout("", ["abcd", Image, "xyz"], [2], max_tokens=9)
    assert got == [2] + ids("abc") + [900, -1, -2, 901, 1]
    assert cut


def test_images_that_alone_overflow_are_refused():
    fits, cut = layout("P", ["a", Image], [5], max_tokens=9)
    assert fits == [2, 900, -1, -2, -3, -4, -5, 901, 1]
    assert cut
    assert layout("P", ["a", Image], [5], max_tokens=8) is None


def test_empty_input_is_the_prefix_alone():
    assert layout("P", [], [])[0] == [2] + ids("P") + [1]
    assert layout("", [], [])[0] == [2, 1]


def test_matches_oracle_on_random_inputs():
    rng = np.random.default_rng(4)
    for _ in range(400):
        parts, rows, oparts, spans = [], [], [], []
        for _ in range(int(rng.integers(0, 6))):
            r = rng.random()
            if r < 0.5:
                t = "".join(chr(int(c)) for c in rng.integers(0x61, 0x7b, int(rng.integers(0, 12))))
                parts.append(t)
                oparts.append(("text", t))
            else:
                kind = Image if r < 0.8 else Audio
                n = int(rng.integers(1, 8))
                parts.append(kind)
                rows.append(n)
                oparts.append(("image" if kind is Image else "audio", None))
                spans.append((n,) + (IMG if kind is Image else AUD))
        prefix = "".join(chr(int(c)) for c in rng.integers(0x41, 0x5b, int(rng.integers(0, 4))))
        mt = int(rng.integers(2, 40))
        want = om.sequence(prefix, oparts, spans, mt, 2, 1, ids)
        got = layout(prefix, parts, rows, max_tokens=mt)
        assert got == (None if want is None else (want[0], want[1])), (prefix, parts, rows, mt)
