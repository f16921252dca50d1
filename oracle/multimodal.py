"""CPU restatement of the reference's mixed-input sequence layout.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker of the library's layout
(csrc/multimodal.cpp).  The product package never imports this module.

MultimodalSequence.init (Sources/GemmaEmbed/MultimodalEmbedding.swift:43-83): the prefix joins the
first text or leads on its own; fixed rows = BOS + EOS + each span's rows and two frame tokens;
nil when those alone exceed max_tokens; text cut from the end, last text part first; ids
[bos] text [begin] -(r + 1)... [end] text ... [eos] with span rows numbered across the input.
"""
from __future__ import annotations


def sequence(prefix, parts, spans, max_tokens, bos, eos, encode):
    """parts: list of ("text", str) / ("image", None) / ("audio", None); spans: list of
    (rows, begin, end) for the non-text parts in order.  Returns (ids, truncated) or None."""
    parts = list(parts)
    if parts and parts[0][0] == "text":
        parts[0] = ("text", prefix + parts[0][1])
    else:
        parts.insert(0, ("text", prefix))
    texts = [encode(p[1]) if p[0] == "text" else None for p in parts]
    assert sum(t is None for t in texts) == len(spans)
    fixed = 2 + sum(rows + 2 for rows, _, _ in spans)
    if fixed > max_tokens:
        return None
    excess = fixed + sum(len(t) for t in texts if t is not None) - max_tokens
    truncated = excess > 0
    for i in reversed(range(len(texts))):
        if excess <= 0:
            break
        if texts[i] is None:
            continue
        cut = min(excess, len(texts[i]))
        texts[i] = texts[i][:len(texts[i]) - cut]
        excess -= cut
    ids, row, k = [bos], 0, 0
    for t in texts:
        if t is not None:
            ids += t
        else:
            rows, begin, end = spans[k]
            k += 1
            ids += [begin] + [-(r + 1) for r in range(row, row + rows)] + [end]
            row += rows
    ids.append(eos)
    return ids, truncated
