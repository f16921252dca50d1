"""Seeded synthetic weights and inputs for the EmbeddingGemma text encoder.

No real checkpoint ships with this project, so every test, the smoke run and the
benchmark use random-init weights written to a GGUF v3 file with the tensor
names, shapes and storage types the reference loader checks
(`Sources/GemmaEmbed/Model/Weights.swift:103-130`, metadata keys from
`Sources/GemmaEmbed/Model/ModelConfig.swift:54-112`).

Random numbers come from the reference test suite's `SeededRandom`
(splitmix64, `Tests/GemmaEmbedTests/KernelTests.swift:9-26`), vectorised with
numpy: the i-th draw (0-based) of `SeededRandom(seed)` is
`mix(seed + (i + 2) * 0x9E3779B97F4A7C15)`, and `floats(n, scale)` maps a draw
`r` to `(float(r >> 40) / 2**24 * 2 - 1) * scale` in float32.

Quantisation to Q8_0 follows ggml's reference rule (blocks of 32 along the
contiguous dimension, `d = amax / 127`, `q = roundf(x / d)` with the scale
stored as fp16), which the reference reads back in
`Sources/GemmaEmbed/Model/Weights.swift:33-41`.

Two architectures are described (both read by the same loader):

* ``"gemma-embedding"`` -- the measured shape: hidden 768, 24 layers, 3 query
  heads and 1 KV head of 256, GeGLU 1152, global attention every 6th layer,
  then mean-pool and a dense 768->3072->768 head (`dense_2.weight`,
  `dense_3.weight`).
* ``"gemma-embedding2"`` -- the reference's own EmbeddingGemma 2 shape
  (`Sources/GemmaEmbed/Model/Architecture.md:7-33`): hidden 512, 4 query heads,
  sliding layers 2 KV x 256, global layers 1 KV x 512, GeGLU 2048, per-layer
  inputs, and a per-token 512->768 output projection before the mean.
"""
from __future__ import annotations

import hashlib
import os
import struct
from dataclasses import dataclass, field

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_C1 = np.uint64(0xBF58476D1CE4E5B9)
_C2 = np.uint64(0x94D049BB133111EB)

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
VOCAB = 262144


# --------------------------------------------------------------------------- random
def _mix(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _C1
    z = (z ^ (z >> np.uint64(27))) * _C2
    return z ^ (z >> np.uint64(31))


def draws(seed: int, n: int, start: int = 0) -> np.ndarray:
    """Draws `start .. start+n-1` of `SeededRandom(seed).next()` as uint64."""
    with np.errstate(over="ignore"):
        i = np.arange(start, start + n, dtype=np.uint64)
        state = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + (i + np.uint64(2)) * GOLDEN
        return _mix(state)


def floats(seed: int, n: int, scale: float = 1.0, start: int = 0) -> np.ndarray:
    """`SeededRandom(seed).floats(n, scale)`: uniform in [-scale, scale) as float32."""
    r = (draws(seed, n, start) >> np.uint64(40)).astype(np.float32)
    return ((r / np.float32(1 << 24)) * np.float32(2) - np.float32(1)) * np.float32(scale)


class SeededRandom:
    """Scalar `SeededRandom` (splitmix64), for short draw sequences such as token ids."""

    def __init__(self, seed: int):
        self.state = (seed + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF

    def next(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        return z ^ (z >> 31)


# --------------------------------------------------------------------------- Q8_0
def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Rows of float32 `[rows][K]` (K % 32 == 0) to Q8_0 bytes `[rows][K/32*34]`."""
    rows, k = x.shape
    assert k % 32 == 0
    b = x.reshape(rows, k // 32, 32).astype(np.float32)
    amax = np.abs(b).max(axis=2)
    d = (amax / np.float32(127)).astype(np.float32)
    inv = np.where(d != 0, np.float32(1) / np.where(d != 0, d, np.float32(1)), np.float32(0)).astype(np.float32)
    v = b * inv[:, :, None]
    q = np.trunc(v + np.copysign(np.float32(0.5), v)).astype(np.int8)  # roundf: half away from zero
    out = np.empty((rows, k // 32, 34), dtype=np.uint8)
    out[:, :, 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, k // 32, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(rows, k // 32 * 34)


def dequantize_q8_0(raw: np.ndarray, k: int) -> np.ndarray:
    """Inverse of `quantize_q8_0`, exact in float32 (fp16 scale times int8)."""
    rows = raw.shape[0]
    blocks = raw.reshape(rows, k // 32, 34)
    d = blocks[:, :, 0:2].copy().view(np.float16).astype(np.float32)
    q = blocks[:, :, 2:].copy().view(np.int8).astype(np.float32)
    return (q * d).reshape(rows, k)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).view(np.uint32)
    rounded = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (rounded >> np.uint32(16)).astype(np.uint16)


# --------------------------------------------------------------------------- architectures
@dataclass
class Arch:
    name: str
    hidden: int
    layers: int
    heads: int
    head_dim_swa: int
    head_dim_global: int
    kv_swa: int
    kv_global: int
    ff: int
    per_layer: int            # 0: no per-layer inputs
    out_dim: int
    dense_head: int           # 0: no pooled dense head
    vocab: int = VOCAB
    sliding_window: int = 1024
    rope_swa: float = 1.0e4
    rope_global: float = 1.0e6
    eps: float = 1e-6
    global_every: int = 6

    def sliding(self, i: int) -> bool:
        return (i % self.global_every) != self.global_every - 1

    def kv(self, i: int) -> int:
        return self.kv_swa if self.sliding(i) else self.kv_global

    def hd(self, i: int) -> int:
        return self.head_dim_swa if self.sliding(i) else self.head_dim_global


ARCHS = {
    "gemma-embedding": dict(hidden=768, layers=24, heads=3, head_dim_swa=256, head_dim_global=256,
                            kv_swa=1, kv_global=1, ff=1152, per_layer=0, out_dim=768, dense_head=3072),
    "gemma-embedding2": dict(hidden=512, layers=24, heads=4, head_dim_swa=256, head_dim_global=512,
                             kv_swa=2, kv_global=1, ff=2048, per_layer=512, out_dim=768, dense_head=0),
}


def make_arch(name: str, layers: int | None = None, vocab: int | None = None) -> Arch:
    kw = dict(ARCHS[name])
    if layers is not None:
        kw["layers"] = layers
    if vocab is not None:
        kw["vocab"] = vocab
    return Arch(name=name, **kw)


@dataclass
class Tensor:
    name: str
    shape: list          # GGUF ne order: contiguous dimension first
    ggml_type: int
    data: bytes = field(repr=False, default=b"")


def _tensor_seed(seed: int, name: str) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little")


def _q8_tensor(name, cols, rows, seed, scale, chunk_rows=8192):
    parts = []
    s = _tensor_seed(seed, name)
    for r0 in range(0, rows, chunk_rows):
        r = min(chunk_rows, rows - r0)
        x = floats(s, r * cols, scale, start=r0 * cols).reshape(r, cols)
        parts.append(quantize_q8_0(x).tobytes())
    return Tensor(name, [cols, rows], GGML_Q8_0, b"".join(parts))


def _f32_tensor(name, n, seed, base, spread):
    x = np.float32(base) * (np.float32(1) + floats(_tensor_seed(seed, name), n, spread))
    return Tensor(name, [n], GGML_F32, x.astype(np.float32).tobytes())


def build_tensors(arch: Arch, seed: int) -> list:
    d, ff, pl = arch.hidden, arch.ff, arch.per_layer
    t = []
    # Embedding rows scaled so that x = row * sqrt(d) has entries of order 1.
    t.append(_q8_tensor("token_embd.weight", d, arch.vocab, seed, 0.06))
    if pl:
        name = "per_layer_model_proj.weight"
        x = floats(_tensor_seed(seed, name), pl * arch.layers * d, (3.0 / d) ** 0.5)
        t.append(Tensor(name, [d, pl * arch.layers], GGML_BF16, to_bf16_bits(x).tobytes()))
        t.append(_f32_tensor("per_layer_proj_norm.weight", pl, seed, 1.0, 0.1))
    for i in range(arch.layers):
        hd, kv = arch.hd(i), arch.kv(i)
        qd, kvd = arch.heads * hd, kv * hd
        p = f"blk.{i}."
        qk_w = hd ** -0.25   # keeps scale-1.0 logits of normed q and k of order 1
        t.append(_f32_tensor(p + "attn_norm.weight", d, seed, 1.0, 0.1))
        t.append(_q8_tensor(p + "attn_q.weight", d, qd, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "attn_k.weight", d, kvd, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "attn_v.weight", d, kvd, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "attn_output.weight", qd, d, seed, (3.0 / qd) ** 0.5))
        t.append(_f32_tensor(p + "attn_q_norm.weight", hd, seed, qk_w, 0.1))
        t.append(_f32_tensor(p + "attn_k_norm.weight", hd, seed, qk_w, 0.1))
        t.append(_f32_tensor(p + "post_attention_norm.weight", d, seed, 1.0, 0.1))
        t.append(_f32_tensor(p + "ffn_norm.weight", d, seed, 1.0, 0.1))
        t.append(_q8_tensor(p + "ffn_gate.weight", d, ff, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "ffn_up.weight", d, ff, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "ffn_down.weight", ff, d, seed, (3.0 / ff) ** 0.5))
        t.append(_f32_tensor(p + "post_ffw_norm.weight", d, seed, 1.0, 0.1))
        if pl:
            t.append(_q8_tensor(p + "inp_gate.weight", d, pl, seed, (3.0 / d) ** 0.5))
            t.append(_q8_tensor(p + "proj.weight", pl, d, seed, (3.0 / pl) ** 0.5))
            t.append(_f32_tensor(p + "post_norm.weight", d, seed, 1.0, 0.1))
            t.append(_f32_tensor(p + "layer_output_scale.weight", 1, seed, 0.9, 0.05))
    t.append(_f32_tensor("output_norm.weight", d, seed, 1.0, 0.1))
    if arch.per_layer:
        t.append(_q8_tensor("output.weight", d, arch.out_dim, seed, (3.0 / d) ** 0.5))
    if arch.dense_head:
        t.append(_q8_tensor("dense_2.weight", d, arch.dense_head, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor("dense_3.weight", arch.dense_head, arch.out_dim, seed, (3.0 / arch.dense_head) ** 0.5))
    return t


# --------------------------------------------------------------------------- tokenizer vocabulary
# A gemma4-style vocabulary for the synthetic files, laid out like the real one
# (Sources/GemmaEmbed/Tokenizer/Tokenizer.swift:30-32 token types): control and user-defined
# tokens first, unused slots, the 256 `<0xXX>` byte tokens, whole newline runs, then the
# pieces of a byte-pair encoding trained here on seeded synthetic prose, then unused filler up
# to the model's vocabulary size.  Spaces are U+2581 inside pieces, as in SentencePiece.
TOKEN_NORMAL, TOKEN_UNKNOWN, TOKEN_CONTROL, TOKEN_USER_DEFINED, TOKEN_UNUSED, TOKEN_BYTE = 1, 2, 3, 4, 5, 6
SPACE_MARK = "▁"
SPECIAL_TOKENS = [("<pad>", TOKEN_CONTROL), ("<eos>", TOKEN_CONTROL), ("<bos>", TOKEN_CONTROL),
                  ("<unk>", TOKEN_UNKNOWN), ("<mask>", TOKEN_USER_DEFINED), ("<start_of_turn>", TOKEN_CONTROL),
                  ("<end_of_turn>", TOKEN_CONTROL), ("<sep>", TOKEN_USER_DEFINED), ("<sep><sep>", TOKEN_USER_DEFINED),
                  # the frames of image and audio rows in a text sequence (Model/InputRow.swift:23-26)
                  ("<|image>", TOKEN_CONTROL), ("<image|>", TOKEN_CONTROL), ("<|audio>", TOKEN_CONTROL),
                  ("<audio|>", TOKEN_CONTROL)]
PAD_ID, EOS_ID, BOS_ID, UNK_ID = 0, 1, 2, 3
UNUSED_HEAD = 60
NEWLINE_RUNS = 31
TOKENIZER_MERGES = 3000
TRAIN_SEED = 20260
TRAIN_WORDS = 60000
LEXICON_SEED = 777
LEXICON_WORDS = 3000

_CONS = ["b", "c", "d", "f", "g", "h", "j", "k", "l", "m", "n", "p", "r", "s", "t", "v", "w", "z",
         "st", "tr", "pl", "ch", "sh", "th", "br", "gr", "qu"]
_VOWELS = ["a", "e", "i", "o", "u", "y", "ai", "ou", "ea", "io"]
_CODAS = ["", "", "", "n", "s", "r", "l", "t", "m", "nd", "st", "ng"]
_ACCENTED = "éèêàäôöüñøçå"
_CYRILLIC = "".join(chr(c) for c in range(0x430, 0x44A))
_SENTENCE_END = [".", ".", ".", "?", "!"]
_SEPARATORS = [(700, " "), (60, "  "), (140, "\n"), (70, "\n\n"), (20, "\n\n\n"), (10, "\t")]


def _lexicon() -> list:
    rng = SeededRandom(LEXICON_SEED)
    words = []
    for _ in range(LEXICON_WORDS):
        r = rng.next() % 100
        if r < 6:    # one to three characters of a 160-character CJK block (3-byte UTF-8)
            words.append("".join(chr(0x4E00 + rng.next() % 160) for _ in range(1 + rng.next() % 3)))
        elif r < 10:  # Cyrillic (2-byte UTF-8)
            words.append("".join(_CYRILLIC[rng.next() % len(_CYRILLIC)] for _ in range(2 + rng.next() % 6)))
        elif r < 13:  # numbers
            words.append(str(rng.next() % (10 ** (1 + rng.next() % 5))))
        else:
            w = "".join(_CONS[rng.next() % len(_CONS)] + _VOWELS[rng.next() % len(_VOWELS)]
                        for _ in range(1 + rng.next() % 3))
            w += _CODAS[rng.next() % len(_CODAS)]
            if rng.next() % 10 == 0:
                k = rng.next() % len(w)
                w = w[:k] + _ACCENTED[rng.next() % len(_ACCENTED)] + w[k + 1:]
            words.append(w)
    return words


_LEX_CACHE: list = []


def synthetic_text(seed: int, n_words: int, extra_chars: str = "") -> str:
    """Seeded prose over a fixed synthetic lexicon with Zipf word frequencies: sentences with
    capitals, commas, brackets and quotes, separated by single and double spaces, newline runs
    and tabs.  `extra_chars` are sprinkled after some words (characters outside the trained
    alphabet exercise the byte fallback)."""
    import bisect
    if not _LEX_CACHE:
        lex = _lexicon()
        cum, acc = [], 0.0
        for i in range(len(lex)):
            acc += 1.0 / (i + 1)
            cum.append(acc)
        _LEX_CACHE.extend([lex, cum])
    lex, cum = _LEX_CACHE
    rng = SeededRandom(seed)
    sep_total = sum(w for w, _ in _SEPARATORS)
    parts = []
    run, cap = 0, True
    for i in range(n_words):
        w = lex[min(bisect.bisect_left(cum, (rng.next() >> 11) / float(1 << 53) * cum[-1]), len(lex) - 1)]
        if cap and w[0].isalpha():
            w = w[0].upper() + w[1:]
        cap = False
        r = rng.next() % 1000
        if r < 60:
            w += ","
        elif r < 70:
            w = "(" + w + ")"
        elif r < 75:
            w = '"' + w + '"'
        elif r < 85 and extra_chars:
            w += extra_chars[rng.next() % len(extra_chars)]
        parts.append(w)
        run += 1
        if i == n_words - 1:
            break
        if run >= 4 and rng.next() % 10 == 0:
            parts.append(_SENTENCE_END[rng.next() % len(_SENTENCE_END)])
            run, cap = 0, True
            x = rng.next() % sep_total
            for weight, sep in _SEPARATORS:
                if x < weight:
                    parts.append(sep)
                    break
                x -= weight
        else:
            parts.append(" ")
    return "".join(parts)


def _training_words(text: str) -> dict:
    """Word counts for BPE training: newline runs dropped, each remaining segment cut before
    every run of U+2581, so a word is its leading space marks plus the text up to the next."""
    import re
    counts: dict = {}
    for seg in re.split("\n+", text.replace(" ", SPACE_MARK)):
        for w in re.findall(f"{SPACE_MARK}*[^{SPACE_MARK}]+|{SPACE_MARK}+$", seg):
            counts[w] = counts.get(w, 0) + 1
    return counts


def train_bpe(counts: dict, n_merges: int, min_char_count: int = 3):
    """Byte-pair training over word counts: the alphabet is every character seen at least
    `min_char_count` times (most frequent first, then by code point); each step merges the
    most frequent adjacent pair of known symbols (ties: the smaller pair of strings) until
    `n_merges` merges or no pair occurs twice.  Returns (alphabet, [(left, right), ...])."""
    import heapq
    char_count: dict = {}
    for w, c in counts.items():
        for ch in w:
            char_count[ch] = char_count.get(ch, 0) + c
    alphabet = sorted((ch for ch, c in char_count.items() if c >= min_char_count),
                      key=lambda ch: (-char_count[ch], ch))
    known = set(alphabet)
    keys = sorted(counts)
    words = [list(w) for w in keys]
    freq = [counts[w] for w in keys]
    pairs: dict = {}
    where: dict = {}

    def account(i, sign, touched):
        syms = words[i]
        for a, b in zip(syms, syms[1:]):
            if a in known and b in known:
                p = (a, b)
                pairs[p] = pairs.get(p, 0) + sign * freq[i]
                touched.add(p)
                if sign > 0:
                    where.setdefault(p, set()).add(i)

    touched: set = set()
    for i in range(len(words)):
        account(i, 1, touched)
    heap = [(-c, a, b) for (a, b), c in pairs.items() if c >= 2]
    heapq.heapify(heap)
    merges = []
    while heap and len(merges) < n_merges:
        negc, a, b = heapq.heappop(heap)
        if pairs.get((a, b), 0) != -negc:
            continue
        merged = a + b
        merges.append((a, b))
        known.add(merged)
        touched = set()
        for i in sorted(where.pop((a, b), ())):
            account(i, -1, touched)
            syms, out, k = words[i], [], 0
            while k < len(syms):
                if k + 1 < len(syms) and syms[k] == a and syms[k + 1] == b:
                    out.append(merged)
                    k += 2
                else:
                    out.append(syms[k])
                    k += 1
            words[i] = out
            account(i, 1, touched)
        pairs.pop((a, b), None)
        for p in sorted(touched):
            c = pairs.get(p, 0)
            if c >= 2 and p != (a, b):
                heapq.heappush(heap, (-c, p[0], p[1]))
    return alphabet, merges


_TRAINED: list = []


def trained_bpe():
    """The alphabet and merges every synthetic vocabulary shares (trained once per process)."""
    if not _TRAINED:
        text = synthetic_text(TRAIN_SEED, TRAIN_WORDS)
        _TRAINED.extend(train_bpe(_training_words(text), TOKENIZER_MERGES))
    return _TRAINED[0], _TRAINED[1]


def tokenizer_vocab(vocab_size: int):
    """(tokens, types, merges) of exactly `vocab_size` entries, or None when the trained
    vocabulary does not fit.  The trained part does not depend on `vocab_size`, so token ids
    agree across files of different sizes.  One trained piece is listed twice (the tokenizer
    maps a piece to its first id)."""
    alphabet, merges = trained_bpe()
    tokens, types, seen = [], [], set()

    def add(t, ty):
        tokens.append(t)
        types.append(ty)
        seen.add(t)

    for t, ty in SPECIAL_TOKENS:
        add(t, ty)
    for k in range(UNUSED_HEAD):
        add(f"<unused{k}>", TOKEN_UNUSED)
    for b in range(256):
        add(f"<0x{b:02X}>", TOKEN_BYTE)
    for k in range(1, NEWLINE_RUNS + 1):
        add("\n" * k, TOKEN_NORMAL)
    for ch in alphabet:
        if ch not in seen:
            add(ch, TOKEN_NORMAL)
    first = None
    for a, b in merges:
        if a + b not in seen:
            add(a + b, TOKEN_NORMAL)
            first = first or a + b
    add(first, TOKEN_NORMAL)
    if len(tokens) > vocab_size:
        return None
    k = UNUSED_HEAD
    while len(tokens) < vocab_size:
        add(f"<unused{k}>", TOKEN_UNUSED)
        k += 1
    return tokens, types, [f"{a} {b}" for a, b in merges]


def tokenizer_metadata(vocab_size: int, add_bos: bool = True, add_eos: bool = True):
    """GGUF key/value records of the synthetic gemma4 tokenizer, or None (see tokenizer_vocab)."""
    v = tokenizer_vocab(vocab_size)
    if v is None:
        return None
    tokens, types, merges = v

    def strings(xs):
        bs = [x.encode() for x in xs]
        return struct.pack("<IQ", 8, len(bs)) + b"".join(struct.pack("<Q", len(b)) + b for b in bs)

    return [
        _kv("tokenizer.ggml.model", 8, _str("gemma4")),
        _kv("tokenizer.ggml.tokens", 9, strings(tokens)),
        _kv("tokenizer.ggml.token_type", 9, struct.pack("<IQ", 5, len(types)) + np.array(types, np.int32).tobytes()),
        _kv("tokenizer.ggml.merges", 9, strings(merges)),
        _kv("tokenizer.ggml.bos_token_id", 4, struct.pack("<I", BOS_ID)),
        _kv("tokenizer.ggml.eos_token_id", 4, struct.pack("<I", EOS_ID)),
        _kv("tokenizer.ggml.padding_token_id", 4, struct.pack("<I", PAD_ID)),
        _kv("tokenizer.ggml.unknown_token_id", 4, struct.pack("<I", UNK_ID)),
        _kv("tokenizer.ggml.add_bos_token", 7, bytes([1 if add_bos else 0])),
        _kv("tokenizer.ggml.add_eos_token", 7, bytes([1 if add_eos else 0])),
    ]


# --------------------------------------------------------------------------- GGUF v3 writer
def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, payload: bytes) -> bytes:
    return _str(key) + struct.pack("<I", vtype) + payload


def metadata(arch: Arch) -> list:
    a = arch.name
    n = arch.layers
    kv = [
        _kv("general.architecture", 8, _str(a)),
        _kv("general.name", 8, _str(f"synthetic-{a}")),
        _kv("general.alignment", 4, struct.pack("<I", 32)),
        _kv(f"{a}.block_count", 4, struct.pack("<I", n)),
        _kv(f"{a}.embedding_length", 4, struct.pack("<I", arch.hidden)),
        _kv(f"{a}.embedding_length_out", 4, struct.pack("<I", arch.out_dim)),
        _kv(f"{a}.embedding_length_per_layer_input", 4, struct.pack("<I", arch.per_layer)),
        _kv(f"{a}.feed_forward_length", 4, struct.pack("<I", arch.ff)),
        _kv(f"{a}.attention.head_count", 4, struct.pack("<I", arch.heads)),
        _kv(f"{a}.attention.head_count_kv", 9,
            struct.pack("<IQ", 5, n) + np.array([arch.kv(i) for i in range(n)], dtype=np.int32).tobytes()),
        _kv(f"{a}.attention.sliding_window_pattern", 9,
            struct.pack("<IQ", 7, n) + bytes(1 if arch.sliding(i) else 0 for i in range(n))),
        _kv(f"{a}.attention.key_length", 4, struct.pack("<I", arch.head_dim_global)),
        _kv(f"{a}.attention.key_length_swa", 4, struct.pack("<I", arch.head_dim_swa)),
        _kv(f"{a}.attention.value_length", 4, struct.pack("<I", arch.head_dim_global)),
        _kv(f"{a}.attention.value_length_swa", 4, struct.pack("<I", arch.head_dim_swa)),
        _kv(f"{a}.attention.sliding_window", 4, struct.pack("<I", arch.sliding_window)),
        _kv(f"{a}.attention.layer_norm_rms_epsilon", 6, struct.pack("<f", arch.eps)),
        _kv(f"{a}.rope.freq_base", 6, struct.pack("<f", arch.rope_global)),
        _kv(f"{a}.rope.freq_base_swa", 6, struct.pack("<f", arch.rope_swa)),
    ]
    tok = tokenizer_metadata(arch.vocab)
    if tok is not None:
        return kv + tok
    # Too small a vocabulary for the trained pieces: placeholder tokens and no tokenizer model.
    toks = [f"<t{i}>".encode() for i in range(arch.vocab)]
    body = b"".join(struct.pack("<Q", len(s)) + s for s in toks)
    kv.append(_kv("tokenizer.ggml.bos_token_id", 4, struct.pack("<I", BOS_ID)))
    kv.append(_kv("tokenizer.ggml.eos_token_id", 4, struct.pack("<I", EOS_ID)))
    kv.append(_kv("tokenizer.ggml.tokens", 9, struct.pack("<IQ", 8, arch.vocab) + body))
    return kv


def write_gguf(path: str, arch: Arch, tensors: list, alignment: int = 32, kvs: list | None = None) -> None:
    """GGUF v3 with `arch`'s metadata (or the given key/value records) and `tensors`."""
    kvs = metadata(arch) if kvs is None else kvs
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kvs)) + b"".join(kvs)
    infos = []
    offset = 0
    offsets = []
    for t in tensors:
        offsets.append(offset)
        infos.append(_str(t.name) + struct.pack("<I", len(t.shape)) +
                     b"".join(struct.pack("<Q", s) for s in t.shape) +
                     struct.pack("<IQ", t.ggml_type, offset))
        offset += (len(t.data) + alignment - 1) // alignment * alignment
    header = head + b"".join(infos)
    pad = (-len(header)) % alignment
    tmp = path + f".tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(header + b"\0" * pad)
        for t, off in zip(tensors, offsets):
            f.write(t.data)
            f.write(b"\0" * ((-len(t.data)) % alignment))
    os.replace(tmp, path)


def cache_dir() -> str:
    d = os.environ.get("GE_SYNTH_CACHE") or os.path.join(os.environ.get("TMPDIR", "/tmp"), "gemma_embed_synth")
    os.makedirs(d, exist_ok=True)
    return d


FORMAT_VERSION = 3


def model_path(arch: str = "gemma-embedding", seed: int = 0, layers: int | None = None,
               vocab: int | None = None) -> str:
    """Path of the synthetic GGUF for (arch, seed, layers, vocab), written on first use."""
    a = make_arch(arch, layers, vocab)
    name = f"{arch}-s{seed}-l{a.layers}-v{a.vocab}-f{FORMAT_VERSION}.gguf"
    path = os.path.join(cache_dir(), name)
    if not os.path.exists(path):
        write_gguf(path, a, build_tensors(a, seed))
    return path


# --------------------------------------------------------------------------- image encoder (mmproj)
# A gemma4v image encoder file laid out like the real mmproj (tensor names, shapes, storage
# types and metadata keys of Tests/GemmaEmbedTests/Fixtures/mmproj.json, vision part), with the
# shapes of BASELINE config 4: 16 layers, hidden 768, 12 heads of 64, MLP 3072, 16x16 patches,
# projected to the text model's width.
VISION = dict(hidden=768, layers=16, heads=12, ff=3072, patch=16, positions=10240)


def vision_tensors(seed: int, projection_dim: int, hidden: int = 768, layers: int = 16, heads: int = 12,
                   ff: int = 3072, patch: int = 16, positions: int = 10240) -> list:
    d, hd, area = hidden, hidden // heads, patch * patch * 3
    t = []
    name = "v.patch_embd.weight"
    w = floats(_tensor_seed(seed, name), d * area, (3.0 / area) ** 0.5)
    t.append(Tensor(name, [patch, patch, 3, d], GGML_F32, w.astype(np.float32).tobytes()))
    name = "v.position_embd.weight"
    w = floats(_tensor_seed(seed, name), d * positions * 2, 0.5)
    t.append(Tensor(name, [d, positions, 2], GGML_F32, w.astype(np.float32).tobytes()))
    qk_w = hd ** -0.25
    for i in range(layers):
        p = f"v.blk.{i}."
        t.append(_f32_tensor(p + "ln1.weight", d, seed, 1.0, 0.1))
        t.append(_q8_tensor(p + "attn_q.weight", d, d, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "attn_k.weight", d, d, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "attn_v.weight", d, d, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "attn_out.weight", d, d, seed, (3.0 / d) ** 0.5))
        t.append(_f32_tensor(p + "attn_q_norm.weight", hd, seed, qk_w, 0.1))
        t.append(_f32_tensor(p + "attn_k_norm.weight", hd, seed, qk_w, 0.1))
        t.append(_f32_tensor(p + "attn_post_norm.weight", d, seed, 1.0, 0.1))
        t.append(_f32_tensor(p + "ln2.weight", d, seed, 1.0, 0.1))
        t.append(_q8_tensor(p + "ffn_gate.weight", d, ff, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "ffn_up.weight", d, ff, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "ffn_down.weight", ff, d, seed, (3.0 / ff) ** 0.5))
        t.append(_f32_tensor(p + "ffn_post_norm.weight", d, seed, 1.0, 0.1))
    t.append(_q8_tensor("mm.input_projection.weight", d, projection_dim, seed, (3.0 / d) ** 0.5))
    return t


def vision_metadata(projection_dim: int, hidden: int = 768, layers: int = 16, heads: int = 12, ff: int = 3072,
                    patch: int = 16, positions: int = 10240, eps: float = 1e-6) -> list:
    del positions  # carried by the position table's shape
    f3 = lambda v: struct.pack("<IQ", 6, 3) + np.array(v, np.float32).tobytes()
    u32 = lambda v: struct.pack("<I", v)
    return [
        _kv("general.architecture", 8, _str("clip")),
        _kv("general.type", 8, _str("mmproj")),
        _kv("general.name", 8, _str("synthetic-gemma4v")),
        _kv("general.alignment", 4, u32(32)),
        _kv("clip.has_vision_encoder", 7, b"\x01"),
        _kv("clip.vision.projection_dim", 4, u32(projection_dim)),
        _kv("clip.vision.image_size", 4, u32(224)),
        _kv("clip.vision.patch_size", 4, u32(patch)),
        _kv("clip.vision.embedding_length", 4, u32(hidden)),
        _kv("clip.vision.feed_forward_length", 4, u32(ff)),
        _kv("clip.vision.block_count", 4, u32(layers)),
        _kv("clip.vision.attention.head_count", 4, u32(heads)),
        _kv("clip.vision.image_mean", 9, f3([0.0, 0.0, 0.0])),
        _kv("clip.vision.image_std", 9, f3([1.0, 1.0, 1.0])),
        _kv("clip.vision.projector_type", 8, _str("gemma4v")),
        _kv("clip.vision.attention.layer_norm_epsilon", 6, struct.pack("<f", eps)),
    ]


def mmproj_path(seed: int = 0, projection_dim: int = 768, layers: int = VISION["layers"],
                positions: int = VISION["positions"]) -> str:
    """Path of the synthetic image encoder for (seed, projection width, layers), written on first use."""
    name = f"mmproj-gemma4v-s{seed}-p{projection_dim}-l{layers}-n{positions}-f{FORMAT_VERSION}.gguf"
    path = os.path.join(cache_dir(), name)
    if not os.path.exists(path):
        kw = dict(VISION, layers=layers, positions=positions)
        arch = Arch(name="clip", hidden=kw["hidden"], layers=layers, heads=kw["heads"], head_dim_swa=0,
                    head_dim_global=0, kv_swa=0, kv_global=0, ff=kw["ff"], per_layer=0, out_dim=0, dense_head=0)
        write_gguf(path, arch, vision_tensors(seed, projection_dim, **kw), kvs=vision_metadata(projection_dim, **kw))
    return path


def synthetic_images(count: int, seed: int, width: int = 768, height: int = 768) -> list:
    """RGB8 images (height x width x 3, uint8) with pixels uniform in 0..255 from SeededRandom(seed)."""
    out = []
    n = width * height * 3
    for i in range(count):
        r = draws(seed, n, start=i * n)
        out.append((r >> np.uint64(56)).astype(np.uint8).reshape(height, width, 3))
    return out


# --------------------------------------------------------------------------- audio encoder (mmproj)
# A gemma4a audio encoder file laid out like the audio part of the real mmproj (tensor names,
# shapes, storage types, clamp scalars and metadata keys of Tests/GemmaEmbedTests/Fixtures/
# mmproj.json), with the shapes of BASELINE config 5: 12 Conformer layers, hidden 1024, 8 heads
# of 128, FFN 4096, 128 mel bins, `a.pre_encode.out` 1024 -> 1536, projected to the text width.
AUDIO = dict(hidden=1024, layers=12, heads=8, ff=4096, mel=128, out_width=1536)
# The linears that carry `.input_min/.input_max/.output_min/.output_max` in the real file.
AUDIO_CLAMPED = ("ffn_up", "ffn_down", "attn_q", "attn_k", "attn_v", "attn_out", "conv_pw1", "conv_pw2",
                 "ffn_up_1", "ffn_down_1")
AUDIO_BOUNDS = dict(input_min=-2.5, input_max=2.5, output_min=-4.0, output_max=4.0)


def _scalar(name: str, value: float) -> "Tensor":
    return Tensor(name, [1], GGML_F32, np.array([value], np.float32).tobytes())


def _uniform_f32(name: str, shape: list, seed: int, scale: float) -> "Tensor":
    n = int(np.prod(shape))
    w = floats(_tensor_seed(seed, name), n, scale)
    return Tensor(name, shape, GGML_F32, w.astype(np.float32).tobytes())


def audio_tensors(seed: int, projection_dim: int, hidden: int = 1024, layers: int = 12, heads: int = 8,
                  ff: int = 4096, mel: int = 128, out_width: int = 1536) -> list:
    d, hd = hidden, hidden // heads
    t = []
    t.append(_uniform_f32("a.conv1d.0.weight", [3, 3, 1, 128], seed, (3.0 / 9) ** 0.5))
    t.append(_f32_tensor("a.conv1d.0.norm.weight", 128, seed, 1.0, 0.1))
    t.append(_uniform_f32("a.conv1d.1.weight", [3, 3, 128, 32], seed, (3.0 / 1152) ** 0.5))
    t.append(_f32_tensor("a.conv1d.1.norm.weight", 32, seed, 1.0, 0.1))
    sub = (mel // 4) * 32
    t.append(_uniform_f32("a.input_projection.weight", [sub, d], seed, (3.0 / sub) ** 0.5))
    for i in range(layers):
        p = f"a.blk.{i}."

        def lin(suffix, n_in, n_out):
            t.append(_q8_tensor(p + suffix + ".weight", n_in, n_out, seed, (3.0 / n_in) ** 0.5))
            if suffix in AUDIO_CLAMPED:
                for k, v in AUDIO_BOUNDS.items():
                    t.append(_scalar(p + suffix + "." + k, v))
        t.append(_f32_tensor(p + "ffn_norm.weight", d, seed, 1.0, 0.1))
        lin("ffn_up", d, ff)
        lin("ffn_down", ff, d)
        t.append(_f32_tensor(p + "ffn_post_norm.weight", d, seed, 1.0, 0.1))
        t.append(_f32_tensor(p + "attn_pre_norm.weight", d, seed, 1.0, 0.1))
        for s in ("attn_q", "attn_k", "attn_v", "attn_out", "attn_k_rel"):
            lin(s, d, d)
        t.append(_f32_tensor(p + "per_dim_scale.weight", hd, seed, 1.0, 0.2))
        t.append(_f32_tensor(p + "attn_post_norm.weight", d, seed, 1.0, 0.1))
        t.append(_f32_tensor(p + "conv_norm.weight", d, seed, 1.0, 0.1))
        lin("conv_pw1", d, 2 * d)
        t.append(_uniform_f32(p + "conv_dw.weight", [5, d], seed, 0.5))
        t.append(_f32_tensor(p + "norm_conv.weight", d, seed, 1.0, 0.1))
        lin("conv_pw2", d, d)
        t.append(_f32_tensor(p + "ffn_norm_1.weight", d, seed, 1.0, 0.1))
        lin("ffn_up_1", d, ff)
        lin("ffn_down_1", ff, d)
        t.append(_f32_tensor(p + "ffn_post_norm_1.weight", d, seed, 1.0, 0.1))
        t.append(_f32_tensor(p + "ln2.weight", d, seed, 1.0, 0.1))
    t.append(_q8_tensor("a.pre_encode.out.weight", d, out_width, seed, (3.0 / d) ** 0.5))
    t.append(_uniform_f32("a.pre_encode.out.bias", [out_width], seed, 0.1))
    t.append(_q8_tensor("mm.a.input_projection.weight", out_width, projection_dim, seed, (3.0 / out_width) ** 0.5))
    return t


def audio_metadata(projection_dim: int, hidden: int = 1024, layers: int = 12, heads: int = 8, ff: int = 4096,
                   mel: int = 128, out_width: int = 1536) -> list:
    del out_width  # carried by a.pre_encode.out's shape
    u32 = lambda v: struct.pack("<I", v)
    return [
        _kv("general.architecture", 8, _str("clip")),
        _kv("general.type", 8, _str("mmproj")),
        _kv("general.name", 8, _str("synthetic-gemma4a")),
        _kv("general.alignment", 4, u32(32)),
        _kv("clip.has_vision_encoder", 7, b"\x00"),
        _kv("clip.has_audio_encoder", 7, b"\x01"),
        _kv("clip.audio.projection_dim", 4, u32(projection_dim)),
        _kv("clip.audio.embedding_length", 4, u32(hidden)),
        _kv("clip.audio.feed_forward_length", 4, u32(ff)),
        _kv("clip.audio.block_count", 4, u32(layers)),
        _kv("clip.audio.attention.head_count", 4, u32(heads)),
        _kv("clip.audio.projector_type", 8, _str("gemma4a")),
        _kv("clip.audio.num_mel_bins", 4, u32(mel)),
        _kv("clip.audio.attention.layer_norm_epsilon", 6, struct.pack("<f", 1e-6)),
    ]


def audio_path(seed: int = 0, projection_dim: int = 768, layers: int = AUDIO["layers"], hidden: int = AUDIO["hidden"],
               heads: int = AUDIO["heads"], ff: int = AUDIO["ff"]) -> str:
    """Path of the synthetic audio encoder for (seed, projection width, shape), written on first use."""
    name = f"mmproj-gemma4a-s{seed}-p{projection_dim}-l{layers}-d{hidden}-h{heads}-f{ff}-v{FORMAT_VERSION}.gguf"
    path = os.path.join(cache_dir(), name)
    if not os.path.exists(path):
        kw = dict(AUDIO, layers=layers, hidden=hidden, heads=heads, ff=ff)
        arch = Arch(name="clip", hidden=hidden, layers=layers, heads=heads, head_dim_swa=0, head_dim_global=0,
                    kv_swa=0, kv_global=0, ff=ff, per_layer=0, out_dim=0, dense_head=0)
        write_gguf(path, arch, audio_tensors(seed, projection_dim, **kw), kvs=audio_metadata(projection_dim, **kw))
    return path


def synthetic_pcm(count: int, seconds: float, seed: int, rate: int = 16000) -> list:
    """Gaussian-noise PCM clips (float32 at `rate`, mono) with standard deviation 0.1 from SeededRandom(seed)."""
    n = int(round(seconds * rate))
    out = []
    for i in range(count):
        u = floats(seed, 2 * n, 1.0, start=i * 2 * n).astype(np.float64).reshape(2, n)
        u1 = np.clip((u[0] + 1.0) / 2.0, 1e-12, 1.0)
        g = np.sqrt(-2.0 * np.log(u1)) * np.cos(np.pi * u[1])
        out.append((0.1 * g).astype(np.float32))
    return out


# --------------------------------------------------------------------------- inputs
def config_sequences(config: int, seed: int = 0, vocab: int = VOCAB, scale_texts: int = 1) -> list:
    """Token-id sequences of a benchmark configuration, drawn from `SeededRandom(seed)`.

    config 1: 8 texts x 128 tokens.  config 2: 64 texts, lengths uniform in 32..512
    (lengths drawn first, then ids).  config 3: 16 x 2048 then 4 x 8192 tokens.
    config 4 (the metric's literal wording): 64 x 512.  Ids are `next() % vocab`.
    """
    rng = SeededRandom(seed)
    if config == 1:
        lens = [128] * 8
    elif config == 2:
        lens = [32 + rng.next() % 481 for _ in range(64 * scale_texts)]
    elif config == 3:
        lens = [2048] * 16 + [8192] * 4
    elif config == 4:
        lens = [512] * 64
    else:
        raise ValueError(f"unknown config {config}")
    return [np.array([rng.next() % vocab for _ in range(n)], dtype=np.int32) for n in lens]


def random_sequences(lengths, seed: int, vocab: int = VOCAB) -> list:
    rng = SeededRandom(seed)
    return [np.array([rng.next() % vocab for _ in range(n)], dtype=np.int32) for n in lengths]
