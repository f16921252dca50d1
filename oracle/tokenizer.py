"""CPU restatement of the reference tokenizer, in plain Python.

TEST INFRASTRUCTURE ONLY: imported by tests/ and by tests/golden/make_tokenizer_golden.py as
the checker of the library's C++ tokenizer.  The product package never imports this module.

It follows Sources/GemmaEmbed/Tokenizer/Tokenizer.swift (the llama.cpp `gemma4` vocabulary
handling) step by step, on bytes:

* construction (Tokenizer.swift:57-98): piece -> first id; merges "left right" split at the
  first space after the first byte, first rank of a repeated pair kept; `<0xXX>` byte tokens
  of type 6; control (3), user-defined (4) and unknown (2) tokens as specials, longest first;
* encode (105-117): BOS if asked and flagged, special-token partition only when parsing
  specials (170-202), EOS if asked and flagged;
* encodeFragment (205-219): spaces to U+2581, then runs of newlines and runs of other bytes;
* encodeWord (236-282): a newline run that is a piece stays whole, else UTF-8 characters
  (284-291) merged lowest rank first, leftmost on ties (min-heap 293-327), a bigram discarded
  when either side changed length; symbols outside the vocabulary fall back to byte tokens;
* decode (120-147): control, unknown and unused tokens dropped, byte tokens reassembled,
  U+2581 back to a space.

`GgufMeta` reads the tokenizer keys of a GGUF v2/v3 file independently of the library's reader.
"""
from __future__ import annotations

import heapq
import struct

NORMAL, UNKNOWN, CONTROL, USER_DEFINED, UNUSED, BYTE = 1, 2, 3, 4, 5, 6
SPACE = b"\xe2\x96\x81"


def utf8_length(lead: int) -> int:
    """Tokenizer.swift:284-291."""
    if lead < 0x80:
        return 1
    if lead & 0xE0 == 0xC0:
        return 2
    if lead & 0xF0 == 0xE0:
        return 3
    if lead & 0xF8 == 0xF0:
        return 4
    return 1


class Tokenizer:
    def __init__(self, tokens, types, merges, bos_id, eos_id, pad_id=0, unknown_id=None,
                 add_bos=True, add_eos=False):
        """init(tokens:types:merges:...) (Tokenizer.swift:57-98); strings are UTF-8 bytes or str."""
        self.pieces = [t.encode() if isinstance(t, str) else bytes(t) for t in tokens]
        self.types = list(types)
        self.bos_id, self.eos_id, self.pad_id, self.unknown_id = bos_id, eos_id, pad_id, unknown_id
        self.add_bos, self.add_eos = add_bos, add_eos
        self.piece_to_id = {}
        for i, p in enumerate(self.pieces):
            self.piece_to_id.setdefault(p, i)
        self.merges = {}
        for rank, m in enumerate(merges):
            b = m.encode() if isinstance(m, str) else bytes(m)
            if len(b) <= 1:
                continue
            split = b.find(b" ", 1)
            if split < 0:
                continue
            self.merges.setdefault((b[:split], b[split + 1:]), rank)
        self.byte_to_id = [-1] * 256
        for v in range(256):
            i = self.piece_to_id.get(b"<0x%02X>" % v)
            if i is not None and self.types[i] == BYTE:
                self.byte_to_id[v] = i
        specials = [(i, self.pieces[i]) for i, t in enumerate(self.types) if t in (CONTROL, USER_DEFINED, UNKNOWN)]
        self.specials = sorted(specials, key=lambda s: -len(s[1]))  # stable: equal lengths keep id order

    @classmethod
    def from_gguf(cls, path: str) -> "Tokenizer":
        """Tokenizer(gguf:) (Tokenizer.swift:40-56)."""
        meta = GgufMeta(path)
        if meta.get("tokenizer.ggml.model") != b"gemma4":
            raise ValueError("unsupported tokenizer model")
        return cls(meta["tokenizer.ggml.tokens"], meta["tokenizer.ggml.token_type"], meta["tokenizer.ggml.merges"],
                   meta["tokenizer.ggml.bos_token_id"], meta["tokenizer.ggml.eos_token_id"],
                   meta.get("tokenizer.ggml.padding_token_id", 0), meta.get("tokenizer.ggml.unknown_token_id"),
                   meta.get("tokenizer.ggml.add_bos_token", True), meta.get("tokenizer.ggml.add_eos_token", False))

    # ------------------------------------------------------------------ encode
    def encode(self, text, add_special_tokens: bool = True, parse_special_tokens: bool = False) -> list:
        data = text.encode() if isinstance(text, str) else bytes(text)
        out = []
        if add_special_tokens and self.add_bos:
            out.append(self.bos_id)
        for frag in self._partition(data, parse_special_tokens):
            if isinstance(frag, int):
                out.append(frag)
            else:
                self._encode_fragment(data[frag[0]:frag[1]], out)
        if add_special_tokens and self.add_eos:
            out.append(self.eos_id)
        return out

    def _partition(self, data: bytes, parse_special: bool) -> list:
        frags = [(0, len(data))]
        if not parse_special:
            return frags
        for sid, sp in self.specials:
            if not sp:
                continue
            nxt = []
            for f in frags:
                if isinstance(f, int):
                    nxt.append(f)
                    continue
                start, end = f
                while True:
                    at = data.find(sp, start, end)
                    if at < 0:
                        break
                    if at > start:
                        nxt.append((start, at))
                    nxt.append(sid)
                    start = at + len(sp)
                if start < end:
                    nxt.append((start, end))
            frags = nxt
        return frags

    def _encode_fragment(self, frag: bytes, out: list) -> None:
        esc = frag.replace(b" ", SPACE)
        i = 0
        while i < len(esc):
            nl = esc[i] == 0x0A
            j = i + 1
            while j < len(esc) and (esc[j] == 0x0A) == nl:
                j += 1
            self._encode_word(esc[i:j], nl, out)
            i = j

    def _encode_word(self, word: bytes, all_newlines: bool, out: list) -> None:
        # symbols: [start, length, prev, next]
        if all_newlines and word in self.piece_to_id:
            syms = [[0, len(word), -1, -1]]
        else:
            syms, off = [], 0
            while off < len(word):
                ln = min(len(word) - off, utf8_length(word[off]))
                idx = len(syms)
                syms.append([off, ln, idx - 1, -1 if off + ln == len(word) else idx + 1])
                off += ln
        heap = []

        def push(left, right):
            if left < 0 or right < 0:
                return
            l, r = syms[left], syms[right]
            key = (word[l[0]:l[0] + l[1]], word[r[0]:r[0] + r[1]])
            rank = self.merges.get(key)
            if rank is None:
                return
            heapq.heappush(heap, (rank, left, right, l[1], r[1]))

        for i in range(1, len(syms)):
            push(i - 1, i)
        while heap:
            rank, left, right, ll, rl = heapq.heappop(heap)
            l, r = syms[left], syms[right]
            if l[1] == 0 or r[1] == 0 or l[1] != ll or r[1] != rl:
                continue
            l[1] += r[1]
            r[1] = 0
            l[3] = r[3]
            if r[3] >= 0:
                syms[r[3]][2] = left
            push(l[2], left)
            push(left, l[3])
        for s in syms:
            if s[1] == 0:
                continue
            piece = word[s[0]:s[0] + s[1]]
            i = self.piece_to_id.get(piece)
            if i is not None:
                out.append(i)
            else:
                for b in piece:
                    if self.byte_to_id[b] >= 0:
                        out.append(self.byte_to_id[b])

    # ------------------------------------------------------------------ decode
    def decode_bytes(self, ids) -> bytes:
        buf = bytearray()
        for i in ids:
            if not 0 <= i < len(self.pieces):
                continue
            t = self.types[i]
            if t in (CONTROL, UNKNOWN, UNUSED):
                continue
            p = self.pieces[i]
            if t == BYTE:
                v = _byte_value(p)
                buf += bytes([v]) if v is not None else p
            else:
                buf += p
        return bytes(buf).replace(SPACE, b" ")

    def decode(self, ids) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def piece(self, i: int):
        return self.pieces[i] if 0 <= i < len(self.pieces) else None

    def is_control(self, i: int) -> bool:
        return 0 <= i < len(self.types) and self.types[i] == CONTROL


def _byte_value(p: bytes):
    """byteValue(ofPiece:) (Tokenizer.swift:160-163)."""
    if len(p) != 6 or not p.startswith(b"<0x") or not p.endswith(b">"):
        return None
    try:
        return int(p[3:5], 16)
    except ValueError:
        return None


class GgufMeta(dict):
    """The metadata of a GGUF v2/v3 file: scalars as int/float/bool/bytes, arrays as lists."""

    _SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}

    def __init__(self, path: str):
        super().__init__()
        with open(path, "rb") as f:
            data = f.read(1 << 20)
            self._f, self._buf, self._pos = f, bytearray(data), 0
            if bytes(self._take(4)) != b"GGUF":
                raise ValueError("not a GGUF file")
            version, = struct.unpack("<I", self._take(4))
            if version not in (2, 3):
                raise ValueError("unsupported GGUF version")
            _, nkv = struct.unpack("<QQ", self._take(16))
            for _ in range(nkv):
                key = bytes(self._string()).decode()
                vtype, = struct.unpack("<I", self._take(4))
                self[key] = self._value(vtype)

    def _take(self, n: int):
        while self._pos + n > len(self._buf):
            more = self._f.read(1 << 20)
            if not more:
                raise ValueError("truncated GGUF header")
            self._buf += more
        b = self._buf[self._pos:self._pos + n]
        self._pos += n
        return b

    def _string(self):
        n, = struct.unpack("<Q", self._take(8))
        return self._take(n)

    def _value(self, vtype: int):
        if vtype == 8:
            return bytes(self._string())
        if vtype == 9:
            elem, count = struct.unpack("<IQ", self._take(12))
            return [self._value(elem) for _ in range(count)]
        fmt = self._SCALAR[vtype]
        v, = struct.unpack(fmt, self._take(struct.calcsize(fmt)))
        return v
