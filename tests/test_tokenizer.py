"""The tokenizer (Sources/GemmaEmbed/Tokenizer/Tokenizer.swift) on CPU: the oracle pinned to
golden ids from an independent BPE implementation, the library's C++ tokenizer against both,
and the behaviours Tests/GemmaEmbedTests/TokenizerTests.swift checks (special ids, control
text not parsed by default, round trips).  No GPU: the tokenizer loads from a GGUF file's
metadata alone."""
import json
import os
import struct
import threading

import numpy as np
import pytest

from oracle.tokenizer import Tokenizer as OracleTokenizer

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tokenizer_cases.json")


@pytest.fixture(scope="module")
def golden():
    return json.load(open(GOLDEN))


@pytest.fixture(scope="module")
def vocab_file(synth, tmp_path_factory):
    """A weightless GGUF carrying the 4096-entry synthetic gemma4 tokenizer."""
    arch = synth.make_arch("gemma-embedding", layers=1, vocab=4096)
    path = str(tmp_path_factory.mktemp("tok") / "vocab4096.gguf")
    synth.write_gguf(path, arch, [], kvs=synth.metadata(arch))
    return path


@pytest.fixture(scope="module")
def oracle_tok(vocab_file):
    return OracleTokenizer.from_gguf(vocab_file)


@pytest.fixture(scope="module")
def tok(ge, vocab_file):
    return ge.Tokenizer.load(vocab_file)


def test_golden_vocabulary_is_the_synthetic_one(synth, golden):
    import hashlib
    tokens, types, merges = synth.tokenizer_vocab(golden["vocab_size"])
    digest = hashlib.sha256(json.dumps([tokens, types, merges], ensure_ascii=False).encode()).hexdigest()
    assert digest == golden["vocab_sha256"]
    assert len(golden["cases"]) >= 100


def test_oracle_matches_golden(oracle_tok, golden):
    for c in golden["cases"]:
        assert oracle_tok.encode(c["text"], False) == c["body"], (c["kind"], c["text"][:60])
        assert oracle_tok.encode(c["text"]) == [golden["bos_id"]] + c["body"] + [golden["eos_id"]]


def test_oracle_matches_independent_bpe_on_fresh_texts(synth, oracle_tok):
    pytest.importorskip("tokenizers")
    from oracle.hf_bpe import HfBpe
    tokens, _, merges = synth.tokenizer_vocab(4096)
    hf = HfBpe(tokens, merges)
    for seed in range(40):
        t = synth.synthetic_text(5000 + seed, 30 + 11 * seed, "ΩλЖ🙂👍🏽ش्ह​é")
        assert oracle_tok.encode(t, False) == hf.encode_body(t), seed


def test_library_matches_golden(tok, golden):
    for c in golden["cases"]:
        assert tok.encode(c["text"], False) == c["body"], (c["kind"], c["text"][:60])
        assert tok.encode(c["text"]) == [golden["bos_id"]] + c["body"] + [golden["eos_id"]]


def test_library_matches_oracle_with_special_parsing(tok, oracle_tok, golden):
    texts = [c["text"] for c in golden["cases"][:60]]
    texts += ["<bos>hello", "a<eos>b<pad>", "<sep><sep><sep>", "<start_of_turn>user\nhi<end_of_turn>", "<mask>"]
    for t in texts:
        for add in (False, True):
            assert tok.encode(t, add, True) == oracle_tok.encode(t, add, True), t[:60]


def test_special_ids(tok):
    """TokenizerTests.testSpecialIds: BOS 2, EOS 1, pad 0; an empty text is [BOS, EOS]."""
    assert (tok.bos_id, tok.eos_id, tok.pad_id, tok.unknown_id) == (2, 1, 0, 3)
    assert tok.encode("", add_special_tokens=True) == [2, 1]
    assert tok.encode("", add_special_tokens=False) == []
    assert len(tok.encode("gawy", add_special_tokens=False)) == 1
    assert tok.vocabulary_size == 4096


def test_control_text_is_not_parsed_by_default(tok):
    """TokenizerTests.testControlTextIsNotParsedByDefault."""
    plain = tok.encode("<bos>hello", add_special_tokens=False)
    assert 2 not in plain
    parsed = tok.encode("<bos>hello", add_special_tokens=False, parse_special_tokens=True)
    assert parsed[0] == 2


def test_round_trip(tok, golden):
    """TokenizerTests.testRoundTrip: decode(encode(s)) == s, with and without BOS/EOS, for
    texts without U+2581 (which decodes to a space)."""
    texts = [c["text"] for c in golden["cases"] if "▁" not in c["text"]]
    assert len(texts) > 80
    for t in texts:
        assert tok.decode(tok.encode(t, False)) == t
        assert tok.decode(tok.encode(t)) == t


def test_decode_matches_oracle_on_random_ids(tok, oracle_tok):
    rng = np.random.default_rng(11)
    for _ in range(300):
        ids = rng.integers(-5, 4200, int(rng.integers(0, 60))).tolist()
        assert tok.decode_bytes(ids) == oracle_tok.decode_bytes(ids)


def test_piece_and_is_control(tok, oracle_tok):
    for i in list(range(0, 400)) + [4095]:
        assert tok.piece(i).encode() == oracle_tok.piece(i)
        assert tok.is_control(i) == oracle_tok.is_control(i)
    assert tok.piece(-1) is None and tok.piece(4096) is None
    assert not tok.is_control(-1) and not tok.is_control(1 << 20)


def test_concurrent_encode_is_consistent(tok, golden):
    texts = [c["text"] for c in golden["cases"]]
    want = [tok.encode(t) for t in texts]
    errors = []

    def run(k):
        for j in range(3):
            for i in range(k, len(texts), 4):
                if tok.encode(texts[i]) != want[i]:
                    errors.append(i)

    th = [threading.Thread(target=run, args=(k,)) for k in range(4)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert not errors


# ------------------------------------------------------------------ a hand-made vocabulary
def _edge_vocab():
    tokens = [("<pad>", 3), ("<eos>", 3), ("<bos>", 3), ("<unk>", 2), ("<ab>", 4), ("<abc>", 4), ("<x>", 4),
              ("<y>", 4), ("", 4)]
    for b in range(256):
        if b in (0x41, 0xF0):  # missing byte tokens: those bytes are dropped
            continue
        tokens.append(("<0x0a>" if b == 0x0A else f"<0x{b:02X}>", 6))  # a lower-case spelling
    tokens += [(t, 1) for t in ["a", "b", "c", "ab", "bc", "abc", "▁", "▁a", "\n", "\n\n", "é", "éa", "qr", "ab"]]
    tokens += [("<unused0>", 5), ("<0xZZ>", 6)]
    merges = ["a b", "b c", "ab c", "a b", "▁ a", "x y", "c", "c ", "\n \n", "é a", "q r", "bc a", " a b"]
    return tokens, merges


def _write_vocab(synth, path, tokens, merges, model="gemma4", drop=(), types_len=None, extra=()):
    def strings(xs):
        bs = [x.encode() for x in xs]
        return struct.pack("<IQ", 8, len(bs)) + b"".join(struct.pack("<Q", len(b)) + b for b in bs)

    types = [t for _, t in tokens][: types_len if types_len is not None else len(tokens)]
    kvs = [
        ("tokenizer.ggml.model", synth._kv("tokenizer.ggml.model", 8, synth._str(model))),
        ("tokenizer.ggml.tokens", synth._kv("tokenizer.ggml.tokens", 9, strings([t for t, _ in tokens]))),
        ("tokenizer.ggml.token_type", synth._kv("tokenizer.ggml.token_type", 9,
                                                struct.pack("<IQ", 5, len(types)) + np.array(types, np.int32).tobytes())),
        ("tokenizer.ggml.merges", synth._kv("tokenizer.ggml.merges", 9, strings(merges))),
        ("tokenizer.ggml.bos_token_id", synth._kv("tokenizer.ggml.bos_token_id", 4, struct.pack("<I", 2))),
        ("tokenizer.ggml.eos_token_id", synth._kv("tokenizer.ggml.eos_token_id", 4, struct.pack("<I", 1))),
        ("tokenizer.ggml.add_eos_token", synth._kv("tokenizer.ggml.add_eos_token", 7, b"\x01")),
    ] + list(extra)
    arch = synth.make_arch("gemma-embedding", layers=1, vocab=256)
    synth.write_gguf(path, arch, [], kvs=[r for k, r in kvs if k not in drop])


@pytest.fixture(scope="module", params=["words-split", "merges-cross-words"])
def edge_pair(ge, synth, tmp_path_factory, request):
    """The hand-made vocabulary, and a variant whose merges join a symbol to a following
    U+2581 (the library then cannot encode words separately)."""
    tokens, merges = _edge_vocab()
    if request.param == "merges-cross-words":
        tokens = tokens + [("b▁a", 1), ("c▁", 1), ("▁▁", 1)]
        merges = ["b ▁a", "▁ ▁", "c ▁"] + merges
    path = str(tmp_path_factory.mktemp("tok") / f"edge-{request.param}.gguf")
    _write_vocab(synth, path, tokens, merges)
    return ge.Tokenizer.load(path), OracleTokenizer.from_gguf(path)


def test_edge_vocabulary_matches_oracle(edge_pair):
    """Merges whose halves or result are not pieces, repeated merges (first rank wins),
    malformed merge lines, a repeated piece (first id wins), missing and lower-case byte
    tokens, specials that overlap or share a length, merges across word starts, and input
    that is not valid UTF-8."""
    lib, orc = edge_pair
    assert lib.unknown_id is None and orc.unknown_id is None
    alphabet = [b"a", b"b", b"c", b"x", b"y", b"q", b"r", b" ", b" ", b"\n", "é".encode(), b"<", b">", b"A",
                b"\xf0", b"\xff", b"\xc3", "▁".encode(), b"<ab>", b"<abc>", b"<x>", b"<y>", b" a", b"b a"]
    rng = np.random.default_rng(5)
    for _ in range(3000):
        s = b"".join(alphabet[int(i)] for i in rng.integers(0, len(alphabet), int(rng.integers(0, 24))))
        for add in (False, True):
            for ps in (False, True):
                assert lib.encode(s, add, ps) == orc.encode(s, add, ps), (s, add, ps)
    for _ in range(500):
        ids = rng.integers(-2, 290, int(rng.integers(0, 30))).tolist()
        assert lib.decode_bytes(ids) == orc.decode_bytes(ids)
    # Spot checks of the rules themselves.
    assert lib.encode("qr", False) == [orc.piece_to_id[b"qr"]]  # halves are no pieces, the result is
    assert lib.encode("xy", False) == [orc.piece_to_id[b"<0x78>"], orc.piece_to_id[b"<0x79>"]]  # result no piece
    assert lib.encode("A", False) == []  # no byte token for 0x41
    assert lib.encode("<abc>", False, True) == [5]  # the longer special first


def test_tokenizer_load_failures(ge, synth, tmp_path):
    tokens, merges = _edge_vocab()
    cases = [
        (dict(model="llama"), "unsupportedArchitecture"),
        (dict(drop=("tokenizer.ggml.model",)), "unsupportedArchitecture"),
        (dict(drop=("tokenizer.ggml.merges",)), "missingMetadata"),
        (dict(drop=("tokenizer.ggml.token_type",)), "missingMetadata"),
        (dict(drop=("tokenizer.ggml.bos_token_id",)), "missingMetadata"),
        (dict(types_len=10), "invalidGGUF"),
    ]
    for i, (kw, case) in enumerate(cases):
        p = str(tmp_path / f"bad{i}.gguf")
        _write_vocab(synth, p, tokens, merges, **kw)
        with pytest.raises(ge.GemmaEmbedError) as e:
            ge.Tokenizer.load(p)
        assert e.value.case == case, (kw, e.value)
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.Tokenizer.load(str(tmp_path / "absent.gguf"))
    assert e.value.case == "fileNotReadable"


def test_task_prefixes(ge):
    """TaskPrefix.prefix (EmbedOptions.swift:22-31)."""
    T = ge.TaskPrefix
    assert T.document() == "title: none | text: "
    assert T.document("A title") == "title: A title | text: "
    assert T.document("") == "title:  | text: "
    assert T.query() == "task: search result | query: "
    assert T.query("code retrieval") == "task: code retrieval | query: "
    assert T.prefix(T.CLUSTERING) == T.clustering == "task: clustering | query: "
    assert T.prefix(T.CLASSIFICATION) == T.classification == "task: classification | query: "
    assert T.prefix(T.SIMILARITY) == T.similarity == "task: sentence similarity | query: "
    assert T.prefix(T.NONE) == T.none == ""
    assert ge.EmbedOptions().task == T.document()
    with pytest.raises(ge.GemmaEmbedError):
        T.prefix(6)


def test_real_vocabulary_fixtures(ge, golden):
    """TokenizerTests.testFixturesMatchExactly: the reference's llama-tokenize ids, checked when
    the real EmbeddingGemma weight file is at GEMMA_EMBED_WEIGHTS (as the reference's test)."""
    path = os.environ.get("GEMMA_EMBED_WEIGHTS")
    if not path or not os.path.exists(path):
        pytest.skip("weights not found; set GEMMA_EMBED_WEIGHTS to the real EmbeddingGemma GGUF")
    tk = ge.Tokenizer.load(path)
    fixtures = golden["reference_fixtures"]
    assert len(fixtures) == 40
    for f in fixtures:
        assert tk.encode(f["input"]) == f["token_ids"], f["i"]
