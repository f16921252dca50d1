"""EmbeddingModel.embed on strings (EmbeddingModel.swift:145-196) on the GPU: the library's
tokenizer and prepare step (task prefix, BOS/EOS, truncation keeping EOS) give the same ids
as the oracle tokenizer, so embedding the texts is bit-identical to embedding those ids, and
close to the CPU oracle's forward of them (EmbeddingModelTests' text-level checks)."""
import json
import os

import numpy as np
import pytest

from oracle.tokenizer import Tokenizer as OracleTokenizer

pytestmark = pytest.mark.gpu

COSINE_MIN = 0.99999
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tokenizer_cases.json")


def cosine(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def text_model(ge, synth, cuda_device):
    path = synth.model_path("gemma-embedding", seed=1, layers=6, vocab=4096)
    model = ge.EmbeddingModel.load(path)
    yield path, model, OracleTokenizer.from_gguf(path)
    model.close()


def texts():
    cases = json.load(open(GOLDEN))["cases"]
    picked = [c["text"] for c in cases if c["kind"] in ("edge", "reference-fixture-input")][:30]
    return picked + ["", "short", "a much longer query about gawy and stait"]


def prepare(orc, prefix, text, max_tokens, eos):
    ids = orc.encode(prefix + text)
    if len(ids) > max_tokens:
        return ids[: max_tokens - 1] + [eos], True
    return ids, False


@pytest.mark.parametrize("task,max_tokens,dims,normalise,batch_size", [
    ("document", 2048, 768, True, None),
    ("query", 64, 256, True, 3),
    ("none", 9, 128, False, None),
    ("similarity", 300, 512, True, 1),
])
def test_embed_texts_equals_embed_of_oracle_ids(ge, text_model, task, max_tokens, dims, normalise, batch_size):
    path, model, orc = text_model
    T = ge.TaskPrefix
    prefix = {"document": T.document(), "query": T.query("code search"), "none": T.none,
              "similarity": T.similarity}[task]
    opts = ge.EmbedOptions(task=prefix, max_tokens=max_tokens, dimensions=dims, normalise=normalise,
                           batch_size=batch_size)
    ts = texts()
    got = model.embed(ts, opts)
    prepared = [prepare(orc, prefix, t, max_tokens, model.info.eos_id) for t in ts]
    want = model.embed([p for p, _ in prepared], opts)
    assert len(got) == len(ts)
    for g, w, (ids, cut) in zip(got, want, prepared):
        assert g.token_count == len(ids) == w.token_count
        assert g.truncated == cut
        assert np.array_equal(g.vector, w.vector)
    if max_tokens == 9:
        assert any(g.truncated for g in got)


def test_text_embedding_matches_cpu_oracle(ge, oracle, text_model):
    path, model, orc = text_model
    ref = oracle.OracleModel(path)
    try:
        ts = ["the first document", "Тйппвн kaikiot 云 gawy, with é and 🙂", texts()[10]]
        got = model.embed(ts, ge.EmbedOptions(normalise=False))
        for t, g in zip(ts, got):
            ids = np.array(orc.encode(ge.TaskPrefix.document() + t), np.int32)
            c = cosine(g.vector, ref.forward(ids))
            assert c >= COSINE_MIN, (t, c)
    finally:
        ref.close()


def test_single_string_and_model_tokenizer(ge, text_model):
    path, model, orc = text_model
    one = model.embed("just one text")
    assert isinstance(one, ge.Embedding)
    assert one.token_count == len(orc.encode(ge.TaskPrefix.document() + "just one text"))
    assert abs(float(np.linalg.norm(one.vector)) - 1.0) < 1e-5
    tk = model.tokenizer
    standalone = ge.Tokenizer.load(path)
    for t in texts():
        assert tk.encode(t) == standalone.encode(t) == orc.encode(t)
    assert (tk.bos_id, tk.eos_id) == (model.info.bos_id, model.info.eos_id)
    assert model.embed([], ge.EmbedOptions()) == []


def test_text_entry_without_tokenizer(ge, synth, cuda_device, tmp_path):
    """A file without tokenizer.ggml.model loads for token ids; strings are refused."""
    arch = synth.make_arch("gemma-embedding", layers=1, vocab=4096)
    kvs = [r for r in synth.metadata(arch) if b"tokenizer.ggml.model" not in r[:40]]
    path = str(tmp_path / "no_tokenizer.gguf")
    synth.write_gguf(path, arch, synth.build_tensors(arch, 3), kvs=kvs)
    with ge.EmbeddingModel.load(path) as m:
        assert len(m.embed([2, 10, 11, 1]).vector) == 768
        with pytest.raises(ge.GemmaEmbedError) as e:
            m.embed("text")
        assert e.value.case == "unsupportedArchitecture"
        with pytest.raises(ge.GemmaEmbedError):
            m.tokenizer
