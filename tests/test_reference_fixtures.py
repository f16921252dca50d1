"""The reference's own llama.cpp goldens for the text forward, on the CPU.

tests/golden/make_forward_golden.py extracts Tests/GemmaEmbedTests/Fixtures/{embeddings,
long_embeddings,activations}.jsonl.  They were computed with the real embeddinggemma-2-Q8_0.gguf,
which is not on this machine, so the two tests that run the oracle on them mirror the
reference's CPUReferenceTests (CPUReferenceTests.swift:39-89) and run only when
GEMMA_EMBED_WEIGHTS points at that file, as the reference's own tests do
(TestSupport.swift:20-25).  The first test checks, without weights, that the committed extracts
agree with each other and with the token fixtures.
"""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ACTIVATION_REL = 0.02   # CPUReferenceTests.swift:62: max(2 % of the llama.cpp sum, 0.5)
ACTIVATION_ABS = 0.5
EMBED_COSINE = 0.9995   # CPUReferenceTests.swift:86
EMBED_MAX_DIFF = 2e-3   # CPUReferenceTests.swift:87


def goldens():
    with open(os.path.join(GOLDEN, "reference_forward.json")) as f:
        fwd = json.load(f)
    vec = np.load(os.path.join(GOLDEN, "reference_vectors.npz"))
    with open(os.path.join(GOLDEN, "tokenizer_cases.json")) as f:
        tok = json.load(f)["reference_fixtures"]
    return fwd, vec, tok


def real_weights():
    path = os.environ.get("GEMMA_EMBED_WEIGHTS")
    if not path or not os.path.exists(path):
        pytest.skip("weights not found; set GEMMA_EMBED_WEIGHTS to the real embeddinggemma-2-Q8_0.gguf")
    return path


def normalised(v):
    v = np.asarray(v, np.float64)
    return v / np.linalg.norm(v)


def test_extracts_agree_with_each_other():
    fwd, vec, tok = goldens()
    emb = vec["embeddings"]
    assert emb.shape == (40, 768) and vec["long_embeddings"].shape == (3, 768)
    assert np.allclose(np.linalg.norm(emb, axis=1), 1.0, atol=1e-5)
    assert np.allclose(np.linalg.norm(vec["long_embeddings"], axis=1), 1.0, atol=1e-5)
    # llama-server's prompt sizes are the token fixtures' lengths
    assert fwd["embeddings"]["prompt_tokens"] == [len(t["token_ids"]) for t in tok]
    assert [r["prompt_tokens"] for r in fwd["long_embeddings"]] == [1054, 1629, 3222]
    acts = fwd["activations"]
    assert [a["i"] for a in acts] == [20, 21, 22]
    for a, final in zip(acts, vec["activation_embeddings"]):
        assert a["token_ids"] == tok[a["i"]]["token_ids"]
        assert len(a["sums"]) == a["n_tensors"] == 1149
        # llama-debug's final vector is llama-server's vector for the same ids
        assert np.abs(final - emb[a["i"]]).max() < 1e-6


def test_oracle_activation_sums_match_llama_cpp(oracle):
    """CPUReferenceTests.testActivationsMatchLlamaCpp: every tensor the oracle's trace names
    (llama.cpp's names) sums within max(2 %, 0.5) of llama.cpp's, more than 200 per text."""
    path = real_weights()
    fwd, _, tok = goldens()
    ref = oracle.OracleModel(path)
    try:
        for a in fwd["activations"]:
            ids = np.array(a["token_ids"], np.int32)
            assert a["token_ids"] == tok[a["i"]]["token_ids"]
            trace = {}
            ref.forward(ids, trace=trace)
            sums = {name: float(np.sum(v, dtype=np.float64)) for name, v in trace.items()}
            checked = 0
            for name, want in a["sums"]:
                if name not in sums:
                    continue
                tol = max(ACTIVATION_REL * abs(want), ACTIVATION_ABS)
                assert abs(sums[name] - want) <= tol, (a["i"], name, sums[name], want)
                checked += 1
            assert checked > 200, (a["i"], checked)
    finally:
        ref.close()


def test_oracle_embeddings_match_llama_cpp(oracle):
    """CPUReferenceTests.testEmbeddingsMatchReference: texts 20, 0 and 35 tokenised by the
    oracle's tokenizer (equal to the fixture ids), then cosine > 0.9995 and max abs diff < 2e-3
    against llama-server's normalised vectors."""
    path = real_weights()
    from oracle.tokenizer import Tokenizer

    _, vec, tok = goldens()
    tk = Tokenizer.from_gguf(path)
    ref = oracle.OracleModel(path)
    try:
        for i in (20, 0, 35):
            ids = tk.encode(tok[i]["input"])
            assert list(ids) == tok[i]["token_ids"], i
            got = normalised(ref.forward(np.array(ids, np.int32)))
            want = vec["embeddings"][i].astype(np.float64)
            assert float(got @ want) > EMBED_COSINE, i
            assert float(np.abs(got - want).max()) < EMBED_MAX_DIFF, i
    finally:
        ref.close()
