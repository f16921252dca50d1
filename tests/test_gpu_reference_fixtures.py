"""The reference's llama.cpp goldens for the whole text forward, on the GPU.

MetalForwardTests.testAllFixturesMatchReferenceEmbeddings (MetalForwardTests.swift:34-52) and
testLongTextsMatchLlamaCppBeyondTheWindow (MetalForwardTests.swift:220-238) restated for the CUDA
path: the 40 fixture texts in one packed batch and the three long texts (1054, 1629, 3222
tokens, past the 512-token half window) against llama-server's vectors at cosine > 0.9995.  The
vectors were computed with the real embeddinggemma-2-Q8_0.gguf, so these tests run only when
GEMMA_EMBED_WEIGHTS points at that file (TestSupport.swift:20-25); the extracts come from
tests/golden/make_forward_golden.py.
"""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
COSINE = 0.9995  # MetalForwardTests.swift:49 and :236


def real_weights():
    path = os.environ.get("GEMMA_EMBED_WEIGHTS")
    if not path or not os.path.exists(path):
        pytest.skip("weights not found; set GEMMA_EMBED_WEIGHTS to the real embeddinggemma-2-Q8_0.gguf")
    return path


def normalised(v):
    v = np.asarray(v, np.float64)
    return v / np.linalg.norm(v)


@pytest.fixture(scope="module")
def real_model(ge, cuda_device):
    path = real_weights()
    with ge.EmbeddingModel.load(path) as m:
        yield m


def test_all_fixtures_in_one_batch_match_llama_cpp(real_model, ge):
    with open(os.path.join(GOLDEN, "tokenizer_cases.json")) as f:
        tok = json.load(f)["reference_fixtures"]
    want = np.load(os.path.join(GOLDEN, "reference_vectors.npz"))["embeddings"]
    seqs = [np.array(t["token_ids"], np.int32) for t in tok]
    toks, pos, ranges = ge.pack(seqs)
    out = real_model.forward_packed(toks, pos, ranges)
    assert out.shape[0] == 40
    for i, (g, w) in enumerate(zip(out, want)):
        assert float(normalised(g) @ w.astype(np.float64)) > COSINE, i


def test_long_texts_match_llama_cpp_beyond_the_window(real_model, ge):
    with open(os.path.join(GOLDEN, "reference_forward.json")) as f:
        rows = json.load(f)["long_embeddings"]
    want = np.load(os.path.join(GOLDEN, "reference_vectors.npz"))["long_embeddings"]
    tk = real_model.tokenizer
    seqs = []
    for r in rows:
        ids = np.array(tk.encode(r["prefix"] + r["text"]), np.int32)
        assert len(ids) == r["prompt_tokens"]
        seqs.append(ids)
    toks, pos, ranges = ge.pack(seqs)
    out = real_model.forward_packed(toks, pos, ranges)
    for r, g, w in zip(rows, out, want):
        assert float(normalised(g) @ w.astype(np.float64)) > COSINE, r["prompt_tokens"]
