"""Extracts the reference's text-forward golden fixtures into tests/golden/.

The reference pins its forward against llama.cpp with three fixture files under
Tests/GemmaEmbedTests/Fixtures/, all computed with the real embeddinggemma-2-Q8_0.gguf:

* embeddings.jsonl -- 40 L2-normalised llama-server vectors, one per text of tokens.jsonl
  (MetalForwardTests.swift:34-52 at cosine > 0.9995; CPUReferenceTests.swift:73-89 for texts
  20, 0, 35 at cosine > 0.9995 and max abs diff < 2e-3);
* long_embeddings.jsonl -- three long texts (1054, 1629, 3222 tokens) with their prefix and
  vectors (MetalForwardTests.swift:220-238, cosine > 0.9995);
* activations.jsonl -- for texts 20..22, the token ids, llama-debug's final vector and the sum
  of every named tensor of the graph (CPUReferenceTests.swift:39-71: each sum the oracle's trace
  also names within max(2 %, 0.5), more than 200 per text).

Written here:
* reference_vectors.npz -- float32 arrays `embeddings` [40][768], `long_embeddings` [3][768],
  `activation_embeddings` [3][768];
* reference_forward.json -- token counts, the long texts with their prefix, and per activation
  text its input, token ids and (name, sum) pairs in the file's order.

Run where the reference checkout exists:  python make_forward_golden.py <reference checkout>
(or set GE_REFERENCE).  The tests read only the files written here.
"""
import json
import os
import sys

import numpy as np

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GE_REFERENCE")
if not REF:
    sys.exit("usage: python make_forward_golden.py <reference checkout> (or set GE_REFERENCE to its path)")
FIX = os.path.join(REF, "Tests/GemmaEmbedTests/Fixtures")
HERE = os.path.dirname(os.path.abspath(__file__))


def lines(name):
    with open(os.path.join(FIX, name)) as f:
        return [json.loads(l) for l in f if l.strip()]


def main():
    emb = lines("embeddings.jsonl")
    assert [r["i"] for r in emb] == list(range(40))
    long = lines("long_embeddings.jsonl")
    assert len(long) == 3
    acts = lines("activations.jsonl")
    meta = {r["i"]: r for r in acts if r.get("record") == "meta"}
    sums = {}
    for r in acts:
        if r.get("record") == "tensor":
            sums.setdefault(r["i"], []).append([r["name"], r["sum"]])
    texts = sorted(meta)
    np.savez_compressed(
        os.path.join(HERE, "reference_vectors.npz"),
        embeddings=np.array([r["embedding"] for r in emb], np.float32),
        long_embeddings=np.array([r["embedding"] for r in long], np.float32),
        activation_embeddings=np.array([meta[i]["final_embedding_l2"] for i in texts], np.float32))
    out = {
        "source": "Tests/GemmaEmbedTests/Fixtures/{embeddings,long_embeddings,activations}.jsonl",
        "weights": "embeddinggemma-2-Q8_0.gguf (README.md:16); absent here, so the tests that use "
                   "these fixtures run only when GEMMA_EMBED_WEIGHTS points at it",
        "embeddings": {"prompt_tokens": [r["prompt_tokens"] for r in emb], "tool": emb[0]["server_model"]},
        "long_embeddings": [{"prefix": r["prefix"], "text": r["text"], "prompt_tokens": r["prompt_tokens"],
                             "source": r["source"]} for r in long],
        "activations": [{"i": i, "input": meta[i]["input"], "token_ids": meta[i]["token_ids"],
                         "n_tensors": meta[i]["n_tensors"], "tool": meta[i]["tool"], "sums": sums[i]}
                        for i in texts],
    }
    with open(os.path.join(HERE, "reference_forward.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print("wrote", len(emb), "embeddings,", len(long), "long texts,", sum(len(v) for v in sums.values()),
          "tensor sums for texts", texts)


if __name__ == "__main__":
    main()
