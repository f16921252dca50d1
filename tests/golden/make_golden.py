"""Regenerates the committed golden fixtures from the reference's own test sources.

Run here (where the reference checkout exists); the fixtures travel with the repository and
the tests never read the reference at run time.

* batches.json -- every `XCTAssertEqual(EmbeddingModel.batches(...), [...])` known answer of
  Tests/GemmaEmbedTests/EmbeddingModelTests.swift (testBatchPlanning).
* q8_layout.json -- name, shape, type and data offset of the real embeddinggemma-2 GGUF's
  tensors from Tests/GemmaEmbedTests/Fixtures/model.json, which pin the Q8_0 / BF16 / F32
  byte sizes and the 32-byte data alignment.
"""
import json
import os
import re
import sys

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GE_REFERENCE")
if not REF:
    sys.exit("usage: python make_golden.py <reference checkout> (or set GE_REFERENCE to its path)")
HERE = os.path.dirname(os.path.abspath(__file__))


def batches():
    src = open(os.path.join(REF, "Tests/GemmaEmbedTests/EmbeddingModelTests.swift")).read()
    pat = re.compile(r"XCTAssertEqual\(EmbeddingModel\.batches\((\[.*?\]), batchSize: (nil|\d+), budgets: (\[.*?\])\), (\[.*?\])\)")
    cases = []
    for costs, bs, budgets, want in pat.findall(src):
        ranges = [[int(a), int(b)] for a, b in re.findall(r"(\d+)\.\.<(\d+)", want)]
        cases.append({"costs": json.loads(costs), "batch_size": None if bs == "nil" else int(bs),
                      "budgets": json.loads(budgets), "ranges": ranges})
    return cases


def q8_layout():
    m = json.load(open(os.path.join(REF, "Tests/GemmaEmbedTests/Fixtures/model.json")))
    return {"tensors": [{k: t[k] for k in ("name", "shape_ne", "type", "offset")} for t in m["tensors"]],
            "bytes": m["bytes"], "tensor_count": m["tensor_count"]}


if __name__ == "__main__":
    b = batches()
    assert len(b) == 6, b
    json.dump({"source": "Tests/GemmaEmbedTests/EmbeddingModelTests.swift:101-109", "cases": b},
              open(os.path.join(HERE, "batches.json"), "w"), indent=1)
    json.dump({"source": "Tests/GemmaEmbedTests/Fixtures/model.json", **q8_layout()},
              open(os.path.join(HERE, "q8_layout.json"), "w"))
    print("wrote", len(b), "batch cases")
