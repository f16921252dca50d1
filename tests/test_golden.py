"""The oracle and the product's host logic against the reference's own known answers."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_batches_known_answers_oracle(oracle):
    cases = json.load(open(os.path.join(GOLDEN, "batches.json")))["cases"]
    assert len(cases) == 6
    for c in cases:
        got = oracle.batches(c["costs"], c["batch_size"], c["budgets"])
        assert [list(r) for r in got] == c["ranges"], c


def test_batches_known_answers_product(ge):
    cases = json.load(open(os.path.join(GOLDEN, "batches.json")))["cases"]
    for c in cases:
        got = ge.EmbeddingModel.batches(c["costs"], c["batch_size"], c["budgets"])
        assert [[r.start, r.stop] for r in got] == c["ranges"], c


def test_batches_product_matches_oracle_random(ge, oracle):
    rng = np.random.default_rng(3)
    for _ in range(200):
        n = int(rng.integers(0, 40))
        k = int(rng.integers(1, 3))
        costs = rng.integers(0, 600, size=(n, k)).tolist()
        budgets = rng.integers(1, 2000, size=k).tolist()
        bs = None if rng.random() < 0.6 else int(rng.integers(1, 6))
        a = oracle.batches(costs, bs, budgets)
        b = ge.EmbeddingModel.batches(costs, bs, budgets)
        assert [list(r) for r in a] == [[r.start, r.stop] for r in b]
        # every range is non-empty and they tile [0, n)
        assert sum(r.stop - r.start for r in b) == n
        assert all(r.stop > r.start for r in b)


def test_q8_0_layout_matches_reference_gguf_directory(synth):
    """Byte sizes of Q8_0 (34 bytes per 32), BF16 and F32 tensors reproduce the offsets of the
    real embeddinggemma-2 GGUF directory, with 32-byte alignment (GGUFFile.swift:60-62)."""
    d = json.load(open(os.path.join(GOLDEN, "q8_layout.json")))
    ts = sorted(d["tensors"], key=lambda t: t["offset"])
    bytes_per = {"Q8_0": (32, 34), "F32": (1, 4), "BF16": (1, 2), "F16": (1, 2)}
    for a, b in zip(ts, ts[1:]):
        n = int(np.prod(a["shape_ne"]))
        blk, bb = bytes_per[a["type"]]
        size = n // blk * bb
        assert b["offset"] == (a["offset"] + size + 31) // 32 * 32, (a, b)
    assert len(ts) == d["tensor_count"]


def test_finish_matches_oracle(ge, oracle):
    rng = np.random.default_rng(1)
    for dims in (768, 512, 256, 128):
        v = rng.normal(size=768).astype(np.float32)
        for norm in (True, False):
            a = ge.EmbeddingModel.finish(v, dims, norm)
            b = oracle.finish(v, dims, norm)
            assert np.array_equal(a, b)
            if norm:
                assert abs(float(np.linalg.norm(a)) - 1) < 1e-5
    z = np.zeros(768, np.float32)
    assert np.array_equal(ge.EmbeddingModel.finish(z, 256, True), z[:256])
