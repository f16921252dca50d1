"""Host logic of the library on CPU (no GPU): the C ABI's exported symbols, the multi-GPU
dispatcher's split of a packed batch, the attention kernel's work schedule and batch packing
(PackedBatch.append, MetalForward.swift:8-21)."""
import ctypes
import importlib
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in ("gemma_embed.h", "gemma_embed_testing.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        names += re.findall(r"GE_API\s+[\w\s\*]+?\b(ge_\w+)\s*\(", text)
    return names


def test_c_abi_exports_every_declared_function(ge):
    lib_mod = importlib.import_module("gemma-embed-swift_b200._lib")
    raw = ctypes.CDLL(lib_mod.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(raw, n), n
    bound = set(lib_mod.SIGNATURES) | set(lib_mod.TEST_SIGNATURES)
    assert bound == set(names), (bound ^ set(names))


def seq_array(lib_mod, lens):
    arr = (lib_mod.GeSeq * max(len(lens), 1))()
    start = 0
    for i, n in enumerate(lens):
        arr[i].start = start
        arr[i].length = n
        start += n
    return arr


def shard_restated(lens, ndev):
    """The dispatcher's rule: longest first (stable) onto the least-loaded device (lowest
    index on ties), cost n + n^2 / 2048."""
    order = sorted(range(len(lens)), key=lambda i: -lens[i])
    load = [0.0] * ndev
    dev = [0] * len(lens)
    for i in order:
        d = min(range(ndev), key=lambda k: (load[k], k))
        load[d] += lens[i] + lens[i] * lens[i] / 2048.0
        dev[i] = d
    return dev


@pytest.mark.parametrize("ndev", [1, 2, 3, 8])
def test_dispatcher_split(ge, ndev):
    lib_mod = importlib.import_module("gemma-embed-swift_b200._lib")
    L = lib_mod.lib()
    rng = np.random.default_rng(ndev)
    for trial in range(20):
        lens = [int(x) for x in rng.integers(1, 3000, int(rng.integers(1, 70)))]
        seqs = seq_array(lib_mod, lens)
        out = (ctypes.c_int32 * len(lens))()
        assert L.ge_test_shard(seqs, len(lens), ndev, out) == 0
        got = list(out)
        assert got == shard_restated(lens, ndev)
        cost = [0.0] * ndev
        for n, d in zip(lens, got):
            cost[d] += n + n * n / 2048.0
        biggest = max(n + n * n / 2048.0 for n in lens)
        assert max(cost) - min(cost) <= biggest + 1e-6


def schedule(L, lib_mod, lens, kvh, group, hw, max_ctas):
    seqs = seq_array(lib_mod, lens)
    ctas, words = ctypes.c_int32(), ctypes.c_int32()
    cap = 4 * sum((n + 127) for n in lens) * kvh + max_ctas + 8
    out = (ctypes.c_uint32 * cap)()
    assert L.ge_test_attention_schedule(seqs, len(lens), kvh, group, hw, max_ctas, out, cap, ctypes.byref(ctas),
                                        ctypes.byref(words)) == 0
    w = np.frombuffer(out, dtype=np.uint32)[: words.value]
    n = (words.value - ctas.value - 1) // 4
    return w[: 4 * n].reshape(n, 4), w[4 * n:], ctas.value


@pytest.mark.parametrize("kvh,group,hw", [(1, 3, 512), (1, 3, 0), (2, 2, 512), (1, 4, 0)])
def test_attention_schedule_covers_every_item_once(ge, kvh, group, hw):
    lib_mod = importlib.import_module("gemma-embed-swift_b200._lib")
    L = lib_mod.lib()
    rng = np.random.default_rng(group + hw)
    T = 128 // group
    for max_ctas in (1, 7, 148):
        lens = [int(x) for x in rng.integers(1, 2500, 40)]
        items, offsets, ctas = schedule(L, lib_mod, lens, kvh, group, hw, max_ctas)
        starts = np.cumsum([0] + lens[:-1])
        want = sorted((int(s), n, t0, kh) for s, n in zip(starts, lens) for t0 in range(0, n, T) for kh in range(kvh))
        assert sorted(map(tuple, items.tolist())) == want
        assert ctas == min(len(want), max_ctas)
        assert offsets[0] == 0 and offsets[-1] == len(want) and np.all(np.diff(offsets.astype(np.int64)) >= 0)

        def cost(it):
            s, n, t0, kh = (int(v) for v in it)
            ks, ke = 0, n
            if hw:
                ks, ke = max(t0 - hw, 0), min(t0 + T - 1 + hw + 1, n)
            ks = ks // 64 * 64
            return (ke - ks + 63) // 64 + 2

        loads = [sum(cost(it) for it in items[offsets[c]:offsets[c + 1]]) for c in range(ctas)]
        assert max(loads) - min(loads) <= max(cost(it) for it in items)
        for c in range(ctas):  # longest items first on every CTA
            cs = [cost(it) for it in items[offsets[c]:offsets[c + 1]]]
            assert cs == sorted(cs, reverse=True)


def test_pack(ge):
    seqs = [[5, 6, 7], [1], [9, 9]]
    tokens, positions, ranges = ge.pack(seqs)
    assert tokens.tolist() == [5, 6, 7, 1, 9, 9]
    assert positions.tolist() == [0, 1, 2, 0, 0, 1]
    assert [(r[0], r[1]) for r in ranges] == [(0, 3), (3, 1), (4, 2)]


def test_id_arrays_address_every_text(ge):
    """EmbeddingModel.embed passes pre-tokenised texts as one buffer with per-text addresses: each
    address reads back exactly its text's ids, for one text and for many of mixed lengths."""
    rng = np.random.default_rng(7)
    for lens in ([5], [1, 300, 17, 2, 64], [3] * 40):
        data = [rng.integers(0, 262144, size=n).astype(np.int32) for n in lens]
        flat, lengths, addrs = ge._id_arrays(data)
        assert lengths.tolist() == lens and addrs.dtype == np.uintp
        for d, a, n in zip(data, addrs.tolist(), lens):
            got = np.ctypeslib.as_array(ctypes.cast(a, ctypes.POINTER(ctypes.c_int32)), shape=(n,))
            assert np.array_equal(got, d)
