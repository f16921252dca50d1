"""The image path on the GPU against the CPU oracle (MetalImageForwardTests,
Tests/GemmaEmbedTests/MetalImageForwardTests.swift): patchify bit for bit, the head-dim-64
attention kernel and the GeGLU-quick epilogue against fp32/float64 references, the vision
tower's rows at cosine >= 0.99999 per row (MetalImageForwardTests.swift:96), whole image
embeddings against the oracle's vision + text towers, and bit-identical results whatever the
batch."""
import ctypes
from importlib import import_module

import numpy as np
import pytest

from oracle import binding as B
from oracle.tokenizer import Tokenizer as OracleTokenizer

pytestmark = pytest.mark.gpu

COSINE_MIN = 0.99999
TOL_F16 = 2e-3


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def lib():
    return import_module("gemma-embed-swift_b200._lib")


@pytest.mark.parametrize("patch,w,h", [(16, 96, 64), (16, 768, 48), (14, 84, 42)])
def test_patchify_bit_exact(cuda_device, patch, w, h):
    """k_patchify equals PreparedImage.init's fp16 patches (oracle or_patchify) bit for bit."""
    rng = np.random.default_rng(w + h)
    img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
    mean, std = np.array([0.5, 0.25, 0.0], np.float32), np.array([0.5, 0.75, 1.0], np.float32)
    area = 3 * patch * patch
    kpad = (area + 63) // 64 * 64
    got = np.zeros(((w // patch) * (h // patch), kpad), np.uint16)
    L = lib().lib()
    f32 = ctypes.POINTER(ctypes.c_float)
    rc = L.ge_test_patchify(img.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), w, h, patch, mean.ctypes.data_as(f32),
                            std.ctypes.data_as(f32), got.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), kpad)
    assert rc == 0, L.ge_test_last_error()
    want = B.patchify(img, patch, mean, std).astype(np.float16)
    assert np.array_equal(got[:, :area], want.view(np.uint16))
    assert not got[:, area:].any()


def attention(q, k, v, lens, heads, hd):
    m = lib()
    L = m.lib()
    ntok = sum(lens)
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
    seqs = (m.GeSeq * len(lens))(*[m.GeSeq(int(s), int(n)) for s, n in zip(starts, lens)])
    out = np.zeros((ntok, heads, hd), np.float16)
    args = [np.ascontiguousarray(x).view(np.uint16) for x in (q, k, v)]
    u16 = ctypes.POINTER(ctypes.c_uint16)
    rc = L.ge_test_attention(*[x.ctypes.data_as(u16) for x in args], ntok, seqs, len(lens), heads, heads, hd, 0,
                             out.view(np.uint16).ctypes.data_as(u16))
    assert rc == 0, L.ge_test_last_error()
    return out.astype(np.float32)


LENGTHS64 = [[1, 7, 64], [128, 129, 255], [2304], [2304, 2304, 5],
             [int(x) for x in np.random.default_rng(9).integers(1, 900, 40)]]


@pytest.mark.parametrize("lens", LENGTHS64)
def test_attention64_packed_sequences(oracle, cuda_device, lens):
    """Head dim 64, twelve heads, no mask inside a sequence and nothing across sequences."""
    heads, hd = 12, 64
    rng = np.random.default_rng(len(lens) + sum(lens))
    ntok = sum(lens)
    q = rng.uniform(-0.3, 0.3, size=(ntok, heads, hd)).astype(np.float16)
    k = rng.uniform(-0.3, 0.3, size=(ntok, heads, hd)).astype(np.float16)
    v = rng.uniform(-1, 1, size=(ntok, heads, hd)).astype(np.float16)
    got = attention(q, k, v, lens, heads, hd)
    s = 0
    for n in lens:
        want = oracle.attention(q[s:s + n].astype(np.float32), k[s:s + n].astype(np.float32),
                                v[s:s + n].astype(np.float32), n, heads, heads, hd).reshape(n, heads, hd)
        g = got[s:s + n]
        assert not np.isnan(g).any()
        rel = np.abs(g - want).max() / np.abs(want).max()
        assert rel < TOL_F16, (n, rel)
        s += n


def test_geglu_quick_epilogue(synth, cuda_device):
    m, k, ff = 300, 768, 1024
    rng = np.random.default_rng(3)
    a = rng.uniform(-1, 1, size=(m, k)).astype(np.float16)
    wg = synth.quantize_q8_0(synth.floats(31, ff * k, (3.0 / k) ** 0.5).reshape(ff, k))
    wu = synth.quantize_q8_0(synth.floats(32, ff * k, (3.0 / k) ** 0.5).reshape(ff, k))
    rows = []
    for j in range(ff // 128):
        rows.append(wg[j * 128:(j + 1) * 128])
        rows.append(wu[j * 128:(j + 1) * 128])
    w = np.ascontiguousarray(np.concatenate(rows))
    L = lib().lib()
    out = np.zeros((m, ff), np.float32)
    rc = L.ge_test_gemm(np.ascontiguousarray(a.view(np.uint16)).ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), m, k,
                        w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), 2 * ff, 5, 0, None,
                        out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == 0, L.ge_test_last_error()
    deq = lambda q: synth.dequantize_q8_0(q, k).astype(np.float16).astype(np.float64)
    gate = a.astype(np.float64) @ deq(wg).T
    up = a.astype(np.float64) @ deq(wu).T
    want = gate / (1 + np.exp(-1.702 * gate)) * up
    rel = np.abs(out - want).max() / np.abs(want).max()
    assert rel < TOL_F16, rel


# ------------------------------------------------------------------ the whole image path
@pytest.fixture(scope="module")
def vision_model(ge, synth, cuda_device):
    text = synth.model_path("gemma-embedding", seed=1, layers=6, vocab=4096)
    mmproj = synth.mmproj_path(seed=2, layers=2, positions=64)
    model = ge.EmbeddingModel.load(text, ge.LoadOptions(image_encoder=mmproj, image_patch_budget=1 << 20))
    vis = B.OracleVision(mmproj)
    ref = B.OracleModel(text)
    yield model, vis, ref, OracleTokenizer.from_gguf(text)
    model.close()
    vis.close()
    ref.close()


def images():
    rng = np.random.default_rng(11)
    # A downscaled, an upscaled (letterboxed) and an exact-size image, at most 100 tokens each.
    return [rng.integers(0, 256, (h, w, 3), dtype=np.uint8) for (w, h) in [(800, 600), (200, 150), (432, 432), (96, 240)]]


def test_image_info(vision_model):
    model = vision_model[0]
    assert (model.info.image_layer_count, model.info.image_hidden_size, model.info.image_patch_size,
            model.info.image_projection_dim) == (2, 768, 16, 768)


def test_vision_tower_rows_match_oracle(vision_model):
    """MetalImageForwardTests.testVisionTowerMatchesCPUReferenceAndLlamaCpp: every projected row
    at cosine > 0.99999 against the CPU reference."""
    model, vis, _, _ = vision_model
    ims = images()
    got = model.image_vectors(ims, max_image_tokens=100)
    for im, rows in zip(ims, got):
        patches, gx, gy = vis.prepare(im, max_image_tokens=100)
        want = vis.forward(patches, gx, gy)
        assert rows.shape == want.shape
        worst = min(cosine(a, b) for a, b in zip(rows, want))
        assert worst > COSINE_MIN, (im.shape, worst)


def test_image_embeddings_match_oracle(ge, vision_model):
    """The text tower over [bos, <|image>, rows, <image|>, eos] (MetalForward.imageBatches,
    Metal/MetalForward.swift:286-296) against the oracle's forward over the oracle's rows."""
    model, vis, ref, tok = vision_model
    begin = tok.encode("<|image>", False, True)
    end = tok.encode("<image|>", False, True)
    assert len(begin) == 1 and len(end) == 1
    ims = images()
    got = model.embed_images(ims, ge.ImageEmbedOptions(normalise=False, max_image_tokens=100))
    for im, e in zip(ims, got):
        patches, gx, gy = vis.prepare(im, max_image_tokens=100)
        rows = vis.forward(patches, gx, gy)
        T = rows.shape[0]
        ids = np.array([2, begin[0]] + [-(r + 1) for r in range(T)] + [end[0], 1], np.int32)
        want = ref.forward_rows(ids, rows)
        assert e.token_count == T + 4
        assert cosine(e.vector, want) > COSINE_MIN


def test_image_batch_independence_bit_exact(ge, vision_model):
    """MetalImageForwardTests.testBatchIndependence / testImageBatchIndependenceAcrossGemmTiles:
    an image embeds the same alone, first or last in a batch of other sizes, bit for bit."""
    model = vision_model[0]
    ims = images()
    opts = ge.ImageEmbedOptions(max_image_tokens=100)
    alone = model.embed_images([ims[1]], opts)[0].vector
    first = model.embed_images([ims[1]] + ims[2:] + ims[:1], opts)[0].vector
    last = model.embed_images(ims[2:] + ims[:1] + [ims[1]], opts)[-1].vector
    assert alone.tobytes() == first.tobytes() == last.tobytes()
    one_at_a_time = model.embed_images(ims, ge.ImageEmbedOptions(max_image_tokens=100, batch_size=1))
    together = model.embed_images(ims, opts)
    for a, b in zip(one_at_a_time, together):
        assert a.vector.tobytes() == b.vector.tobytes()


def test_image_options_and_errors(ge, synth, vision_model):
    model = vision_model[0]
    im = images()[2]
    one = model.embed_images(im, ge.ImageEmbedOptions(dimensions=256))
    assert one.vector.shape == (256,) and abs(float(np.linalg.norm(one.vector)) - 1) < 1e-5
    assert model.embed_images([], ge.ImageEmbedOptions()) == []
    for bad in (ge.ImageEmbedOptions(max_image_tokens=0), ge.ImageEmbedOptions(max_image_tokens=1121),
                ge.ImageEmbedOptions(dimensions=100)):
        with pytest.raises(ge.GemmaEmbedError) as e:
            model.embed_images([im], bad)
        assert e.value.case == "invalidOptions"
    with pytest.raises(ge.GemmaEmbedError) as e:
        model.embed_images([np.zeros((4, 4), np.uint8)])
    assert e.value.case == "imageDecoding"
    text_only = ge.EmbeddingModel.load(synth.model_path("gemma-embedding", seed=1, layers=6, vocab=4096))
    try:
        with pytest.raises(ge.GemmaEmbedError) as e:
            text_only.embed_images([im])
        assert e.value.case == "imageEncoderNotLoaded"
    finally:
        text_only.close()


def test_multimodal_inputs_match_oracle(ge, vision_model):
    """embed(_ inputs: [MultimodalInput]) (MultimodalEmbedding.swift:100-206) against the oracle:
    its tokenizer, vision tower and layout (oracle/multimodal.py), then the text tower over the
    sequence with the input's image rows."""
    from oracle import multimodal as om
    model, vis, ref, tok = vision_model
    begin = tok.encode("<|image>", False, True)[0]
    end = tok.encode("<image|>", False, True)[0]
    ims = images()
    inputs = [["a photo of gawy stait", ims[1], "and more words"], [ims[2]], ["only text here"],
              [ims[0], ims[3], "two pictures"]]
    prefix = ge.TaskPrefix.document()
    opts = ge.MultimodalEmbedOptions(task=prefix, normalise=False, max_image_tokens=100)
    got = model.embed_multimodal(inputs, opts)
    for parts, e in zip(inputs, got):
        rows, oparts, spans = [], [], []
        for p in parts:
            if isinstance(p, str):
                oparts.append(("text", p))
            else:
                patches, gx, gy = vis.prepare(p, max_image_tokens=100)
                r = vis.forward(patches, gx, gy)
                rows.append(r)
                oparts.append(("image", None))
                spans.append((r.shape[0], begin, end))
        ids, cut = om.sequence(prefix, oparts, spans, 2048, 2, 1, lambda t: tok.encode(t, False))
        assert e.token_count == len(ids) and not e.truncated
        vec = np.concatenate(rows) if rows else np.zeros((1, 768), np.float32)
        want = ref.forward_rows(np.array(ids, np.int32), vec)
        assert cosine(e.vector, want) > COSINE_MIN
    # A text-only input is the text embedding, bit for bit.
    text = model.embed("only text here", ge.EmbedOptions(task=prefix, normalise=False))
    assert text.vector.tobytes() == got[2].vector.tobytes()
    # Text is cut from the end when the images leave too little room; frames stay whole.
    small = model.embed_multimodal([["some leading text " * 20, ims[2]]],
                                   ge.MultimodalEmbedOptions(max_tokens=120, max_image_tokens=100))[0]
    assert small.truncated and small.token_count == 120
    with pytest.raises(ge.GemmaEmbedError) as exc:
        model.embed_multimodal([[ims[2]]], ge.MultimodalEmbedOptions(max_tokens=50, max_image_tokens=100))
    assert exc.value.case == "invalidOptions"
