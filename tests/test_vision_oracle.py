"""The oracle's image path on CPU, pinned where the reference's tests give known answers or an
independent implementation exists: fp16 rounding against numpy, ImageResizer.targetSize against
the reference's own cases (Tests/GemmaEmbedTests/ImagePreprocessingTests.swift:97-106), the
bicubic resize against Pillow (whose resampler the reference ports operation for operation,
Image/ImageResizer.swift:51-53), the patch layout, and the vision forward against a float64
numpy restatement of CPUVisionReference.forward (Model/CPUVisionReference.swift:89-165)."""
import math

import numpy as np
import pytest

from oracle import binding as B


@pytest.fixture(scope="module")
def tiny_mmproj(synth):
    """Two layers, a 64-entry position table, projected to 768."""
    return synth.mmproj_path(seed=3, layers=2, positions=64)


def test_round_f16_matches_numpy():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(5000).astype(np.float32) * s
                           for s in (1e-8, 6e-5, 1e-3, 1.0, 300.0, 6e4, 7e4)])
    edge = np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 6.1035156e-05, 5.9604645e-08, 2.9802322e-08,
                     1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11, -(1.0 + 2 ** -11)], np.float32)
    for v in np.concatenate([vals, edge]):
        with np.errstate(over="ignore"):
            want = np.float32(np.float16(v))
        assert np.float32(B.round_f16(float(v))) == want, v


def test_target_size_known_answers():
    """ImagePreprocessingTests.testTargetSizeBranches (alignment 48, 70..256 tokens)."""
    cases = [((1600, 1600), (768, 768)), ((1728, 1728), (768, 768)), ((640, 640), (624, 624)),
             ((800, 400), (816, 384)), ((200, 150), (480, 384))]
    for (w, h), want in cases:
        assert B.target_size(w, h, 48, 70 * 2304, 256 * 2304) == want


def test_bicubic_resize_matches_pillow():
    from PIL import Image
    rng = np.random.default_rng(1)
    sizes = [(100, 80, 48, 40), (37, 53, 96, 96), (300, 200, 300, 144), (1024, 768, 512, 384), (13, 7, 113, 71),
             (640, 480, 624, 480), (48, 480, 48, 96), (5, 5, 480, 480)]
    for _ in range(8):
        w, h = int(rng.integers(8, 400)), int(rng.integers(8, 400))
        sizes.append((w, h, 48 * int(rng.integers(1, 12)), 48 * int(rng.integers(1, 12))))
    for w, h, tw, th in sizes:
        img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
        got = B.fit_image(img, tw, th)
        scale = min(np.float32(tw) / np.float32(w), np.float32(th) / np.float32(h))
        fw = min(math.ceil(np.float32(w) * scale), tw)
        fh = min(math.ceil(np.float32(h) * scale), th)
        want = np.asarray(Image.fromarray(img).resize((fw, fh), Image.BICUBIC))
        ox, oy = (tw - fw) // 2, (th - fh) // 2
        assert np.array_equal(got[oy:oy + fh, ox:ox + fw], want), (w, h, tw, th)
        # the letterbox around the fitted image is black
        mask = np.ones((th, tw), bool)
        mask[oy:oy + fh, ox:ox + fw] = False
        assert not got[mask].any()


def test_patch_layout():
    rng = np.random.default_rng(2)
    p, gx, gy = 16, 3, 2
    img = rng.integers(0, 256, (gy * p, gx * p, 3), dtype=np.uint8)
    mean, std = [0.1, 0.2, 0.3], [0.5, 0.6, 0.7]
    got = B.patchify(img, p, mean, std)
    assert got.shape == (gx * gy, 3 * p * p)
    f = (img.astype(np.float32) / np.float32(255) - np.array(mean, np.float32)) / np.array(std, np.float32)
    v = (np.float32(2) * f - np.float32(1)).astype(np.float16).astype(np.float32)
    for py in range(gy):
        for px in range(gx):
            block = v[py * p:(py + 1) * p, px * p:(px + 1) * p, :]  # [ky][kx][c]
            assert np.array_equal(got[py * gx + px], block.transpose(2, 0, 1).reshape(-1))


def _matrix(vis, name, rows, cols):
    return B.tensor(vis._h, name).reshape(rows, cols).astype(np.float64)


def _numpy_vision(vis, patches, gx, gy):
    """CPUVisionReference.forward in float64 with the oracle's dequantised weights."""
    I = vis.info
    d, hd, heads, ff, L = I.hidden, I.head_dim, I.heads, I.ff, I.layers
    eps = float(I.eps)

    def rms(x, w=None):
        y = x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
        return y * w if w is not None else y

    P = gx * gy
    px = np.arange(P) % gx
    py = np.arange(P) // gx
    area = 3 * I.patch * I.patch
    x = patches.astype(np.float64) @ _matrix(vis, "v.patch_embd.weight", d, area).T
    pos = _matrix(vis, "v.position_embd.weight", 2 * I.position_count, d)
    x = x + pos[px] + pos[I.position_count + py]
    quarter = hd // 4
    inv = 100.0 ** (-2.0 * np.arange(quarter) / (hd // 2))
    ang_x, ang_y = px[:, None] * inv[None], py[:, None] * inv[None]

    def rope(t):  # t: [P][heads][hd]
        t = t.copy()
        for off, ang in ((0, ang_x), (hd // 2, ang_y)):
            c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
            a, b = t[:, :, off:off + quarter].copy(), t[:, :, off + quarter:off + 2 * quarter].copy()
            t[:, :, off:off + quarter] = a * c - b * s
            t[:, :, off + quarter:off + 2 * quarter] = a * s + b * c
        return t

    vec = lambda name, n: _matrix(vis, name, 1, n)[0]
    for l in range(L):
        pre = f"v.blk.{l}."
        a = rms(x, vec(pre + "ln1.weight", d))
        q = (a @ _matrix(vis, pre + "attn_q.weight", d, d).T).reshape(P, heads, hd)
        k = (a @ _matrix(vis, pre + "attn_k.weight", d, d).T).reshape(P, heads, hd)
        v = (a @ _matrix(vis, pre + "attn_v.weight", d, d).T).reshape(P, heads, hd)
        q = rope(rms(q, vec(pre + "attn_q_norm.weight", hd)))
        k = rope(rms(k, vec(pre + "attn_k_norm.weight", hd)))
        v = rms(v)
        s = np.einsum("ihd,jhd->hij", q, k)
        s = np.exp(s - s.max(-1, keepdims=True))
        s /= s.sum(-1, keepdims=True)
        att = np.einsum("hij,jhd->ihd", s, v).reshape(P, d)
        o = rms(att @ _matrix(vis, pre + "attn_out.weight", d, d).T, vec(pre + "attn_post_norm.weight", d))
        x = x + o
        f = rms(x, vec(pre + "ln2.weight", d))
        g = f @ _matrix(vis, pre + "ffn_gate.weight", ff, d).T
        u = f @ _matrix(vis, pre + "ffn_up.weight", ff, d).T
        act = g / (1 + np.exp(-1.702 * g)) * u
        dn = rms(act @ _matrix(vis, pre + "ffn_down.weight", d, ff).T, vec(pre + "ffn_post_norm.weight", d))
        x = x + dn
    m = I.merge
    grid = x.reshape(gy, gx, d)
    pooled = grid.reshape(gy // m, m, gx // m, m, d).sum((1, 3)).reshape(-1, d) * (math.sqrt(d) / (m * m))
    return rms(pooled) @ _matrix(vis, "mm.input_projection.weight", I.projection_dim, d).T


def test_vision_forward_matches_numpy(tiny_mmproj):
    vis = B.OracleVision(tiny_mmproj)
    try:
        assert (vis.info.hidden, vis.info.heads, vis.info.head_dim, vis.info.layers) == (768, 12, 64, 2)
        rng = np.random.default_rng(4)
        img = rng.integers(0, 256, (9 * 16, 6 * 16, 3), dtype=np.uint8)
        patches = B.patchify(img, 16, [0, 0, 0], [1, 1, 1])
        got = vis.forward(patches, 6, 9)
        want = _numpy_vision(vis, patches, 6, 9)
        assert got.shape == (6, 768)
        rel = np.abs(got - want).max() / np.abs(want).max()
        assert rel < 1e-4, rel
    finally:
        vis.close()


def test_vision_open_failures(synth, tmp_path):
    """VisionConfig.init's refusals (VisionConfig.swift:43-71): another projector is an invalid
    file, a missing key is missing metadata, a mis-shaped tensor a shape mismatch."""
    tensors = synth.vision_tensors(1, 768, layers=1, positions=8)
    good = synth.vision_metadata(768, layers=1)
    key = lambda r: r[8:8 + int.from_bytes(r[:8], "little")].decode()
    bad_proj = [r for r in good if key(r) != "clip.vision.projector_type"] + [
        synth._kv("clip.vision.projector_type", 8, synth._str("llava"))]
    no_layers = [r for r in good if key(r) != "clip.vision.block_count"]
    short = [t for t in tensors if t.name != "v.blk.0.attn_q_norm.weight"] + [
        synth.Tensor("v.blk.0.attn_q_norm.weight", [32], synth.GGML_F32, b"\0" * 128)]
    arch = synth.make_arch("gemma-embedding", layers=1, vocab=256)
    for i, (kvs, ts, code) in enumerate([(bad_proj, tensors, 2), (no_layers, tensors, 6), (good, short, 7)]):
        p = str(tmp_path / f"bad{i}.gguf")
        synth.write_gguf(p, arch, ts, kvs=kvs)
        with pytest.raises(B.OracleError) as e:
            B.OracleVision(p)
        assert e.value.code == code, e.value


def test_forward_rows_vector_rows_stand_for_tokens(synth, oracle):
    """A vector row holding a token's scaled embedding gives that token's result (InputRow.vector is
    entered unscaled, CPUReference.swift:191-202)."""
    path = synth.model_path("gemma-embedding", seed=1, layers=2, vocab=4096)
    m = oracle.OracleModel(path)
    try:
        ids = np.array([2, 100, 200, 300, 1], np.int32)
        d = m.info.hidden
        vec = np.stack([m.dequantize_row("token_embd.weight", int(t), d) for t in ids[1:4]]) * np.float32(math.sqrt(d))
        want = m.forward(ids)
        got = m.forward_rows(np.array([2, -1, -2, -3, 1], np.int32), vec)
        assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
    finally:
        m.close()
