"""The oracle's audio path on CPU, pinned where the reference's tests give known answers or an
independent implementation exists:

* frame and token counts against AudioPreprocessingTests (Tests/GemmaEmbedTests/
  AudioPreprocessingTests.swift:8-33) and llama-server's `prompt_tokens` for every fixture clip
  (Fixtures/audio/embeddings.jsonl), both committed as tests/golden/audio_counts.json;
* the log-mel front end bit for bit against a numpy float32 restatement of the reference's
  butterflies and four-bin mel sums (Audio/AudioPreprocessor.swift:178-249), and within the
  reference's own tolerances (AudioPreprocessingTests.swift:60-62) against numpy's float64 FFT;
* the Conformer forward against a float64 numpy restatement of CPUAudioReference.forward
  (Model/CPUAudioReference.swift:186-283);
* the loader's refusals (Model/AudioConfig.swift:50-85, AudioWeights.swift:67-135)."""
import json
import os

import numpy as np
import pytest

from oracle import binding as B

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "audio_counts.json")
TINY = dict(layers=2, hidden=128, heads=2, ff=256)


@pytest.fixture(scope="module")
def tiny_audio(synth):
    return synth.audio_path(seed=5, **TINY)


def _signals():
    rate = 16000
    t = np.arange(int(1.5 * rate)) / rate
    rng = np.random.default_rng(11)
    chirp_t = np.arange(rate) / rate
    return {
        "sine-440": (0.5 * np.sin(2 * np.pi * 440 * t)).astype(np.float32),
        "chirp": (0.4 * np.sin(2 * np.pi * (200 * chirp_t + 2900 * chirp_t ** 2))).astype(np.float32),
        "noise": rng.uniform(-0.5, 0.5, rate).astype(np.float32),
        "silence": np.zeros(rate, np.float32),
        "short": (0.3 * np.sin(2 * np.pi * 523 * np.arange(4800) / rate)).astype(np.float32),
        "clicks": np.where(np.arange(rate) % 1600 == 0, 0.9, 0.0).astype(np.float32),
    }


# ------------------------------------------------------------------ counts
def test_frame_and_token_counts_known_answers():
    g = json.load(open(GOLDEN))["counts"]
    for samples, frames in g["frame_count"]:
        assert B.frame_count(samples) == frames, samples
    for samples, tokens in g["token_count"]:
        assert B.audio_token_count(samples) == tokens, samples
    c = g["chunking"]
    parts = B.chunks(np.full(c["samples"], 0.01, np.float32))
    assert [B.frame_count(len(p)) for p in parts] == c["frames"]
    assert [B.tokens_for_frames(B.frame_count(len(p))) for p in parts] == c["tokens"]
    assert B.audio_token_count(c["samples"]) == c["total"]


def test_fixture_clip_prompt_tokens():
    """llama-server's prompt_tokens = the clip's rows + 4 frame rows, for every 16 kHz fixture clip
    (the channel count does not change the frame count; other rates are resampled first)."""
    clips = json.load(open(GOLDEN))["clips"]
    checked = 0
    for c in clips:
        if c["sample_rate"] != 16000:
            continue
        samples = int(round(c["seconds"] * 16000))
        assert B.audio_token_count(samples) + 4 == c["prompt_tokens"], c["file"]
        checked += 1
    assert checked >= 20


def test_too_short_clip_is_refused():
    with pytest.raises(B.OracleError):
        B.log_mel(np.full(1, 0.1, np.float32))
    with pytest.raises(B.OracleError):
        B.log_mel(np.zeros(0, np.float32))
    assert B.log_mel(np.full(2, 0.1, np.float32)).shape == (1, 128)


# ------------------------------------------------------------------ log-mel
def _frames(chunk, hann):
    n = len(chunk)
    frames = B.frame_count(n)
    padded = np.zeros((frames - 1) * 160 + 512, np.float32)
    padded[160:160 + n] = chunk
    idx = np.arange(frames)[:, None] * 160 + np.arange(512)[None, :]
    return hann[None, :] * padded[idx]


def _log_mel_float32(chunk, t):
    """The reference's arithmetic in numpy float32 (each op rounds to single, none fused)."""
    x = _frames(chunk, t["hann"])
    F = x.shape[0]
    re = np.zeros((F, 512), np.float32)
    im = np.zeros((F, 512), np.float32)
    re[:, t["bitrev"]] = x
    count = 2
    while count <= 512:
        half, step = count // 2, 512 // count
        base = np.arange(0, 512, count)
        k = np.tile(np.arange(half), len(base))
        ev = (base[:, None] + np.arange(half)[None, :]).ravel()
        od = ev + half
        c, s = t["cos"][k * step], -t["sin"][k * step]
        ro, io, er, ei = re[:, od], im[:, od], re[:, ev], im[:, ev]
        re[:, ev] = (er + c * ro) - s * io
        im[:, ev] = (ei + c * io) + s * ro
        re[:, od] = (er - c * ro) + s * io
        im[:, od] = (ei - c * io) - s * ro
        count *= 2
    mag = np.sqrt(re[:, :257] * re[:, :257] + im[:, :257] * im[:, :257])
    w = t["filters"]
    out = np.zeros((F, w.shape[0]), np.float32)
    floor = np.float64(np.float32(0.001))
    for m in range(w.shape[0]):
        lo, hi = int(t["lo"][m]), int(t["hi"][m])
        acc = np.zeros(F, np.float64)
        k = lo
        while k < min(hi, 257 - 3):
            p = mag[:, k] * w[m, k] + mag[:, k + 1] * w[m, k + 1]
            p = p + mag[:, k + 2] * w[m, k + 2]
            p = p + mag[:, k + 3] * w[m, k + 3]
            acc += p.astype(np.float64)
            k += 4
        while k < hi:
            acc += (mag[:, k] * w[m, k]).astype(np.float64)
            k += 1
        out[:, m] = np.log(np.maximum(acc, floor)).astype(np.float32)
    return out


def test_log_mel_matches_float32_restatement_bitwise():
    t = B.audio_tables(128)
    for name, s in _signals().items():
        got = B.log_mel(s)
        want = _log_mel_float32(s, t)
        assert got.shape == want.shape, name
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


def _htk_filters(mel_bins=128):
    mel = lambda f: 2595 * np.log10(1 + f / 700)
    hz = 700 * (10 ** (np.linspace(mel(0.0), mel(8000.0), mel_bins + 2) / 2595) - 1)
    f = np.arange(257) * 16000 / 512
    left, centre, right = hz[:-2, None], hz[1:-1, None], hz[2:, None]
    up = (f[None, :] - left) / (centre - left)
    down = (right - f[None, :]) / (right - centre)
    return np.where((f >= left) & (f <= centre), up, np.where((f > centre) & (f <= right), down, 0.0))


def test_log_mel_matches_float64_fft():
    """An independent float64 FFT and filterbank; bands as the reference's own check against
    llama.cpp (AudioPreprocessingTests.swift:60-62)."""
    hann = np.zeros(512)
    hann[:320] = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(320) / 320)
    filt = _htk_filters()
    t = B.audio_tables(128)
    np.testing.assert_allclose(t["filters"], filt, rtol=0, atol=1e-6)
    for name, s in _signals().items():
        got = B.log_mel(s)
        spec = np.abs(np.fft.rfft(_frames(s.astype(np.float64), hann), axis=1))
        want = np.log(np.maximum(spec @ filt.T, np.float32(0.001)))
        d = np.abs(got - want)
        assert d[want > -2].max(initial=0) < 1e-4, name
        assert d[(want > -6) & (want <= -2)].max(initial=0) < 2e-3, name
        assert d[want <= -6].max(initial=0) < 5e-3, name


def test_log_mel_chunks_are_independent():
    s = np.random.default_rng(3).normal(0, 0.1, 480000 + 16000).astype(np.float32)
    parts = B.chunks(s)
    assert [len(p) for p in parts] == [480000, 16000]
    whole = B.log_mel(parts[1])
    again = B.log_mel(s[480000:].copy())
    assert np.array_equal(whole, again)


# ------------------------------------------------------------------ Conformer forward
def _bound(h, base, which, default):
    try:
        return float(B.tensor(h, f"{base}.{which}")[0, 0])
    except B.OracleError:
        return default


def _linear(h, base, x):
    big = np.finfo(np.float32).max
    lo, hi = _bound(h, base, "input_min", -big), _bound(h, base, "input_max", big)
    y = np.clip(x, lo, hi) @ B.tensor(h, base + ".weight").astype(np.float64).T
    y = np.clip(y, _bound(h, base, "output_min", -big), _bound(h, base, "output_max", big))
    try:
        y = y + B.tensor(h, base + ".bias").astype(np.float64).ravel()
    except B.OracleError:
        pass
    return y


def _rms(x, w=None, eps=1e-6):
    y = x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return y * w if w is not None else y


def _vec(h, name):
    return B.tensor(h, name).astype(np.float64).ravel()


def _subsample(x, w, norm, eps=1e-6):
    """x [T][F][C]; w [O][C][3][3]."""
    T, F, C = x.shape
    OT, OF = (T - 1) // 2 + 1, (F - 1) // 2 + 1
    xp = np.zeros((T + 2 + 1, F + 2 + 1, C))
    xp[1:T + 1, 1:F + 1] = x.astype(np.float32).astype(np.float16).astype(np.float64)
    out = np.zeros((OT, OF, w.shape[0]))
    for kh in range(3):
        for kw in range(3):
            win = xp[kh:kh + 2 * OT:2, kw:kw + 2 * OF:2, :]
            out += np.einsum("tfc,oc->tfo", win, w[:, :, kh, kw])
    mean = out.mean(-1, keepdims=True)
    var = ((out - mean) ** 2).mean(-1, keepdims=True)
    return np.maximum(0, (out - mean) / np.sqrt(var + eps) * norm)


def _numpy_audio(aud, mel):
    h, A = aud._h, aud.info
    d, H, hd = A.hidden, A.heads, A.head_dim
    silu = lambda v: v / (1 + np.exp(-v))
    x = mel.astype(np.float64)[:, :, None]
    cin = 1
    for i, cout in enumerate((128, 32)):
        w = B.tensor(h, f"a.conv1d.{i}.weight").astype(np.float64).reshape(cout, cin, 3, 3)
        x = _subsample(x, w, _vec(h, f"a.conv1d.{i}.norm.weight"))
        cin = cout
    T = x.shape[0]
    x = _linear(h, "a.input_projection", x.reshape(T, -1))
    ts = d // 2
    inc = np.log(10000) / max(ts - 1, 1)
    pos = np.arange(13)[:, None] * np.exp(-np.arange(ts) * inc)[None, :]
    table = np.concatenate([np.sin(pos), np.cos(pos)], axis=1)
    qs = (1 / np.sqrt(hd)) / np.log(2)
    ks = np.log(1 + np.e) / np.log(2)
    for l in range(A.layers):
        p = f"a.blk.{l}."
        v = lambda n: _vec(h, p + n + ".weight")
        up = silu(_linear(h, p + "ffn_up", _rms(x, v("ffn_norm"))))
        x = x + 0.5 * _rms(_linear(h, p + "ffn_down", up), v("ffn_post_norm"))
        a = _rms(x, v("attn_pre_norm"))
        q = _linear(h, p + "attn_q", a).reshape(T, H, hd) * (qs * v("per_dim_scale"))
        k = _linear(h, p + "attn_k", a).reshape(T, H, hd) * ks
        vv = _linear(h, p + "attn_v", a).reshape(T, H, hd)
        rel = _linear(h, p + "attn_k_rel", table).reshape(13, H, hd)
        o = np.zeros((T, H, hd))
        for t in range(T):
            j = np.arange(max(0, t - 11), t + 1)
            s = np.einsum("hi,jhi->hj", q[t], k[j]) + np.einsum("hi,jhi->hj", q[t], rel[t - j])
            s = 50 * np.tanh(s / 50)
            pr = np.exp(s - s.max(-1, keepdims=True))
            pr /= pr.sum(-1, keepdims=True)
            o[t] = np.einsum("hj,jhi->hi", pr, vv[j])
        x = x + _rms(_linear(h, p + "attn_out", o.reshape(T, d)), v("attn_post_norm"))
        pw1 = _linear(h, p + "conv_pw1", _rms(x, v("conv_norm")))
        glu = pw1[:, :d] / (1 + np.exp(-pw1[:, d:]))
        dw = B.tensor(h, p + "conv_dw.weight").astype(np.float64)  # [d][5]
        gp = np.concatenate([np.zeros((4, d)), glu])
        conv = sum(gp[kk:kk + T] * dw[:, kk] for kk in range(5))
        x = x + _linear(h, p + "conv_pw2", silu(_rms(conv, v("norm_conv"))))
        up = silu(_linear(h, p + "ffn_up_1", _rms(x, v("ffn_norm_1"))))
        x = x + 0.5 * _rms(_linear(h, p + "ffn_down_1", up), v("ffn_post_norm_1"))
        x = _rms(x, v("ln2"))
    out = _rms(_linear(h, "a.pre_encode.out", x))
    return _linear(h, "mm.a.input_projection", out)


def test_audio_info(tiny_audio):
    aud = B.OracleAudio(tiny_audio)
    i = aud.info
    assert (i.hidden, i.layers, i.heads, i.head_dim, i.ff, i.mel_bins) == (128, 2, 2, 64, 256, 128)
    assert (i.projection_dim, i.output_width, i.window, i.relative_positions, i.dw_kernel) == (768, 1536, 12, 13, 5)
    assert abs(i.eps - 1e-6) < 1e-12 and i.softcap == 50 and i.ff_residual == 0.5


def test_audio_forward_matches_numpy(tiny_audio):
    aud = B.OracleAudio(tiny_audio)
    for name in ("noise", "sine-440", "short"):
        mel = B.log_mel(_signals()[name])
        trace = {}
        got = aud.forward(mel, trace=trace)
        want = _numpy_audio(aud, mel)
        assert got.shape == (B.tokens_for_frames(mel.shape[0]), 768)
        assert np.abs(got - want).max() <= 2e-4 * np.abs(want).max(), name
        cos = (got * want).sum(1) / np.linalg.norm(got, axis=1) / np.linalg.norm(want, axis=1)
        assert cos.min() > 0.99999, name
        for key in ("mel", "subsample-0", "subsample-1", "encoder_in", "k_rel-0", "attn-1", "conv_dw-1",
                    "layer_out-1", "out_proj", "projected"):
            assert key in trace, key
        assert np.array_equal(trace["projected"], got.ravel())


def test_audio_sinusoid_layout():
    v = B.audio_sinusoid(3, 16)
    inc = np.float32(np.log(np.float32(10000)) / np.float32(7))
    want = np.float32(3) * np.exp(-np.arange(8, dtype=np.float32) * inc)
    np.testing.assert_allclose(v[:8], np.sin(want), atol=1e-6)
    np.testing.assert_allclose(v[8:], np.cos(want), atol=1e-6)
    assert np.array_equal(B.audio_sinusoid(0, 16), np.r_[np.zeros(8), np.ones(8)].astype(np.float32))


def test_audio_open_failures(synth, tmp_path):
    kw = dict(layers=1, hidden=128, heads=2, ff=256)
    arch = synth.Arch(name="clip", hidden=128, layers=1, heads=2, head_dim_swa=0, head_dim_global=0, kv_swa=0,
                      kv_global=0, ff=256, per_layer=0, out_dim=0, dense_head=0)
    tensors = synth.audio_tensors(1, 768, **kw)

    def write(name, kvs, ts=tensors):
        p = str(tmp_path / name)
        synth.write_gguf(p, arch, ts, kvs=kvs)
        return p

    def swap(kvs, key, vtype, payload):
        return [synth._kv(key, vtype, payload) if k.startswith(synth._str(key)) else k for k in kvs]

    meta = synth.audio_metadata(768, **kw)
    cases = [
        (write("noaudio.gguf", swap(meta, "clip.has_audio_encoder", 7, b"\x00")), B.OracleError, 2),
        (write("proj.gguf", swap(meta, "clip.audio.projector_type", 8, synth._str("gemma4v"))), B.OracleError, 2),
        (write("mel.gguf", swap(meta, "clip.audio.num_mel_bins", 4, (126).to_bytes(4, "little"))), B.OracleError, 2),
        (write("heads.gguf", swap(meta, "clip.audio.attention.head_count", 4, (3).to_bytes(4, "little"))),
         B.OracleError, 2),
        (write("missing.gguf", meta, [t for t in tensors if t.name != "a.blk.0.conv_dw.weight"]), B.OracleError, 5),
    ]
    for path, exc, code in cases:
        with pytest.raises(exc) as e:
            B.OracleAudio(path)
        assert e.value.code == code, path
    # the vision file has no audio encoder
    with pytest.raises(B.OracleError):
        B.OracleAudio(synth.mmproj_path(seed=3, layers=2, positions=64))
