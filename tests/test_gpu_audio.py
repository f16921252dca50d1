"""The audio path on the GPU against the CPU oracle (MetalAudioForwardTests and
AudioEmbeddingTests, Tests/GemmaEmbedTests/MetalAudioForwardTests.swift and
AudioEmbeddingTests.swift): the log-mel front end bit for bit, the audio tower's projected rows
at cosine > 0.99999 per row (MetalAudioForwardTests.swift:76), whole clip embeddings against the
oracle's audio + text towers, clips that span two 30-second chunks, bit-identical results
whatever the batch, and the API's refusals."""
import ctypes
from importlib import import_module

import numpy as np
import pytest

from oracle import binding as B
from oracle.tokenizer import Tokenizer as OracleTokenizer

pytestmark = pytest.mark.gpu

COSINE_MIN = 0.99999
# The GPU-shaped audio encoder: head dim 128 as the real one, fewer and narrower layers.
SMALL = dict(layers=2, hidden=512, heads=4, ff=1024)


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def lib():
    return import_module("gemma-embed-swift_b200._lib")


def gpu_log_mel(samples):
    s = np.ascontiguousarray(samples, np.float32)
    frames = ctypes.c_int32(0)
    out = np.zeros((B.frame_count(len(s)), 128), np.float32)
    f32 = ctypes.POINTER(ctypes.c_float)
    L = lib().lib()
    rc = L.ge_test_log_mel(s.ctypes.data_as(f32), len(s), 128, out.ctypes.data_as(f32), ctypes.byref(frames))
    assert rc == 0, L.ge_test_last_error()
    assert frames.value == out.shape[0]
    return out


def signals():
    rng = np.random.default_rng(7)
    t = np.arange(24000) / 16000
    return {
        "sine": (0.5 * np.sin(2 * np.pi * 440 * t)).astype(np.float32),
        "noise": rng.normal(0, 0.1, 16000).astype(np.float32),
        "loud": rng.uniform(-1, 1, 7000).astype(np.float32),
        "silence": np.zeros(3200, np.float32),
        "two": np.array([0.3, -0.2], np.float32),
        "odd": rng.normal(0, 0.2, 4801).astype(np.float32),
        "chunk": rng.normal(0, 0.05, 480000).astype(np.float32),
    }


@pytest.mark.parametrize("name", list(signals()))
def test_log_mel_bit_exact(cuda_device, name):
    """k_log_mel equals AudioFrontEnd.logMel (oracle or_audio_log_mel) bit for bit: the same
    butterflies in the same order with separately rounded operations, the same four-bin sums."""
    s = signals()[name]
    got = gpu_log_mel(s)
    want = B.log_mel(s)
    assert got.shape == want.shape
    diff = got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64)
    # The last step is a double-precision log rounded to float: CUDA's and the host's log may
    # differ in the double's last place, which reaches the float only at a rounding boundary.
    assert np.abs(diff).max() <= 1, name
    assert np.count_nonzero(diff) <= max(1, got.size // 100000), name


# ------------------------------------------------------------------ the whole audio path
@pytest.fixture(scope="module")
def audio_model(ge, synth, cuda_device):
    text = synth.model_path("gemma-embedding", seed=1, layers=6, vocab=4096)
    enc = synth.audio_path(seed=4, **SMALL)
    model = ge.EmbeddingModel.load(text, ge.LoadOptions(audio_encoder=enc))
    aud = B.OracleAudio(enc)
    ref = B.OracleModel(text)
    yield model, aud, ref, OracleTokenizer.from_gguf(text)
    model.close()
    aud.close()
    ref.close()


def clips():
    rng = np.random.default_rng(21)
    t = np.arange(20000) / 16000
    return [rng.normal(0, 0.1, 16000).astype(np.float32),             # 1 s: 25 rows
            (0.4 * np.sin(2 * np.pi * 523 * t)).astype(np.float32),  # 1.25 s
            rng.normal(0, 0.05, 4800).astype(np.float32),             # 0.3 s: 8 rows
            rng.uniform(-0.5, 0.5, 3000).astype(np.float32)]


def long_clip():
    """35 s: a full 30-second chunk and a 5-second one (750 + 125 rows)."""
    return np.random.default_rng(5).normal(0, 0.08, 560000).astype(np.float32)


def test_audio_info(audio_model):
    info = audio_model[0].info
    assert (info.audio_layer_count, info.audio_hidden_size, info.audio_head_count, info.audio_feed_forward_size,
            info.audio_mel_bins, info.audio_projection_dim) == (2, 512, 4, 1024, 128, 768)


def test_audio_tower_rows_match_oracle(audio_model):
    """MetalAudioForwardTests.testAudioTowerMatchesCPUReferenceAndLlamaCpp: every projected row
    at cosine > 0.99999 against the CPU reference, chunk by chunk."""
    model, aud, _, _ = audio_model
    cs = clips() + [long_clip()]
    got = model.audio_vectors(cs)
    for c, rows in zip(cs, got):
        want = aud.embed_rows(c)
        assert rows.shape == want.shape, (len(c), rows.shape, want.shape)
        worst = min(cosine(a, b) for a, b in zip(rows, want))
        assert worst > COSINE_MIN, (len(c), worst)


def test_audio_embeddings_match_oracle(ge, audio_model):
    """The text tower over [bos, <|audio>, rows, <audio|>, eos] against the oracle's forward over
    the oracle's rows."""
    model, aud, ref, tok = audio_model
    begin = tok.encode("<|audio>", False, True)
    end = tok.encode("<audio|>", False, True)
    assert len(begin) == 1 and len(end) == 1
    cs = clips() + [long_clip()]
    got = model.embed_audios(cs, ge.AudioEmbedOptions(normalise=False))
    for c, e in zip(cs, got):
        rows = aud.embed_rows(c)
        T = rows.shape[0]
        ids = np.array([2, begin[0]] + [-(r + 1) for r in range(T)] + [end[0], 1], np.int32)
        want = ref.forward_rows(ids, rows)
        assert e.token_count == T + 4 == B.audio_token_count(len(c)) + 4
        assert cosine(e.vector, want) > COSINE_MIN


def test_audio_batch_independence_bit_exact(ge, audio_model):
    """A clip embeds the same alone, first or last in a batch, and one clip per batch or all
    together, bit for bit."""
    model = audio_model[0]
    cs = clips()
    alone = model.embed_audios([cs[1]])[0].vector
    first = model.embed_audios([cs[1]] + cs[2:] + cs[:1])[0].vector
    last = model.embed_audios(cs[2:] + cs[:1] + [cs[1]])[-1].vector
    assert alone.tobytes() == first.tobytes() == last.tobytes()
    one_at_a_time = model.embed_audios(cs, ge.AudioEmbedOptions(batch_size=1))
    together = model.embed_audios(cs)
    for a, b in zip(one_at_a_time, together):
        assert a.vector.tobytes() == b.vector.tobytes()


def test_audio_device_forward_matches_host_api(ge, audio_model):
    """ge_audio_forward_device on device-resident samples gives the pooled rows of embed_audios."""
    import torch
    model = audio_model[0]
    cs = clips()
    host = model.embed_audios(cs, ge.AudioEmbedOptions(normalise=False))
    pcm = torch.from_numpy(np.concatenate(cs)).cuda()
    out = torch.zeros((len(cs), model.info.output_dimensions), dtype=torch.float32, device="cuda")
    model.audio_forward_device(pcm.data_ptr(), [len(c) for c in cs], out.data_ptr(),
                               stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for e, row in zip(host, out.cpu().numpy()):
        assert np.array_equal(e.vector, row)


def test_audio_options_and_errors(ge, synth, audio_model):
    model = audio_model[0]
    c = clips()[0]
    one = model.embed_audios(c, ge.AudioEmbedOptions(dimensions=256))
    assert one.vector.shape == (256,) and abs(float(np.linalg.norm(one.vector)) - 1) < 1e-5
    assert one.token_count == 25 + 4
    assert model.embed_audios([], ge.AudioEmbedOptions()) == []
    for bad in (ge.AudioEmbedOptions(dimensions=100), ge.AudioEmbedOptions(max_tokens=4),
                ge.AudioEmbedOptions(max_tokens=model.info.max_tokens + 1), ge.AudioEmbedOptions(batch_size=0)):
        with pytest.raises(ge.GemmaEmbedError) as e:
            model.embed_audios([c], bad)
        assert e.value.case == "invalidOptions"
    # A clip needing more rows than max_tokens is refused, not cut (AudioEmbedding.swift:86-91).
    with pytest.raises(ge.GemmaEmbedError) as e:
        model.embed_audios([c], ge.AudioEmbedOptions(max_tokens=28))
    assert e.value.case == "invalidOptions"
    assert model.embed_audios([c], ge.AudioEmbedOptions(max_tokens=29))[0].token_count == 29
    for bad_clip in (np.zeros(1, np.float32), np.zeros(0, np.float32), (c, 0, 1), (c, 16000, 0)):
        with pytest.raises(ge.GemmaEmbedError) as e:
            model.embed_audios([bad_clip])
        assert e.value.case == "audioDecoding"
    text_only = ge.EmbeddingModel.load(synth.model_path("gemma-embedding", seed=1, layers=6, vocab=4096))
    try:
        with pytest.raises(ge.GemmaEmbedError) as e:
            text_only.embed_audios([c])
        assert e.value.case == "audioEncoderNotLoaded"
    finally:
        text_only.close()


def test_audio_encoder_load_refusals(ge, synth, cuda_device):
    text = synth.model_path("gemma-embedding", seed=1, layers=6, vocab=4096)
    # projects to 512, the text model is 768 wide (MetalForward.swift:90-92)
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.EmbeddingModel.load(text, ge.LoadOptions(audio_encoder=synth.audio_path(seed=4, projection_dim=512, **SMALL)))
    assert e.value.case == "invalidGGUF"
    # head dim 64: a shape the kernels are not built for
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.EmbeddingModel.load(text, ge.LoadOptions(audio_encoder=synth.audio_path(seed=4, layers=1, hidden=512,
                                                                                     heads=8, ff=1024)))
    assert e.value.case == "unsupportedArchitecture"
    # an image-only mmproj has no audio encoder
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.EmbeddingModel.load(text, ge.LoadOptions(audio_encoder=synth.mmproj_path(seed=2, layers=2, positions=64)))
    assert e.value.case == "invalidGGUF"


def test_multimodal_text_images_and_clips_match_oracle(ge, synth, cuda_device):
    """embed(_ inputs: [MultimodalInput]) (MultimodalEmbedding.swift:100-206) with text, images and
    clips in one input: the oracle's towers and layout (oracle/multimodal.py), then the text tower
    over the sequence with the input's rows in reading order."""
    from oracle import multimodal as om
    text = synth.model_path("gemma-embedding", seed=1, layers=6, vocab=4096)
    mmproj = synth.mmproj_path(seed=2, layers=2, positions=64)
    enc = synth.audio_path(seed=4, **SMALL)
    model = ge.EmbeddingModel.load(text, ge.LoadOptions(image_encoder=mmproj, audio_encoder=enc,
                                                        image_patch_budget=1 << 20))
    vis, aud, ref = B.OracleVision(mmproj), B.OracleAudio(enc), B.OracleModel(text)
    tok = OracleTokenizer.from_gguf(text)
    try:
        marks = {k: tok.encode(k, False, True)[0] for k in ("<|image>", "<image|>", "<|audio>", "<audio|>")}
        rng = np.random.default_rng(31)
        img = rng.integers(0, 256, (240, 320, 3), dtype=np.uint8)
        cs = clips()
        inputs = [["a spoken gawy stait", cs[0], "and the end"], [cs[1]], [img, cs[2], "both kinds"],
                  [cs[3], img, cs[0]], ["only text here"]]
        prefix = ge.TaskPrefix.document()
        got = model.embed_multimodal(inputs, ge.MultimodalEmbedOptions(task=prefix, normalise=False,
                                                                       max_image_tokens=100))
        for parts, e in zip(inputs, got):
            rows, oparts, spans = [], [], []
            for p in parts:
                if isinstance(p, str):
                    oparts.append(("text", p))
                elif p.ndim == 3:
                    patches, gx, gy = vis.prepare(p, max_image_tokens=100)
                    r = vis.forward(patches, gx, gy)
                    rows.append(r)
                    oparts.append(("image", None))
                    spans.append((r.shape[0], marks["<|image>"], marks["<image|>"]))
                else:
                    r = aud.embed_rows(p)
                    rows.append(r)
                    oparts.append(("audio", None))
                    spans.append((r.shape[0], marks["<|audio>"], marks["<audio|>"]))
            ids, cut = om.sequence(prefix, oparts, spans, 2048, 2, 1, lambda t: tok.encode(t, False))
            assert e.token_count == len(ids) and not e.truncated
            vec = np.concatenate(rows) if rows else np.zeros((1, 768), np.float32)
            want = ref.forward_rows(np.array(ids, np.int32), vec)
            assert cosine(e.vector, want) > COSINE_MIN
        # A clip-only input equals embed(audios:) on that clip, bit for bit.
        alone = model.embed_audios([cs[1]], ge.AudioEmbedOptions(normalise=False))[0]
        only = model.embed_multimodal([[cs[1]]], ge.MultimodalEmbedOptions(task="", normalise=False))[0]
        assert only.token_count == alone.token_count
        assert only.vector.tobytes() == alone.vector.tobytes()
    finally:
        model.close()
        vis.close()
        aud.close()
        ref.close()


def test_audio_chunk_edges_match_oracle(ge, audio_model):
    """Clips at the front end's edges: two samples (one frame, one row), exactly one 30-second
    chunk (750 rows), and two samples past it (a second chunk of one frame and one row).  One
    sample past it leaves a chunk without a frame, where the reference stops on a precondition
    (AudioPreprocessor.swift:144): refused."""
    model, aud, _, _ = audio_model
    rng = np.random.default_rng(41)
    cs = [np.array([0.25, -0.5], np.float32), rng.normal(0, 0.05, 480000).astype(np.float32),
          rng.normal(0, 0.05, 480002).astype(np.float32)]
    got = model.audio_vectors(cs)
    assert [g.shape[0] for g in got] == [1, 750, 751]
    with pytest.raises(ge.GemmaEmbedError) as e:
        model.embed_audios([np.zeros(480001, np.float32)])
    assert e.value.case == "audioDecoding"
    for c, rows in zip(cs, got):
        want = aud.embed_rows(c)
        assert rows.shape == want.shape
        worst = min(cosine(a, b) for a, b in zip(rows, want))
        assert worst > COSINE_MIN, (len(c), worst)


def test_device_forwards_back_to_back(ge, audio_model):
    """Two device-resident audio forwards with different clips, enqueued on one stream without a
    synchronisation between them, each give the pooled rows of embed_audios on its own clips: the
    second call's staging of its chunk table waits for the first call's copies."""
    import torch
    model = audio_model[0]
    a, b = clips(), [long_clip(), clips()[2]]
    want_a = model.embed_audios(a, ge.AudioEmbedOptions(normalise=False))
    want_b = model.embed_audios(b, ge.AudioEmbedOptions(normalise=False))
    od = model.info.output_dimensions
    pa, pb = torch.from_numpy(np.concatenate(a)).cuda(), torch.from_numpy(np.concatenate(b)).cuda()
    oa = torch.zeros((len(a), od), dtype=torch.float32, device="cuda")
    ob = torch.zeros((len(b), od), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    for _ in range(3):
        model.audio_forward_device(pa.data_ptr(), [len(c) for c in a], oa.data_ptr(), stream=stream.cuda_stream)
        model.audio_forward_device(pb.data_ptr(), [len(c) for c in b], ob.data_ptr(), stream=stream.cuda_stream)
    torch.cuda.synchronize()
    for e, row in zip(want_a, oa.cpu().numpy()):
        assert np.array_equal(e.vector, row)
    for e, row in zip(want_b, ob.cpu().numpy()):
        assert np.array_equal(e.vector, row)


def test_other_rates_and_channels_are_converted(ge, audio_model):
    """Clips at other rates and channel counts embed as their 16 kHz mono conversion
    (MiniaudioConverter, restated in the oracle) does, bit for bit."""
    model = audio_model[0]
    rng = np.random.default_rng(8)
    inputs = [(rng.uniform(-0.5, 0.5, 2 * 22050).astype(np.float32), 44100, 2),
              (rng.uniform(-0.5, 0.5, 12000).astype(np.float32), 8000, 1),
              (rng.uniform(-0.5, 0.5, 4 * 24000).astype(np.float32), 48000, 4)]
    got = model.embed_audios(inputs, ge.AudioEmbedOptions(normalise=False))
    converted = [B.to_mono16k(x, rate, ch) for x, rate, ch in inputs]
    want = model.embed_audios(converted, ge.AudioEmbedOptions(normalise=False))
    for g, w, c in zip(got, want, converted):
        assert g.token_count == w.token_count == B.audio_token_count(len(c)) + 4
        assert g.vector.tobytes() == w.vector.tobytes()


def _wav(pcm16: np.ndarray, rate: int, channels: int) -> bytes:
    """A plain 16-bit PCM RIFF/WAVE file around interleaved int16 samples."""
    import struct
    payload = np.asarray(pcm16, "<i2").tobytes()
    fmt = struct.pack("<HHIIHH", 1, channels, rate, rate * 2 * channels, 2 * channels, 16)
    body = b"fmt " + struct.pack("<I", 16) + fmt + b"data" + struct.pack("<I", len(payload)) + payload
    return b"RIFF" + struct.pack("<I", 4 + len(body)) + b"WAVE" + body


def test_wav_inputs_embed_as_their_decoded_samples(ge, audio_model, tmp_path):
    """AudioInput.data and .url (Audio/AudioInput.swift:9-11): WAV bytes and files embed exactly
    as their samples, decoded as dr_wav decodes them (oracle/wav.py), do; a batch mixing the
    forms is bit-identical to each form alone, and a malformed file names its clip."""
    from oracle import wav as W
    model = audio_model[0]
    rng = np.random.default_rng(12)
    wavs = [_wav(rng.integers(-20000, 20000, 2 * 22050, dtype=np.int16), 22050, 2),
            _wav(rng.integers(-20000, 20000, 40000, dtype=np.int16), 16000, 1),
            _wav(rng.integers(-20000, 20000, 3 * 16000, dtype=np.int16), 48000, 1)]
    path = tmp_path / "clip.wav"
    path.write_bytes(wavs[0])
    opts = ge.AudioEmbedOptions(normalise=False)
    got = model.embed_audios([ge.AudioInput.data(w) for w in wavs], opts)
    decoded = [W.decode(w) for w in wavs]
    want = model.embed_audios([(x, rate, ch) for x, rate, ch in decoded], opts)
    for g, w, (x, rate, ch) in zip(got, want, decoded):
        assert g.token_count == w.token_count == B.audio_token_count(len(B.to_mono16k(x, rate, ch))) + 4
        assert g.vector.tobytes() == w.vector.tobytes()
    from_url = model.embed_audios(ge.AudioInput.url(path), opts)
    assert from_url.vector.tobytes() == got[0].vector.tobytes()
    mixed = model.embed_audios([decoded[1][0], ge.AudioInput.data(wavs[0]), ge.AudioInput.url(path)], opts)
    assert mixed[0].vector.tobytes() == got[1].vector.tobytes()
    assert mixed[1].vector.tobytes() == got[0].vector.tobytes() == mixed[2].vector.tobytes()
    only = model.embed_multimodal([[ge.AudioInput.data(wavs[2])]], ge.MultimodalEmbedOptions(task="", normalise=False))[0]
    assert only.vector.tobytes() == got[2].vector.tobytes()
    bad = wavs[1][:36] + b"junk" + wavs[1][40:]
    with pytest.raises(ge.GemmaEmbedError) as e:
        model.embed_audios([ge.AudioInput.data(wavs[0]), ge.AudioInput.data(bad)], opts)
    assert e.value.message == "cannot decode audio: audio 1: WAV: no data chunk"
    with pytest.raises(ge.GemmaEmbedError) as e:
        model.embed_audios([ge.AudioInput.data(b"ID3 an mp3 file, say")], opts)
    assert e.value.case == "audioDecoding" and "not a WAV file" in e.value.message
