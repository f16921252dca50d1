"""The library's own multi-GPU dispatch (EmbeddingModel on several devices): texts, images and
clips of one call spread over the model's devices (csrc/api.cpp), and every vector equals, bit
for bit, the one a single-device model gives.  Skipped on a box with one GPU."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL_AUDIO = dict(layers=2, hidden=512, heads=4, ff=1024)


@pytest.fixture(scope="module")
def two_models(ge, synth, cuda_device):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    text = synth.model_path("gemma-embedding", seed=1, layers=6, vocab=4096)
    opts = dict(image_encoder=synth.mmproj_path(seed=2, layers=2, positions=64),
                audio_encoder=synth.audio_path(seed=4, **SMALL_AUDIO), image_patch_budget=1 << 20)
    one = ge.EmbeddingModel.load(text, ge.LoadOptions(devices=(0,), **opts))
    two = ge.EmbeddingModel.load(text, ge.LoadOptions(devices=(0, 1), **opts))
    yield one, two
    one.close()
    two.close()


def test_two_devices_equal_one(ge, synth, two_models):
    one, two = two_models
    assert two.info.device_count == 2
    rng = np.random.default_rng(3)
    texts = [synth.synthetic_text(s, 20 + 15 * s) for s in range(9)]
    images = [rng.integers(0, 256, (h, w, 3), dtype=np.uint8) for (w, h) in [(640, 480), (200, 150), (432, 432),
                                                                               (96, 240), (300, 300)]]
    clips = [rng.normal(0, 0.1, n).astype(np.float32) for n in (16000, 4800, 560000, 2, 40000)]
    for a, b in zip(one.embed(texts), two.embed(texts)):
        assert a.vector.tobytes() == b.vector.tobytes() and a.token_count == b.token_count
    opts = ge.ImageEmbedOptions(max_image_tokens=100)
    for a, b in zip(one.embed_images(images, opts), two.embed_images(images, opts)):
        assert a.vector.tobytes() == b.vector.tobytes() and a.token_count == b.token_count
    for a, b in zip(one.embed_audios(clips), two.embed_audios(clips)):
        assert a.vector.tobytes() == b.vector.tobytes() and a.token_count == b.token_count
