"""GGUF loading failures on CPU (no GPU needed: the file is read and checked before any device
is touched), mirroring GGUFReaderTests and the ModelWeights shape checks
(Tests/GemmaEmbedTests/GGUFReaderTests.swift, Sources/GemmaEmbed/Model/Weights.swift:100-131):
each defect maps to its GemmaEmbedError case."""
import dataclasses
import os
import struct

import pytest


@pytest.fixture(scope="module")
def small(synth):
    arch = synth.make_arch("gemma-embedding", layers=1, vocab=256)
    return arch, synth.build_tensors(arch, 0)


def load_case(ge, path):
    with pytest.raises(ge.GemmaEmbedError) as e:
        ge.EmbeddingModel.load(path)
    return e.value.case


def write(synth, tmp_path, name, arch, tensors, kvs=None):
    path = str(tmp_path / name)
    synth.write_gguf(path, arch, tensors, kvs=kvs)
    return path


def key_of(record: bytes) -> str:
    (n,) = struct.unpack_from("<Q", record, 0)
    return record[8:8 + n].decode()


def test_missing_file(ge, tmp_path):
    assert load_case(ge, str(tmp_path / "absent.gguf")) == "fileNotReadable"


def test_bad_magic(ge, synth, small, tmp_path):
    path = write(synth, tmp_path, "m.gguf", *small)
    data = bytearray(open(path, "rb").read())
    data[:4] = b"GGUX"
    open(path, "wb").write(data)
    assert load_case(ge, path) == "invalidGGUF"


def test_truncated_header(ge, synth, small, tmp_path):
    path = write(synth, tmp_path, "t.gguf", *small)
    data = open(path, "rb").read()
    open(path, "wb").write(data[:200])
    assert load_case(ge, path) == "invalidGGUF"


def test_tensor_data_past_end_of_file(ge, synth, small, tmp_path):
    path = write(synth, tmp_path, "e.gguf", *small)
    size = os.path.getsize(path)
    with open(path, "r+b") as f:
        f.truncate(size - 4096)
    assert load_case(ge, path) == "invalidGGUF"


def test_missing_tensor(ge, synth, small, tmp_path):
    arch, tensors = small
    kept = [t for t in tensors if t.name != "blk.0.ffn_down.weight"]
    assert len(kept) == len(tensors) - 1
    assert load_case(ge, write(synth, tmp_path, "mt.gguf", arch, kept)) == "missingTensor"


def test_tensor_shape_mismatch(ge, synth, small, tmp_path):
    arch, tensors = small
    bad = [dataclasses.replace(t, shape=(t.shape[0], t.shape[1] // 2)) if t.name == "blk.0.attn_output.weight" else t
           for t in tensors]
    assert load_case(ge, write(synth, tmp_path, "sh.gguf", arch, bad)) == "tensorShapeMismatch"


def test_unsupported_tensor_type(ge, synth, small, tmp_path):
    arch, tensors = small
    bad = []
    for t in tensors:
        if t.name == "token_embd.weight":
            n = t.shape[0] * t.shape[1]
            t = dataclasses.replace(t, ggml_type=0, data=b"\0" * (4 * n))  # F32 where Q8_0 is required
        bad.append(t)
    assert load_case(ge, write(synth, tmp_path, "ty.gguf", arch, bad)) == "unsupportedTensorType"


def test_unsupported_architecture(ge, synth, small, tmp_path):
    arch, tensors = small
    kvs = synth.metadata(arch)
    kvs = [synth._kv("general.architecture", 8, synth._str("llama")) if key_of(r) == "general.architecture" else r
           for r in kvs]
    assert load_case(ge, write(synth, tmp_path, "ar.gguf", arch, tensors, kvs)) == "unsupportedArchitecture"


def test_missing_metadata(ge, synth, small, tmp_path):
    arch, tensors = small
    kvs = [r for r in synth.metadata(arch) if not key_of(r).endswith(".block_count")]
    assert load_case(ge, write(synth, tmp_path, "md.gguf", arch, tensors, kvs)) == "missingMetadata"


def test_valid_file_without_a_gpu(ge, synth, small, tmp_path, cuda_available):
    """A well-formed file gets past every check; on a machine without a GPU the load then
    reports noDevice."""
    if cuda_available:
        pytest.skip("a GPU is present: the load succeeds (covered by the GPU tests)")
    assert load_case(ge, write(synth, tmp_path, "ok.gguf", *small)) == "noDevice"
