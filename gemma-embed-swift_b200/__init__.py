"""B200 EmbeddingGemma text encoder behind the reference's EmbeddingModel API.

Python mirror of `Sources/GemmaEmbed/EmbeddingModel.swift`, `EmbedOptions.swift` and
`Tokenizer/Tokenizer.swift` over the C ABI of libgemma_embed_cuda.so (include/gemma_embed.h).
Texts are strings (tokenised by the library's C++ tokenizer from the GGUF vocabulary, behind
the task prefix of `EmbedOptions.task`) or pre-tokenised lists of token ids.

    model = EmbeddingModel.load(path)
    docs = model.embed(["first document", "second document"])    # list[Embedding]
    query = model.embed("a question", EmbedOptions(task=TaskPrefix.query()))
    ids = model.tokenizer.encode("some text")                      # [bos, ..., eos]
    raw = model.embed_tokens([[2, 651, 1]])                        # pooled, unnormalised [n][768]
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import Callable, Optional, Sequence

import numpy as np

from . import _lib

__all__ = ["EmbeddingModel", "EmbedOptions", "LoadOptions", "ImageEmbedOptions", "MultimodalEmbedOptions", "AudioEmbedOptions",
           "AudioInput", "audio_tokens", "audio_to_mono16k", "decode_wav", "Embedding",
           "EmbeddingProgress", "ModelInfo", "GemmaEmbedError", "TaskPrefix", "Tokenizer", "ALLOWED_DIMENSIONS"]

ALLOWED_DIMENSIONS = (768, 512, 256, 128)

# ge_status codes (include/gemma_embed.h) by GemmaEmbedError case (Errors.swift:6-23).
STATUS = {
    0: "ok", 1: "fileNotReadable", 2: "invalidGGUF", 3: "unsupportedTensorType", 4: "unsupportedArchitecture",
    5: "missingTensor", 6: "missingMetadata", 7: "tensorShapeMismatch", 8: "noDevice", 9: "invalidOptions",
    10: "gpuFailure", 11: "outOfMemory", 12: "timeout", 13: "cancelled", 14: "imageDecoding",
    15: "imageEncoderNotLoaded", 16: "audioDecoding", 17: "audioEncoderNotLoaded",
}
LOAD_NO_GRAPHS = 1
LOAD_Q8_ONLY = 2
LOAD_NO_PDL = 4
LOAD_FUSED_RESIDUAL = 8
LOAD_FUSED_QKV = 16
LOAD_SINGLE_CTA_GEMM = 32


class GemmaEmbedError(RuntimeError):
    """A failed call: `.case` names the GemmaEmbedError case, `.code` the ge_status value."""

    def __init__(self, code: int, message: str):
        self.code = code
        self.case = STATUS.get(code, "unknown")
        self.message = message
        super().__init__(f"{self.case}: {message}")


def _text_out(call) -> bytes:
    """Runs `call(buffer, cap, &len)` with the library's buffer convention (the full length comes
    back; a second call gets it all when the first buffer was too small)."""
    n = ctypes.c_int64(0)
    buf = ctypes.create_string_buffer(256)
    call(buf, 256, ctypes.byref(n))
    if n.value > 256:
        buf = ctypes.create_string_buffer(int(n.value))
        call(buf, n.value, ctypes.byref(n))
    return buf.raw[:n.value]


class TaskPrefix:
    """TaskPrefix (EmbedOptions.swift:5-32): each member is the prefix string itself
    (TaskPrefix.prefix), built by the library's ge_task_prefix."""

    DOCUMENT, QUERY, CLUSTERING, CLASSIFICATION, SIMILARITY, NONE = range(6)

    @staticmethod
    def prefix(task: int, arg: Optional[str] = None) -> str:
        L = _lib.lib()
        a = None if arg is None else arg.encode()

        def call(buf, cap, n):
            _check(L.ge_task_prefix(task, a, buf, cap, n))
        return _text_out(call).decode()

    @staticmethod
    def document(title: Optional[str] = None) -> str:
        return TaskPrefix.prefix(TaskPrefix.DOCUMENT, title)

    @staticmethod
    def query(task: Optional[str] = None) -> str:
        return TaskPrefix.prefix(TaskPrefix.QUERY, task)

    clustering = "task: clustering | query: "
    classification = "task: classification | query: "
    similarity = "task: sentence similarity | query: "
    none = ""


@dataclass
class EmbedOptions:
    """EmbedOptions (EmbedOptions.swift:34-56).  `task` is the prefix string (TaskPrefix);
    it applies to string texts, not to pre-tokenised ones."""
    task: str = "title: none | text: "
    max_tokens: int = 2048
    dimensions: int = 768
    normalise: bool = True
    batch_size: Optional[int] = None


class Tokenizer:
    """Tokenizer (Tokenizer/Tokenizer.swift:10-328) of a GGUF file, in the library's C++.

    `Tokenizer.load(path)` reads only the file's tokenizer metadata (no weights, no GPU);
    `EmbeddingModel.tokenizer` is the loaded model's own."""

    def __init__(self, handle, owner=None):
        self._h = handle
        self._owner = owner  # the EmbeddingModel that owns a borrowed handle
        info = _lib.GeTokenizerInfo()
        _check(_lib.lib().ge_tokenizer_get_info(handle, ctypes.byref(info)))
        self.bos_id, self.eos_id, self.pad_id = info.bos_id, info.eos_id, info.pad_id
        self.unknown_id = None if info.unknown_id < 0 else info.unknown_id
        self.vocabulary_size = info.vocabulary_size
        self.add_bos, self.add_eos = bool(info.add_bos), bool(info.add_eos)

    @classmethod
    def load(cls, path: str) -> "Tokenizer":
        """Tokenizer(gguf:) (Tokenizer.swift:40-56)."""
        h = ctypes.c_void_p()
        _check(_lib.lib().ge_tokenizer_load(str(path).encode(), ctypes.byref(h)), None)
        return cls(h)

    def close(self):
        if self._h and self._owner is None:
            _lib.lib().ge_tokenizer_free(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, text, add_special_tokens: bool = True, parse_special_tokens: bool = False) -> list:
        """encode(_:addSpecialTokens:parseSpecialTokens:) (Tokenizer.swift:105-117); `text` is a
        str or UTF-8 bytes."""
        data = text.encode() if isinstance(text, str) else bytes(text)
        flags = (1 if add_special_tokens else 0) | (2 if parse_special_tokens else 0)
        L = _lib.lib()
        n = ctypes.c_int64(0)
        cap = len(data) + 8
        out = np.zeros(cap, dtype=np.int32)
        _check(L.ge_tokenize(self._h, data, len(data), flags, _ptr(out, ctypes.c_int32), cap, ctypes.byref(n)))
        if n.value > cap:
            out = np.zeros(int(n.value), dtype=np.int32)
            _check(L.ge_tokenize(self._h, data, len(data), flags, _ptr(out, ctypes.c_int32), n.value, ctypes.byref(n)))
        return out[:n.value].tolist()

    def decode_bytes(self, ids) -> bytes:
        """decode(_:) (Tokenizer.swift:120-147) as UTF-8 bytes."""
        a = _i32(ids)
        L = _lib.lib()

        def call(buf, cap, n):
            _check(L.ge_detokenize(self._h, _ptr(a, ctypes.c_int32), len(a), buf, cap, n))
        return _text_out(call)

    def decode(self, ids) -> str:
        """decode(_:): invalid UTF-8 left by split byte tokens shows as U+FFFD, as
        String(decoding:as:) does."""
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def piece(self, token_id: int) -> Optional[str]:
        """piece(_:) (Tokenizer.swift:150-153): None outside the vocabulary."""
        if not 0 <= token_id < self.vocabulary_size:
            return None
        L = _lib.lib()

        def call(buf, cap, n):
            _check(L.ge_token_piece(self._h, token_id, buf, cap, n))
        return _text_out(call).decode("utf-8", errors="replace")

    def is_control(self, token_id: int) -> bool:
        """isControl(_:) (Tokenizer.swift:155-158)."""
        return bool(_lib.lib().ge_token_is_control(self._h, token_id))


@dataclass
class LoadOptions:
    """LoadOptions (EmbedOptions.swift:171-203): the fields a text forward uses, plus devices."""
    batch_token_budget: int = 8192
    devices: Sequence[int] = (0,)
    use_graphs: bool = True
    q8_only: bool = False
    programmatic_launch: bool = True  # overlap each kernel's set-up with its predecessor's tail
    fused_residual: bool = False  # run each residual step inside the projection before it
    fused_qkv: bool = False  # run the q/k/v norms and RoPE inside the q/k/v projection (head dim 256)
    cta_pair_gemm: bool = True  # large batches' projections on CTA pairs (256 x 256 tiles); bit-identical
    image_encoder: Optional[str] = None  # LoadOptions.imageEncoder: the mmproj GGUF
    image_patch_budget: int = 4096       # ImageEmbedOptions.patchBudget: patches per image batch
    audio_encoder: Optional[str] = None  # LoadOptions.audioEncoder: the mmproj GGUF with a gemma4a tower
    audio_frame_budget: int = 96000      # log-mel frames per audio batch (AudioEmbedOptions.frameBudget)


@dataclass
class MultimodalEmbedOptions:
    """MultimodalEmbedOptions (EmbedOptions.swift:117-147)."""
    task: str = "title: none | text: "
    max_tokens: int = 2048
    dimensions: int = 768
    normalise: bool = True
    max_image_tokens: int = 256
    batch_size: Optional[int] = None


@dataclass
class ImageEmbedOptions:
    """ImageEmbedOptions (EmbedOptions.swift:59-88)."""
    dimensions: int = 768
    normalise: bool = True
    max_image_tokens: int = 256
    batch_size: Optional[int] = None


@dataclass
class AudioEmbedOptions:
    """AudioEmbedOptions (EmbedOptions.swift:91-114)."""
    dimensions: int = 768
    normalise: bool = True
    max_tokens: Optional[int] = None  # None: the model's limit
    batch_size: Optional[int] = None


@dataclass
class Embedding:
    vector: np.ndarray
    token_count: int
    truncated: bool


@dataclass
class EmbeddingProgress:
    completed_texts: int
    total_texts: int
    completed_tokens: int


@dataclass
class ModelInfo:
    architecture: str
    name: str
    layer_count: int
    hidden_size: int
    output_dimensions: int
    feed_forward_size: int
    per_layer_input_size: int
    head_count: int
    vocabulary_size: int
    sliding_window: int
    max_tokens: int
    norm_epsilon: float
    quantization: str
    file_size: int
    device_count: int
    device_name: str
    eos_id: int
    bos_id: int
    # ImageEncoderInfo (VisionConfig.swift:5-17); zeros without an image encoder.
    image_layer_count: int = 0
    image_hidden_size: int = 0
    image_patch_size: int = 0
    image_projection_dim: int = 0
    # AudioEncoderInfo (AudioConfig.swift:5-19); zeros without an audio encoder.
    audio_layer_count: int = 0
    audio_hidden_size: int = 0
    audio_head_count: int = 0
    audio_feed_forward_size: int = 0
    audio_mel_bins: int = 0
    audio_projection_dim: int = 0


AUDIO_SAMPLE_RATE = 16000


def audio_tokens(samples: int) -> int:
    """AudioFrontEnd.tokenCount(samples:) (Audio/AudioPreprocessor.swift:86-95)."""
    return int(_lib.lib().ge_audio_tokens(int(samples)))


class AudioInput:
    """A sound to embed (AudioInput, Audio/AudioInput.swift:6-14): WAV bytes (`data`), a WAV file
    (`url`) or PCM samples (`samples`).  The library decodes WAV itself as dr_wav does; other
    containers, which the reference hands to AVFoundation, must be decoded to samples first."""

    def __init__(self, kind: str, value, sample_rate: int = AUDIO_SAMPLE_RATE, channels: int = 1):
        self.kind, self.value, self.sample_rate, self.channels = kind, value, sample_rate, channels

    @classmethod
    def data(cls, data: bytes) -> "AudioInput":
        return cls("data", bytes(data))

    @classmethod
    def url(cls, path) -> "AudioInput":
        return cls("url", os.fspath(path))

    @classmethod
    def samples(cls, samples, sample_rate: int, channels: int = 1) -> "AudioInput":
        return cls("samples", samples, sample_rate, channels)


def decode_wav(data: bytes):
    """WAVDecoder.decode (Audio/WAVDecoder.swift:29-84): the interleaved float32 samples of a
    RIFF/WAVE file (frames x channels, flattened), its sample rate and its channel count."""
    L = _lib.lib()
    buf = (ctypes.c_uint8 * max(len(data), 1)).from_buffer_copy(bytes(data) or b"\0")
    frames, rate, ch = ctypes.c_int64(0), ctypes.c_int32(0), ctypes.c_int32(0)
    refs = (ctypes.byref(frames), ctypes.byref(rate), ctypes.byref(ch))
    rc = L.ge_audio_decode_wav(buf, len(data), None, 0, *refs)
    if rc != 0:
        raise GemmaEmbedError(rc, (L.ge_last_error(None) or b"").decode())
    out = np.zeros(max(frames.value * ch.value, 1), np.float32)
    _check(L.ge_audio_decode_wav(buf, len(data), _ptr(out, ctypes.c_float), out.size, *refs), None)
    return out[:frames.value * ch.value], rate.value, ch.value


def audio_to_mono16k(samples, sample_rate: int = AUDIO_SAMPLE_RATE, channels: int = 1) -> np.ndarray:
    """AudioDecoder.decode (Audio/AudioDecoder.swift:17-41) without the embedding: interleaved
    float samples at any rate and channel count (or an AudioInput) as the 16 kHz mono samples the
    audio encoder reads, converted as MiniaudioConverter.toMono16k
    (Audio/MiniaudioConverter.swift:23-37) converts them."""
    clip = samples if isinstance(samples, AudioInput) else (samples, sample_rate, channels)
    c, keep = _audios([clip])
    n = ctypes.c_int64(0)
    L = _lib.lib()
    if L.ge_audio_convert(c, None, 0, ctypes.byref(n)) != 0:
        raise GemmaEmbedError(16, (L.ge_last_error(None) or b"").decode())
    out = np.zeros(max(n.value, 1), np.float32)
    _check(L.ge_audio_convert(c, _ptr(out, ctypes.c_float), n.value, ctypes.byref(n)), None)
    return out[:n.value]


def _read_audio_file(path: str):
    """AudioDecoder.decode's `.url` case (Audio/AudioDecoder.swift:19-26): a WAV file's samples,
    with the path in front of the reason when it cannot be read or decoded."""
    try:
        with open(path, "rb") as f:
            data = f.read()
    except OSError:
        raise GemmaEmbedError(16, f"cannot decode audio: {path} is not readable") from None
    if not (len(data) >= 12 and data[:4] == b"RIFF" and data[8:12] == b"WAVE"):
        raise GemmaEmbedError(16, f"cannot decode audio: {path}: not a WAV file; other containers (MP3, M4A, "
                                  "AIFF, CAF, FLAC) must be decoded to samples by the caller")
    try:
        return decode_wav(data)
    except GemmaEmbedError as e:
        raise GemmaEmbedError(e.code, e.message.replace("cannot decode audio: ", f"cannot decode audio: {path}: ", 1)) from None


def _audios(clips):
    """ge_audio views of the clips (kept alive by the returned list): 16 kHz mono float32 sample
    arrays, (samples, sample_rate, channels) tuples or AudioInput values."""
    c = (_lib.GeAudio * max(len(clips), 1))()
    keep = []
    for i, clip in enumerate(clips):
        rate, channels = AUDIO_SAMPLE_RATE, 1
        if isinstance(clip, AudioInput):
            if clip.kind == "data":
                b = (ctypes.c_uint8 * max(len(clip.value), 1)).from_buffer_copy(clip.value or b"\0")
                keep.append(b)
                c[i].wav = ctypes.cast(b, ctypes.POINTER(ctypes.c_uint8))
                c[i].wav_bytes = len(clip.value)
                continue
            if clip.kind == "url":
                clip, rate, channels = _read_audio_file(clip.value)
            else:
                clip, rate, channels = clip.value, clip.sample_rate, clip.channels
        elif isinstance(clip, tuple):
            clip, rate, channels = clip
        a = np.ascontiguousarray(np.asarray(clip, dtype=np.float32).reshape(-1))
        if channels > 0 and a.size % int(channels):
            raise GemmaEmbedError(16, f"cannot decode audio: {a.size} samples do not split over {int(channels)} channels")
        keep.append(a)
        c[i].samples = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        c[i].count = a.size // max(int(channels), 1) if channels > 0 else a.size
        c[i].sample_rate = int(rate)
        c[i].channels = int(channels)
    return c, keep


def _images(images):
    """ge_image views of HxWx3 uint8 arrays (kept alive by the returned list)."""
    arrs = [np.ascontiguousarray(np.asarray(im, dtype=np.uint8)) for im in images]
    for a in arrs:
        if a.ndim != 3 or a.shape[2] != 3:
            raise GemmaEmbedError(14, "imageDecoding: an image must be a height x width x 3 array of uint8")
    c = (_lib.GeImage * max(len(arrs), 1))()
    for i, a in enumerate(arrs):
        c[i].rgb = a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))
        c[i].width = a.shape[1]
        c[i].height = a.shape[0]
    return c, arrs


def _check(rc: int, handle=None):
    if rc != 0:
        msg = _lib.lib().ge_last_error(handle)
        raise GemmaEmbedError(rc, msg.decode() if msg else "")


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


def _id_arrays(data) -> tuple:
    """Token-id arrays for ge_embed_tokens: the texts' ids in one int32 buffer, their lengths,
    and each text's address in that buffer (uintp), computed from the offsets with one ctypes
    conversion per call instead of one per text (about 2.5 us each).  The addresses are valid
    while the returned buffer is alive."""
    n = len(data)
    lens = np.fromiter((len(s) for s in data), dtype=np.int32, count=n)
    flat = np.concatenate(data) if n > 1 else data[0]
    starts = np.zeros(n, dtype=np.int64)
    np.cumsum(lens[:-1], out=starts[1:])
    addrs = (flat.ctypes.data + 4 * starts).astype(np.uintp)
    return flat, lens, addrs


def pack(sequences) -> tuple:
    """PackedBatch.append over `sequences` (MetalForward.swift:17-21): ids, positions, ranges."""
    seqs = [_i32(s) for s in sequences]
    lens = [len(s) for s in seqs]
    tokens = np.concatenate(seqs) if seqs else np.zeros(0, np.int32)
    positions = np.concatenate([np.arange(n, dtype=np.int32) for n in lens]) if seqs else np.zeros(0, np.int32)
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64) if seqs else np.zeros(0, np.int64)
    return tokens, positions, [(int(s), int(n)) for s, n in zip(starts, lens)]


class EmbeddingModel:
    """EmbeddingModel (EmbeddingModel.swift:24-290) on one or more B200 GPUs."""

    def __init__(self, handle, options: LoadOptions):
        self._h = handle
        self._tokenizer = None
        self.options = options
        info = _lib.GeInfo()
        _check(_lib.lib().ge_info_get(handle, ctypes.byref(info)), handle)
        self.info = ModelInfo(
            architecture=info.architecture.decode(), name=info.name.decode(), layer_count=info.layer_count,
            hidden_size=info.hidden_size, output_dimensions=info.output_dimensions,
            feed_forward_size=info.feed_forward_size, per_layer_input_size=info.per_layer_input_size,
            head_count=info.head_count, vocabulary_size=info.vocabulary_size, sliding_window=info.sliding_window,
            max_tokens=info.max_tokens, norm_epsilon=info.norm_epsilon, quantization=info.quantization.decode(),
            file_size=info.file_size, device_count=info.device_count, device_name=info.device_name.decode(),
            eos_id=info.eos_id, bos_id=info.bos_id, image_layer_count=info.image_layer_count,
            image_hidden_size=info.image_hidden_size, image_patch_size=info.image_patch_size,
            image_projection_dim=info.image_projection_dim, audio_layer_count=info.audio_layer_count,
            audio_hidden_size=info.audio_hidden_size, audio_head_count=info.audio_head_count,
            audio_feed_forward_size=info.audio_feed_forward_size, audio_mel_bins=info.audio_mel_bins,
            audio_projection_dim=info.audio_projection_dim)

    def counters(self) -> dict:
        """The library's running counts for this model (ge_info_get): kernel launches, bytes
        copied host to device and back by the forwards, and CUDA graphs captured."""
        info = _lib.GeInfo()
        _check(_lib.lib().ge_info_get(self._h, ctypes.byref(info)), self._h)
        return {"kernel_launches": int(info.kernel_launches), "host_to_device_bytes": int(info.host_to_device_bytes),
                "device_to_host_bytes": int(info.device_to_host_bytes), "graph_captures": int(info.graph_captures)}

    @classmethod
    def load(cls, path: str, options: Optional[LoadOptions] = None) -> "EmbeddingModel":
        """EmbeddingModel.load(from:options:) (EmbeddingModel.swift:40-122)."""
        options = options or LoadOptions()
        L = _lib.lib()
        o = _lib.GeLoadOpts()
        L.ge_load_opts_default(ctypes.byref(o))
        mask = 0
        for d in options.devices:
            mask |= 1 << int(d)
        o.device_mask = mask
        o.batch_token_budget = int(options.batch_token_budget)
        o.flags = ((0 if options.use_graphs else LOAD_NO_GRAPHS) | (LOAD_Q8_ONLY if options.q8_only else 0)
                   | (0 if options.programmatic_launch else LOAD_NO_PDL)
                   | (LOAD_FUSED_RESIDUAL if options.fused_residual else 0)
                   | (LOAD_FUSED_QKV if options.fused_qkv else 0)
                   | (0 if options.cta_pair_gemm else LOAD_SINGLE_CTA_GEMM))
        o.image_encoder_path = str(options.image_encoder).encode() if options.image_encoder else None
        o.image_patch_budget = int(options.image_patch_budget)
        o.audio_encoder_path = str(options.audio_encoder).encode() if options.audio_encoder else None
        o.audio_frame_budget = int(options.audio_frame_budget)
        h = ctypes.c_void_p()
        _check(L.ge_load(str(path).encode(), ctypes.byref(o), ctypes.byref(h)), None)
        return cls(h, options)

    @property
    def tokenizer(self) -> Tokenizer:
        """EmbeddingModel.tokenizer (EmbeddingModel.swift:26)."""
        if self._tokenizer is None:
            h = _lib.lib().ge_model_tokenizer(self._h)
            if not h:
                raise GemmaEmbedError(4, "unsupportedArchitecture: tokenizer model missing")
            self._tokenizer = Tokenizer(ctypes.c_void_p(h), owner=self)
        return self._tokenizer

    def close(self):
        if self._tokenizer is not None:
            self._tokenizer._h = None
            self._tokenizer = None
        if self._h:
            _lib.lib().ge_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -------------------------------------------------------------- forward entry points
    def forward_packed(self, tokens, positions, seqs) -> np.ndarray:
        """MetalForward.run over one PackedBatch: pooled, unnormalised [nseq][output_dimensions]."""
        tokens = _i32(tokens)
        pos = None if positions is None else _i32(positions)
        arr = (_lib.GeSeq * max(len(seqs), 1))(*[_lib.GeSeq(int(s), int(n)) for s, n in seqs])
        out = np.zeros((len(seqs), self.info.output_dimensions), dtype=np.float32)
        _check(_lib.lib().ge_forward_packed(self._h, _ptr(tokens, ctypes.c_int32),
                                           None if pos is None else _ptr(pos, ctypes.c_int32), len(tokens), arr,
                                           len(seqs), _ptr(out, ctypes.c_float)), self._h)
        return out

    def embed_tokens(self, sequences) -> np.ndarray:
        """embedTokens (EmbeddingModel.swift:285-289): pooled, unnormalised vectors."""
        tokens, positions, seqs = pack(sequences)
        return self.forward_packed(tokens, positions, seqs)

    def forward_device(self, d_tokens, seqs, d_out, stream=None, device: int = 0) -> None:
        """The forward over device-resident ids: torch int32 / float32 CUDA tensors or raw pointers."""
        tp = d_tokens.data_ptr() if hasattr(d_tokens, "data_ptr") else int(d_tokens)
        op = d_out.data_ptr() if hasattr(d_out, "data_ptr") else int(d_out)
        ntok = int(sum(n for _, n in seqs))
        # A torch stream, a raw cudaStream_t, or None for the legacy default stream.
        sp = stream.cuda_stream if hasattr(stream, "cuda_stream") else (stream or 0)
        arr = (_lib.GeSeq * max(len(seqs), 1))(*[_lib.GeSeq(int(s), int(n)) for s, n in seqs])
        _check(_lib.lib().ge_forward_device(self._h, device, ctypes.c_void_p(tp), ntok, arr, len(seqs),
                                           ctypes.c_void_p(op), ctypes.c_void_p(sp)), self._h)

    def profile(self, tokens, seqs, reps: int = 10) -> list:
        """Profiler.profile (Metal/Profiler.swift:16-88): per kernel class, mean ms per launch over
        `reps` back-to-back launches, algorithmic FLOPs and bytes per launch, launches per forward."""
        tokens = _i32(tokens)
        arr = (_lib.GeSeq * max(len(seqs), 1))(*[_lib.GeSeq(int(s), int(n)) for s, n in seqs])
        cap = 64
        out = (_lib.GeKernelTime * cap)()
        cnt = ctypes.c_int32(0)
        _check(_lib.lib().ge_profile(self._h, _ptr(tokens, ctypes.c_int32), len(tokens), arr, len(seqs), reps, out, cap,
                                    ctypes.byref(cnt)), self._h)
        return [{"name": out[i].name.decode(), "ms_per_launch": out[i].ms_per_launch,
                 "flops_per_launch": out[i].flops_per_launch, "bytes_per_launch": out[i].bytes_per_launch,
                 "launches_per_forward": out[i].launches_per_forward} for i in range(cnt.value)]

    def profile_images(self, images, max_image_tokens: int = 256, reps: int = 5) -> list:
        """Profiler.profileImages (Metal/Profiler.swift:114-200): "image_forward" (vision and text
        towers) and "vision_tower" in ms, then each vision kernel class like `profile`."""
        c, keep = _images(list(images))
        cap = 64
        out = (_lib.GeKernelTime * cap)()
        cnt = ctypes.c_int32(0)
        _check(_lib.lib().ge_profile_images(self._h, c, len(keep), max_image_tokens, reps, out, cap, ctypes.byref(cnt)),
               self._h)
        return [{"name": out[i].name.decode(), "ms_per_launch": out[i].ms_per_launch,
                 "flops_per_launch": out[i].flops_per_launch, "bytes_per_launch": out[i].bytes_per_launch,
                 "launches_per_forward": out[i].launches_per_forward} for i in range(cnt.value)]

    def image_forward_device(self, d_rgb, sizes, d_out, stream=None, device: int = 0) -> None:
        """ge_image_forward_device: pixels already on the GPU (`d_rgb`, images back to back at their
        tower sizes (width, height) in `sizes`) to pooled rows in `d_out`, on `stream`."""
        c = (_lib.GeImage * max(len(sizes), 1))()
        for i, (w, h) in enumerate(sizes):
            c[i].width = int(w)
            c[i].height = int(h)
        _check(_lib.lib().ge_image_forward_device(self._h, device, ctypes.c_void_p(int(d_rgb)), c, len(sizes),
                                                  ctypes.c_void_p(int(d_out)), ctypes.c_void_p(int(stream or 0))),
               self._h)

    def pool_head_noalloc(self, d_hidden, ntok: int, d_seqs, nseq: int, d_out, stream=None, device: int = 0) -> None:
        """Mean-pool and head over caller-owned device buffers without allocating (ge_pool_head_noalloc),
        for callers that cannot allocate device memory.  Arguments are torch CUDA tensors or raw
        device pointers: d_hidden [ntok][hidden] fp32, d_seqs [nseq][2] uint32/int32 (start, length),
        d_out [nseq][output_dimensions] fp32.  At most 128 sequences per call."""
        ptr = lambda t: t.data_ptr() if hasattr(t, "data_ptr") else int(t)
        sp = stream.cuda_stream if hasattr(stream, "cuda_stream") else (stream or 0)
        _check(_lib.lib().ge_pool_head_noalloc(self._h, device, ctypes.c_void_p(ptr(d_hidden)), ntok,
                                              ctypes.c_void_p(ptr(d_seqs)), nseq, ctypes.c_void_p(ptr(d_out)),
                                              ctypes.c_void_p(sp)), self._h)

    def trace(self, tokens, layer: int) -> np.ndarray:
        """The residual stream after `layer` ("l_out-<layer>"), or result_norm for layer -1: [ntok][hidden]."""
        tokens = _i32(tokens)
        out = np.zeros((len(tokens), self.info.hidden_size), dtype=np.float32)
        _check(_lib.lib().ge_forward_trace(self._h, _ptr(tokens, ctypes.c_int32), len(tokens), layer,
                                          _ptr(out, ctypes.c_float)), self._h)
        return out

    # -------------------------------------------------------------- EmbeddingModel API
    def embed(self, texts, options: Optional[EmbedOptions] = None,
              progress: Optional[Callable[[EmbeddingProgress], Optional[bool]]] = None) -> list:
        """embed(_ texts:options:progress:) (EmbeddingModel.swift:145-175).

        `texts` is a str (one text, returns one Embedding), a list of str, a list of ints (one
        pre-tokenised text) or a list of int lists.  Strings get `options.task` in front and
        are tokenised by the library; token ids are taken as they are.  `progress` runs after
        every batch; returning True cancels the call between batches (GemmaEmbedError
        'cancelled')."""
        options = options or EmbedOptions()
        if options.batch_size is not None and options.batch_size < 1:
            raise GemmaEmbedError(9, "invalid options: batchSize must be at least 1")
        as_text = isinstance(texts, (str, bytes)) or (len(texts) > 0 and isinstance(texts[0], (str, bytes)))
        single = isinstance(texts, (str, bytes)) or (len(texts) > 0 and np.isscalar(texts[0]) and not as_text)
        if as_text:
            items = [texts] if single else list(texts)
            data = [t.encode() if isinstance(t, str) else bytes(t) for t in items]
        else:
            data = [_i32(texts)] if single else [_i32(t) for t in texts]
        n = len(data)
        dims = options.dimensions
        o = _lib.GeEmbedOpts(options.max_tokens, dims, int(options.normalise), options.batch_size or 0)
        L = _lib.lib()
        if n == 0:
            _check(L.ge_embed_tokens(self._h, None, None, 0, ctypes.byref(o), None, None, None,
                                     _lib.PROGRESS_FN(0), None), self._h)
            return []
        out = np.zeros((n, dims if dims > 0 else 1), dtype=np.float32)
        counts = np.zeros(n, dtype=np.int32)
        trunc = np.zeros(n, dtype=np.int32)
        cb = _lib.PROGRESS_FN(0)
        if progress is not None:
            def _cb(done, total, tokens, user):
                return 1 if progress(EmbeddingProgress(done, total, tokens)) else 0
            cb = _lib.PROGRESS_FN(_cb)
        if as_text:
            ptrs = (ctypes.c_char_p * n)(*data)
            lens = np.array([len(d) for d in data], dtype=np.int64)
            _check(L.ge_embed_texts(self._h, ptrs, _ptr(lens, ctypes.c_int64), n, options.task.encode(),
                                    ctypes.byref(o), _ptr(out, ctypes.c_float), _ptr(counts, ctypes.c_int32),
                                    _ptr(trunc, ctypes.c_int32), cb, None), self._h)
        else:
            flat, lens, addrs = _id_arrays(data)  # `flat` stays alive through the call
            _check(L.ge_embed_tokens(self._h, addrs.ctypes.data_as(ctypes.POINTER(_lib.i32p)),
                                     _ptr(lens, ctypes.c_int32), n, ctypes.byref(o),
                                     _ptr(out, ctypes.c_float), _ptr(counts, ctypes.c_int32),
                                     _ptr(trunc, ctypes.c_int32), cb, None), self._h)
        # Each vector is its own row of `out` (rows are disjoint views, not copies).
        res = [Embedding(v, c, bool(t)) for v, c, t in zip(out, counts.tolist(), trunc.tolist())]
        return res[0] if single else res

    def embed_images(self, images, options: Optional[ImageEmbedOptions] = None,
                     progress: Optional[Callable[[EmbeddingProgress], Optional[bool]]] = None) -> list:
        """embed(images:options:progress:) (ImageEmbedding.swift:17-33) over decoded images, each a
        height x width x 3 uint8 array; a single array embeds one image and returns one Embedding."""
        options = options or ImageEmbedOptions()
        single = isinstance(images, np.ndarray) and images.ndim == 3
        items = [images] if single else list(images)
        c, keep = _images(items)
        n = len(items)
        if options.batch_size is not None and options.batch_size < 1:
            raise GemmaEmbedError(9, "invalid options: batchSize must be at least 1")
        o = _lib.GeImageOpts(options.dimensions, int(options.normalise), options.max_image_tokens,
                             options.batch_size or 0)
        out = np.zeros((max(n, 1), options.dimensions if options.dimensions > 0 else 1), dtype=np.float32)
        counts = np.zeros(max(n, 1), dtype=np.int32)
        cb = _lib.PROGRESS_FN(0)
        if progress is not None:
            def _cb(done, total, tokens, user):
                return 1 if progress(EmbeddingProgress(done, total, tokens)) else 0
            cb = _lib.PROGRESS_FN(_cb)
        _check(_lib.lib().ge_embed_images(self._h, c, n, ctypes.byref(o), _ptr(out, ctypes.c_float),
                                          _ptr(counts, ctypes.c_int32), cb, None), self._h)
        del keep
        res = [Embedding(out[i].copy(), int(counts[i]), False) for i in range(n)]
        return res[0] if single else res

    def embed_multimodal(self, inputs, options: Optional[MultimodalEmbedOptions] = None,
                         progress: Optional[Callable[[EmbeddingProgress], Optional[bool]]] = None) -> list:
        """embed(_ inputs: [MultimodalInput], options:progress:) (MultimodalEmbedding.swift:100-206).
        Each input is a list of parts in reading order: str (text), a height x width x 3 uint8
        array (an image), or a 1-D float32 array of 16 kHz mono samples, a (samples, rate,
        channels) tuple or an AudioInput (a clip)."""
        options = options or MultimodalEmbedOptions()
        if options.batch_size is not None and options.batch_size < 1:
            raise GemmaEmbedError(9, "invalid options: batchSize must be at least 1")
        keep, arrays = [], []
        c_inputs = (_lib.GeMultimodalInput * max(len(inputs), 1))()
        for i, parts in enumerate(inputs):
            cp = (_lib.GePart * max(len(parts), 1))()
            for k, part in enumerate(parts):
                if isinstance(part, (str, bytes)):
                    data = part.encode() if isinstance(part, str) else bytes(part)
                    keep.append(data)
                    cp[k].kind, cp[k].text, cp[k].text_len = 0, data, len(data)
                elif isinstance(part, (tuple, AudioInput)) or np.asarray(part).ndim == 1:
                    c, arrs = _audios([part])
                    arrays.append(arrs)
                    cp[k].kind = 2
                    cp[k].audio = c[0]
                else:
                    c, arrs = _images([part])
                    arrays.append(arrs)
                    cp[k].kind = 1
                    cp[k].image = c[0]
            keep.append(cp)
            c_inputs[i].parts = cp
            c_inputs[i].count = len(parts)
        n = len(inputs)
        o = _lib.GeMultimodalOpts(options.max_tokens, options.dimensions, int(options.normalise),
                                  options.max_image_tokens, options.batch_size or 0)
        out = np.zeros((max(n, 1), options.dimensions if options.dimensions > 0 else 1), dtype=np.float32)
        counts = np.zeros(max(n, 1), dtype=np.int32)
        trunc = np.zeros(max(n, 1), dtype=np.int32)
        cb = _lib.PROGRESS_FN(0)
        if progress is not None:
            def _cb(done, total, tokens, user):
                return 1 if progress(EmbeddingProgress(done, total, tokens)) else 0
            cb = _lib.PROGRESS_FN(_cb)
        _check(_lib.lib().ge_embed_multimodal(self._h, c_inputs, n, options.task.encode(), ctypes.byref(o),
                                              _ptr(out, ctypes.c_float), _ptr(counts, ctypes.c_int32),
                                              _ptr(trunc, ctypes.c_int32), cb, None), self._h)
        del keep, arrays
        return [Embedding(out[i].copy(), int(counts[i]), bool(trunc[i])) for i in range(n)]

    def embed_audios(self, clips, options: Optional[AudioEmbedOptions] = None,
                     progress: Optional[Callable[[EmbeddingProgress], Optional[bool]]] = None) -> list:
        """embed(audios:options:progress:) (AudioEmbedding.swift:17-33) over clips: 16 kHz mono
        float32 arrays, (interleaved samples, rate, channels) tuples at any rate and channel count
        (converted as audio_to_mono16k does) or AudioInput values (WAV bytes or files); a single
        1-D array or AudioInput embeds one clip and returns one Embedding."""
        options = options or AudioEmbedOptions()
        single = (isinstance(clips, np.ndarray) and clips.ndim == 1) or isinstance(clips, AudioInput)
        items = [clips] if single else list(clips)
        c, keep = _audios(items)
        n = len(items)
        if options.batch_size is not None and options.batch_size < 1:
            raise GemmaEmbedError(9, "invalid options: batchSize must be at least 1")
        o = _lib.GeAudioOpts(options.dimensions, int(options.normalise), options.max_tokens or 0,
                             options.batch_size or 0)
        out = np.zeros((max(n, 1), options.dimensions if options.dimensions > 0 else 1), dtype=np.float32)
        counts = np.zeros(max(n, 1), dtype=np.int32)
        cb = _lib.PROGRESS_FN(0)
        if progress is not None:
            def _cb(done, total, tokens, user):
                return 1 if progress(EmbeddingProgress(done, total, tokens)) else 0
            cb = _lib.PROGRESS_FN(_cb)
        _check(_lib.lib().ge_embed_audios(self._h, c, n, ctypes.byref(o), _ptr(out, ctypes.c_float),
                                          _ptr(counts, ctypes.c_int32), cb, None), self._h)
        del keep
        res = [Embedding(out[i].copy(), int(counts[i]), False) for i in range(n)]
        return res[0] if single else res

    def audio_vectors(self, clips) -> list:
        """The audio tower's projected rows of each clip (MetalForward's audio rows)."""
        items = list(clips)
        c, keep = _audios(items)
        n = len(items)
        L = _lib.lib()
        per = [int(L.ge_audio_tokens(int(c[i].count))) for i in range(n)]
        cap = max(sum(per), 1)
        out = np.zeros((cap, self.info.audio_projection_dim or 1), dtype=np.float32)
        rows = np.zeros(max(n, 1), dtype=np.int32)
        _check(L.ge_audio_vectors(self._h, c, n, _ptr(out, ctypes.c_float), cap, _ptr(rows, ctypes.c_int32)), self._h)
        del keep
        res, r0 = [], 0
        for i in range(n):
            res.append(out[r0:r0 + rows[i]].copy())
            r0 += int(rows[i])
        return res

    def audio_forward_device(self, d_pcm, counts, d_out, stream=None, device: int = 0) -> None:
        """ge_audio_forward_device: 16 kHz samples already on the GPU (`d_pcm`, clips back to back with
        the sample counts in `counts`) to pooled rows in `d_out`, on `stream`."""
        c = (_lib.GeAudio * max(len(counts), 1))()
        for i, n in enumerate(counts):
            c[i].count = int(n)
            c[i].sample_rate = AUDIO_SAMPLE_RATE
            c[i].channels = 1
        _check(_lib.lib().ge_audio_forward_device(self._h, device, ctypes.c_void_p(int(d_pcm)), c, len(counts),
                                                  ctypes.c_void_p(int(d_out)), ctypes.c_void_p(int(stream or 0))),
               self._h)

    def profile_audios(self, clips, reps: int = 5) -> list:
        """Profiler.profileAudio (Metal/Profiler.swift:202-295): "audio_forward" (audio and text
        towers) and "audio_tower" in ms, then each audio kernel class like `profile`."""
        c, keep = _audios(list(clips))
        cap = 64
        out = (_lib.GeKernelTime * cap)()
        cnt = ctypes.c_int32(0)
        _check(_lib.lib().ge_profile_audios(self._h, c, len(keep), reps, out, cap, ctypes.byref(cnt)), self._h)
        return [{"name": out[i].name.decode(), "ms_per_launch": out[i].ms_per_launch,
                 "flops_per_launch": out[i].flops_per_launch, "bytes_per_launch": out[i].bytes_per_launch,
                 "launches_per_forward": out[i].launches_per_forward} for i in range(cnt.value)]

    def image_vectors(self, images, max_image_tokens: int = 256) -> list:
        """MetalForward.imageVectors (Metal/MetalForward.swift:227-238): each image's projected rows."""
        items = list(images)
        c, keep = _images(items)
        n = len(items)
        L = _lib.lib()
        per = [L.ge_image_tokens(self._h, a.shape[1], a.shape[0], max_image_tokens) for a in keep]
        if any(t < 0 for t in per):
            raise GemmaEmbedError(15, "imageEncoderNotLoaded: no image encoder is loaded")
        cap = max(sum(per), 1)
        out = np.zeros((cap, self.info.image_projection_dim or 1), dtype=np.float32)
        rows = np.zeros(max(n, 1), dtype=np.int32)
        _check(L.ge_image_vectors(self._h, c, n, max_image_tokens, _ptr(out, ctypes.c_float), cap,
                                  _ptr(rows, ctypes.c_int32)), self._h)
        del keep
        res, r0 = [], 0
        for i in range(n):
            res.append(out[r0:r0 + rows[i]].copy())
            r0 += int(rows[i])
        return res

    @staticmethod
    def similarity(a: Embedding, b: Embedding) -> float:
        """Dot product of the common prefix (EmbeddingModel.swift:178-182)."""
        k = min(len(a.vector), len(b.vector))
        return float(np.dot(a.vector[:k].astype(np.float32), b.vector[:k].astype(np.float32)))

    @staticmethod
    def batches(costs, batch_size: Optional[int], budgets) -> list:
        """EmbeddingModel.batches (EmbeddingModel.swift:200-215) as a list of ranges."""
        n, k = len(costs), len(budgets)
        c = np.ascontiguousarray(np.array(costs, dtype=np.int64).reshape(n, k)) if n else np.zeros((0, k), np.int64)
        b = np.ascontiguousarray(np.array(budgets, dtype=np.int64))
        out = np.zeros(max(2 * n, 2), dtype=np.int32)
        cnt = ctypes.c_int32(0)
        _check(_lib.lib().ge_batches(_ptr(c, ctypes.c_int64), n, k, batch_size or 0, _ptr(b, ctypes.c_int64),
                                    _ptr(out, ctypes.c_int32), ctypes.byref(cnt)))
        return [range(int(out[2 * i]), int(out[2 * i + 1])) for i in range(cnt.value)]

    @staticmethod
    def finish(vector, dimensions: int, normalise: bool) -> np.ndarray:
        """EmbeddingModel.finish (EmbeddingModel.swift:260-267)."""
        v = np.ascontiguousarray(np.asarray(vector, dtype=np.float32))
        out = np.zeros(min(dimensions, len(v)), dtype=np.float32)
        _check(_lib.lib().ge_finish(_ptr(v, ctypes.c_float), len(v), dimensions, int(normalise),
                                   _ptr(out, ctypes.c_float)))
        return out
