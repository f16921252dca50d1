"""Seeded synthetic weights and inputs for the EmbeddingGemma text encoder.

No real checkpoint ships with this project, so every test, the smoke run and the
benchmark use random-init weights written to a GGUF v3 file with the tensor
names, shapes and storage types the reference loader checks
(`Sources/GemmaEmbed/Model/Weights.swift:103-130`, metadata keys from
`Sources/GemmaEmbed/Model/ModelConfig.swift:54-112`).

Random numbers come from the reference test suite's `SeededRandom`
(splitmix64, `Tests/GemmaEmbedTests/KernelTests.swift:9-26`), vectorised with
numpy: the i-th draw (0-based) of `SeededRandom(seed)` is
`mix(seed + (i + 2) * 0x9E3779B97F4A7C15)`, and `floats(n, scale)` maps a draw
`r` to `(float(r >> 40) / 2**24 * 2 - 1) * scale` in float32.

Quantisation to Q8_0 follows ggml's reference rule (blocks of 32 along the
contiguous dimension, `d = amax / 127`, `q = roundf(x / d)` with the scale
stored as fp16), which the reference reads back in
`Sources/GemmaEmbed/Model/Weights.swift:33-41`.

Two architectures are described (both read by the same loader):

* ``"gemma-embedding"`` -- the measured shape: hidden 768, 24 layers, 3 query
  heads and 1 KV head of 256, GeGLU 1152, global attention every 6th layer,
  then mean-pool and a dense 768->3072->768 head (`dense_2.weight`,
  `dense_3.weight`).
* ``"gemma-embedding2"`` -- the reference's own EmbeddingGemma 2 shape
  (`Sources/GemmaEmbed/Model/Architecture.md:7-33`): hidden 512, 4 query heads,
  sliding layers 2 KV x 256, global layers 1 KV x 512, GeGLU 2048, per-layer
  inputs, and a per-token 512->768 output projection before the mean.
"""
from __future__ import annotations

import hashlib
import os
import struct
from dataclasses import dataclass, field

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_C1 = np.uint64(0xBF58476D1CE4E5B9)
_C2 = np.uint64(0x94D049BB133111EB)

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
VOCAB = 262144


# --------------------------------------------------------------------------- random
def _mix(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _C1
    z = (z ^ (z >> np.uint64(27))) * _C2
    return z ^ (z >> np.uint64(31))


def draws(seed: int, n: int, start: int = 0) -> np.ndarray:
    """Draws `start .. start+n-1` of `SeededRandom(seed).next()` as uint64."""
    with np.errstate(over="ignore"):
        i = np.arange(start, start + n, dtype=np.uint64)
        state = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + (i + np.uint64(2)) * GOLDEN
        return _mix(state)


def floats(seed: int, n: int, scale: float = 1.0, start: int = 0) -> np.ndarray:
    """`SeededRandom(seed).floats(n, scale)`: uniform in [-scale, scale) as float32."""
    r = (draws(seed, n, start) >> np.uint64(40)).astype(np.float32)
    return ((r / np.float32(1 << 24)) * np.float32(2) - np.float32(1)) * np.float32(scale)


class SeededRandom:
    """Scalar `SeededRandom` (splitmix64), for short draw sequences such as token ids."""

    def __init__(self, seed: int):
        self.state = (seed + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF

    def next(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        return z ^ (z >> 31)


# --------------------------------------------------------------------------- Q8_0
def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Rows of float32 `[rows][K]` (K % 32 == 0) to Q8_0 bytes `[rows][K/32*34]`."""
    rows, k = x.shape
    assert k % 32 == 0
    b = x.reshape(rows, k // 32, 32).astype(np.float32)
    amax = np.abs(b).max(axis=2)
    d = (amax / np.float32(127)).astype(np.float32)
    inv = np.where(d != 0, np.float32(1) / np.where(d != 0, d, np.float32(1)), np.float32(0)).astype(np.float32)
    v = b * inv[:, :, None]
    q = np.trunc(v + np.copysign(np.float32(0.5), v)).astype(np.int8)  # roundf: half away from zero
    out = np.empty((rows, k // 32, 34), dtype=np.uint8)
    out[:, :, 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, k // 32, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(rows, k // 32 * 34)


def dequantize_q8_0(raw: np.ndarray, k: int) -> np.ndarray:
    """Inverse of `quantize_q8_0`, exact in float32 (fp16 scale times int8)."""
    rows = raw.shape[0]
    blocks = raw.reshape(rows, k // 32, 34)
    d = blocks[:, :, 0:2].copy().view(np.float16).astype(np.float32)
    q = blocks[:, :, 2:].copy().view(np.int8).astype(np.float32)
    return (q * d).reshape(rows, k)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).view(np.uint32)
    rounded = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (rounded >> np.uint32(16)).astype(np.uint16)


# --------------------------------------------------------------------------- architectures
@dataclass
class Arch:
    name: str
    hidden: int
    layers: int
    heads: int
    head_dim_swa: int
    head_dim_global: int
    kv_swa: int
    kv_global: int
    ff: int
    per_layer: int            # 0: no per-layer inputs
    out_dim: int
    dense_head: int           # 0: no pooled dense head
    vocab: int = VOCAB
    sliding_window: int = 1024
    rope_swa: float = 1.0e4
    rope_global: float = 1.0e6
    eps: float = 1e-6
    global_every: int = 6

    def sliding(self, i: int) -> bool:
        return (i % self.global_every) != self.global_every - 1

    def kv(self, i: int) -> int:
        return self.kv_swa if self.sliding(i) else self.kv_global

    def hd(self, i: int) -> int:
        return self.head_dim_swa if self.sliding(i) else self.head_dim_global


ARCHS = {
    "gemma-embedding": dict(hidden=768, layers=24, heads=3, head_dim_swa=256, head_dim_global=256,
                            kv_swa=1, kv_global=1, ff=1152, per_layer=0, out_dim=768, dense_head=3072),
    "gemma-embedding2": dict(hidden=512, layers=24, heads=4, head_dim_swa=256, head_dim_global=512,
                             kv_swa=2, kv_global=1, ff=2048, per_layer=512, out_dim=768, dense_head=0),
}


def make_arch(name: str, layers: int | None = None, vocab: int | None = None) -> Arch:
    kw = dict(ARCHS[name])
    if layers is not None:
        kw["layers"] = layers
    if vocab is not None:
        kw["vocab"] = vocab
    return Arch(name=name, **kw)


@dataclass
class Tensor:
    name: str
    shape: list          # GGUF ne order: contiguous dimension first
    ggml_type: int
    data: bytes = field(repr=False, default=b"")


def _tensor_seed(seed: int, name: str) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little")


def _q8_tensor(name, cols, rows, seed, scale, chunk_rows=8192):
    parts = []
    s = _tensor_seed(seed, name)
    for r0 in range(0, rows, chunk_rows):
        r = min(chunk_rows, rows - r0)
        x = floats(s, r * cols, scale, start=r0 * cols).reshape(r, cols)
        parts.append(quantize_q8_0(x).tobytes())
    return Tensor(name, [cols, rows], GGML_Q8_0, b"".join(parts))


def _f32_tensor(name, n, seed, base, spread):
    x = np.float32(base) * (np.float32(1) + floats(_tensor_seed(seed, name), n, spread))
    return Tensor(name, [n], GGML_F32, x.astype(np.float32).tobytes())


def build_tensors(arch: Arch, seed: int) -> list:
    d, ff, pl = arch.hidden, arch.ff, arch.per_layer
    t = []
    # Embedding rows scaled so that x = row * sqrt(d) has entries of order 1.
    t.append(_q8_tensor("token_embd.weight", d, arch.vocab, seed, 0.06))
    if pl:
        name = "per_layer_model_proj.weight"
        x = floats(_tensor_seed(seed, name), pl * arch.layers * d, (3.0 / d) ** 0.5)
        t.append(Tensor(name, [d, pl * arch.layers], GGML_BF16, to_bf16_bits(x).tobytes()))
        t.append(_f32_tensor("per_layer_proj_norm.weight", pl, seed, 1.0, 0.1))
    for i in range(arch.layers):
        hd, kv = arch.hd(i), arch.kv(i)
        qd, kvd = arch.heads * hd, kv * hd
        p = f"blk.{i}."
        qk_w = hd ** -0.25   # keeps scale-1.0 logits of normed q and k of order 1
        t.append(_f32_tensor(p + "attn_norm.weight", d, seed, 1.0, 0.1))
        t.append(_q8_tensor(p + "attn_q.weight", d, qd, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "attn_k.weight", d, kvd, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "attn_v.weight", d, kvd, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "attn_output.weight", qd, d, seed, (3.0 / qd) ** 0.5))
        t.append(_f32_tensor(p + "attn_q_norm.weight", hd, seed, qk_w, 0.1))
        t.append(_f32_tensor(p + "attn_k_norm.weight", hd, seed, qk_w, 0.1))
        t.append(_f32_tensor(p + "post_attention_norm.weight", d, seed, 1.0, 0.1))
        t.append(_f32_tensor(p + "ffn_norm.weight", d, seed, 1.0, 0.1))
        t.append(_q8_tensor(p + "ffn_gate.weight", d, ff, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "ffn_up.weight", d, ff, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor(p + "ffn_down.weight", ff, d, seed, (3.0 / ff) ** 0.5))
        t.append(_f32_tensor(p + "post_ffw_norm.weight", d, seed, 1.0, 0.1))
        if pl:
            t.append(_q8_tensor(p + "inp_gate.weight", d, pl, seed, (3.0 / d) ** 0.5))
            t.append(_q8_tensor(p + "proj.weight", pl, d, seed, (3.0 / pl) ** 0.5))
            t.append(_f32_tensor(p + "post_norm.weight", d, seed, 1.0, 0.1))
            t.append(_f32_tensor(p + "layer_output_scale.weight", 1, seed, 0.9, 0.05))
    t.append(_f32_tensor("output_norm.weight", d, seed, 1.0, 0.1))
    if arch.per_layer:
        t.append(_q8_tensor("output.weight", d, arch.out_dim, seed, (3.0 / d) ** 0.5))
    if arch.dense_head:
        t.append(_q8_tensor("dense_2.weight", d, arch.dense_head, seed, (3.0 / d) ** 0.5))
        t.append(_q8_tensor("dense_3.weight", arch.dense_head, arch.out_dim, seed, (3.0 / arch.dense_head) ** 0.5))
    return t


# --------------------------------------------------------------------------- GGUF v3 writer
def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, payload: bytes) -> bytes:
    return _str(key) + struct.pack("<I", vtype) + payload


def metadata(arch: Arch) -> list:
    a = arch.name
    n = arch.layers
    kv = [
        _kv("general.architecture", 8, _str(a)),
        _kv("general.name", 8, _str(f"synthetic-{a}")),
        _kv("general.alignment", 4, struct.pack("<I", 32)),
        _kv(f"{a}.block_count", 4, struct.pack("<I", n)),
        _kv(f"{a}.embedding_length", 4, struct.pack("<I", arch.hidden)),
        _kv(f"{a}.embedding_length_out", 4, struct.pack("<I", arch.out_dim)),
        _kv(f"{a}.embedding_length_per_layer_input", 4, struct.pack("<I", arch.per_layer)),
        _kv(f"{a}.feed_forward_length", 4, struct.pack("<I", arch.ff)),
        _kv(f"{a}.attention.head_count", 4, struct.pack("<I", arch.heads)),
        _kv(f"{a}.attention.head_count_kv", 9,
            struct.pack("<IQ", 5, n) + np.array([arch.kv(i) for i in range(n)], dtype=np.int32).tobytes()),
        _kv(f"{a}.attention.sliding_window_pattern", 9,
            struct.pack("<IQ", 7, n) + bytes(1 if arch.sliding(i) else 0 for i in range(n))),
        _kv(f"{a}.attention.key_length", 4, struct.pack("<I", arch.head_dim_global)),
        _kv(f"{a}.attention.key_length_swa", 4, struct.pack("<I", arch.head_dim_swa)),
        _kv(f"{a}.attention.value_length", 4, struct.pack("<I", arch.head_dim_global)),
        _kv(f"{a}.attention.value_length_swa", 4, struct.pack("<I", arch.head_dim_swa)),
        _kv(f"{a}.attention.sliding_window", 4, struct.pack("<I", arch.sliding_window)),
        _kv(f"{a}.attention.layer_norm_rms_epsilon", 6, struct.pack("<f", arch.eps)),
        _kv(f"{a}.rope.freq_base", 6, struct.pack("<f", arch.rope_global)),
        _kv(f"{a}.rope.freq_base_swa", 6, struct.pack("<f", arch.rope_swa)),
        _kv("tokenizer.ggml.bos_token_id", 4, struct.pack("<I", 2)),
        _kv("tokenizer.ggml.eos_token_id", 4, struct.pack("<I", 1)),
    ]
    toks = [f"<t{i}>".encode() for i in range(arch.vocab)]
    body = b"".join(struct.pack("<Q", len(s)) + s for s in toks)
    kv.append(_kv("tokenizer.ggml.tokens", 9, struct.pack("<IQ", 8, arch.vocab) + body))
    return kv


def write_gguf(path: str, arch: Arch, tensors: list, alignment: int = 32, kvs: list | None = None) -> None:
    """GGUF v3 with `arch`'s metadata (or the given key/value records) and `tensors`."""
    kvs = metadata(arch) if kvs is None else kvs
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kvs)) + b"".join(kvs)
    infos = []
    offset = 0
    offsets = []
    for t in tensors:
        offsets.append(offset)
        infos.append(_str(t.name) + struct.pack("<I", len(t.shape)) +
                     b"".join(struct.pack("<Q", s) for s in t.shape) +
                     struct.pack("<IQ", t.ggml_type, offset))
        offset += (len(t.data) + alignment - 1) // alignment * alignment
    header = head + b"".join(infos)
    pad = (-len(header)) % alignment
    tmp = path + f".tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(header + b"\0" * pad)
        for t, off in zip(tensors, offsets):
            f.write(t.data)
            f.write(b"\0" * ((-len(t.data)) % alignment))
    os.replace(tmp, path)


def cache_dir() -> str:
    d = os.environ.get("GE_SYNTH_CACHE") or os.path.join(os.environ.get("TMPDIR", "/tmp"), "gemma_embed_synth")
    os.makedirs(d, exist_ok=True)
    return d


FORMAT_VERSION = 1


def model_path(arch: str = "gemma-embedding", seed: int = 0, layers: int | None = None,
               vocab: int | None = None) -> str:
    """Path of the synthetic GGUF for (arch, seed, layers, vocab), written on first use."""
    a = make_arch(arch, layers, vocab)
    name = f"{arch}-s{seed}-l{a.layers}-v{a.vocab}-f{FORMAT_VERSION}.gguf"
    path = os.path.join(cache_dir(), name)
    if not os.path.exists(path):
        write_gguf(path, a, build_tensors(a, seed))
    return path


# --------------------------------------------------------------------------- inputs
def config_sequences(config: int, seed: int = 0, vocab: int = VOCAB, scale_texts: int = 1) -> list:
    """Token-id sequences of a benchmark configuration, drawn from `SeededRandom(seed)`.

    config 1: 8 texts x 128 tokens.  config 2: 64 texts, lengths uniform in 32..512
    (lengths drawn first, then ids).  config 3: 16 x 2048 then 4 x 8192 tokens.
    config 4 (the metric's literal wording): 64 x 512.  Ids are `next() % vocab`.
    """
    rng = SeededRandom(seed)
    if config == 1:
        lens = [128] * 8
    elif config == 2:
        lens = [32 + rng.next() % 481 for _ in range(64 * scale_texts)]
    elif config == 3:
        lens = [2048] * 16 + [8192] * 4
    elif config == 4:
        lens = [512] * 64
    else:
        raise ValueError(f"unknown config {config}")
    return [np.array([rng.next() % vocab for _ in range(n)], dtype=np.int32) for n in lens]


def random_sequences(lengths, seed: int, vocab: int = VOCAB) -> list:
    rng = SeededRandom(seed)
    return [np.array([rng.next() % vocab for _ in range(n)], dtype=np.int32) for n in lengths]
