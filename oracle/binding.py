"""ctypes binding of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline and reference arms, as the checker of the CUDA path.
The product package never imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

TRACE_FN = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int64, ctypes.c_void_p)


class OrInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("hidden", "layers", "heads", "ff", "per_layer", "out_dim", "dense_head", "vocab",
                 "sliding_window", "max_tokens")] + [
        ("eps", ctypes.c_float),
        ("kv_heads", ctypes.c_int32 * 64), ("head_dim", ctypes.c_int32 * 64), ("sliding", ctypes.c_int32 * 64),
        ("rope_base", ctypes.c_float * 64)]


class OrVisionInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("hidden", "layers", "heads", "head_dim", "ff", "patch", "projection_dim",
                                             "position_count", "merge")] + [
        ("eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("mean", ctypes.c_float * 3),
        ("std", ctypes.c_float * 3)]


class OrAudioInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("hidden", "layers", "heads", "head_dim", "ff", "mel_bins",
                                             "projection_dim", "output_width", "window", "relative_positions",
                                             "dw_kernel")] + [
        ("sub_channels", ctypes.c_int32 * 2), ("eps", ctypes.c_float), ("softcap", ctypes.c_float),
        ("ff_residual", ctypes.c_float)]


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "oracle.c")):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER
        f32p, i32p, i64p = P(ctypes.c_float), P(ctypes.c_int32), P(ctypes.c_int64)
        L.or_open.argtypes = [ctypes.c_char_p, P(ctypes.c_void_p), ctypes.c_char_p, ctypes.c_int]
        L.or_close.argtypes = [ctypes.c_void_p]
        L.or_get_info.argtypes = [ctypes.c_void_p, P(OrInfo)]
        L.or_forward.argtypes = [ctypes.c_void_p, i32p, ctypes.c_int32, f32p, TRACE_FN, ctypes.c_void_p]
        L.or_dequantize_row.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int64, f32p, ctypes.c_int64]
        L.or_matmul.argtypes = [f32p, ctypes.c_int64, ctypes.c_int64, f32p, ctypes.c_int64, f32p]
        L.or_rmsnorm.argtypes = [f32p, ctypes.c_int64, ctypes.c_int64, f32p, ctypes.c_float, f32p]
        L.or_gelu_tanh.argtypes = [ctypes.c_float]
        L.or_gelu_tanh.restype = ctypes.c_float
        L.or_rope_table.argtypes = [ctypes.c_int32, ctypes.c_float, ctypes.c_int32, f32p]
        L.or_attention.argtypes = [f32p, f32p, f32p] + [ctypes.c_int32] * 4 + [ctypes.c_float, ctypes.c_int32, f32p]
        L.or_batches.argtypes = [i64p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, i64p, i32p]
        L.or_batches.restype = ctypes.c_int32
        L.or_finish.argtypes = [f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, f32p]
        L.or_seeded_next.argtypes = [P(ctypes.c_uint64)]
        L.or_seeded_next.restype = ctypes.c_uint64
        L.or_set_threads.argtypes = [ctypes.c_int]
        L.or_threads.restype = ctypes.c_int
        u8p = P(ctypes.c_uint8)
        L.or_forward_rows.argtypes = [ctypes.c_void_p, i32p, ctypes.c_int32, f32p, ctypes.c_int64, f32p, TRACE_FN,
                                      ctypes.c_void_p]
        L.or_vision_open.argtypes = [ctypes.c_char_p, P(ctypes.c_void_p), ctypes.c_char_p, ctypes.c_int]
        L.or_vision_get_info.argtypes = [ctypes.c_void_p, P(OrVisionInfo)]
        L.or_vision_forward.argtypes = [ctypes.c_void_p, f32p, ctypes.c_int32, ctypes.c_int32, f32p, TRACE_FN,
                                        ctypes.c_void_p]
        L.or_target_size.argtypes = [ctypes.c_int32] * 5 + [i32p, i32p]
        L.or_fit_image.argtypes = [u8p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, u8p]
        L.or_patchify.argtypes = [u8p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, f32p, f32p, f32p]
        L.or_round_f16.argtypes = [ctypes.c_float]
        L.or_round_f16.restype = ctypes.c_float
        L.or_tensor_shape.argtypes = [ctypes.c_void_p, ctypes.c_char_p, i64p, i32p]
        L.or_audio_open.argtypes = [ctypes.c_char_p, P(ctypes.c_void_p), ctypes.c_char_p, ctypes.c_int]
        L.or_audio_get_info.argtypes = [ctypes.c_void_p, P(OrAudioInfo)]
        L.or_audio_forward.argtypes = [ctypes.c_void_p, f32p, ctypes.c_int32, f32p, TRACE_FN, ctypes.c_void_p]
        L.or_audio_sinusoid.argtypes = [ctypes.c_int32, ctypes.c_int32, f32p]
        L.or_audio_attention.argtypes = [f32p, f32p, f32p, f32p] + [ctypes.c_int32] * 4 + [ctypes.c_float, f32p]
        L.or_audio_depthwise.argtypes = [f32p, ctypes.c_int32, ctypes.c_int32, f32p, ctypes.c_int32, f32p]
        L.or_audio_frame_count.argtypes = [ctypes.c_int64]
        L.or_audio_frame_count.restype = ctypes.c_int32
        L.or_audio_tokens_for_frames.argtypes = [ctypes.c_int32]
        L.or_audio_tokens_for_frames.restype = ctypes.c_int32
        L.or_audio_token_count.argtypes = [ctypes.c_int64]
        L.or_audio_token_count.restype = ctypes.c_int64
        L.or_audio_tables.argtypes = [ctypes.c_int32, f32p, f32p, f32p, f32p, i32p, i32p, i32p]
        L.or_audio_log_mel.argtypes = [f32p, ctypes.c_int64, ctypes.c_int32, f32p]
        L.or_audio_log_mel.restype = ctypes.c_int32
        L.or_audio_frames_after_resampling.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64]
        L.or_audio_frames_after_resampling.restype = ctypes.c_uint64
        L.or_audio_to_mono16k.argtypes = [f32p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, f32p]
        L.or_audio_to_mono16k.restype = ctypes.c_int64
        _lib = L
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class OracleError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


class OracleModel:
    """CPUReference over a GGUF file: one sequence per `forward` call."""

    def __init__(self, path: str):
        L = lib()
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = L.or_open(path.encode(), ctypes.byref(h), err, 512)
        if rc:
            raise OracleError(rc, err.value.decode())
        self._h = h
        info = OrInfo()
        L.or_get_info(h, ctypes.byref(info))
        self.info = info

    def close(self):
        if self._h:
            lib().or_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def out_dim(self) -> int:
        return self.info.out_dim

    def forward(self, tokens, trace: dict | None = None, trace_names=None) -> np.ndarray:
        """Pooled, unnormalised vector of one sequence; fills `trace[name]` when given."""
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(self.info.out_dim, dtype=np.float32)
        cb = TRACE_FN(0)
        if trace is not None:
            def _cb(name, data, n, user):
                key = name.decode()
                if trace_names is None or key in trace_names:
                    trace[key] = np.ctypeslib.as_array(data, shape=(n,)).copy()
            cb = TRACE_FN(_cb)
        rc = lib().or_forward(self._h, toks.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(toks),
                              out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), cb, None)
        if rc:
            raise OracleError(rc, "forward rejected its input")
        return out

    def forward_rows(self, ids, vectors, trace: dict | None = None) -> np.ndarray:
        """Pooled vector of one sequence whose ids -(r + 1) are rows r of `vectors` (unscaled)."""
        toks = np.ascontiguousarray(ids, dtype=np.int32)
        vec = np.ascontiguousarray(vectors, dtype=np.float32).reshape(-1, self.info.hidden)
        out = np.zeros(self.info.out_dim, dtype=np.float32)
        cb = _trace_cb(trace)
        rc = lib().or_forward_rows(self._h, toks.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(toks),
                                   vec.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), vec.shape[0],
                                   out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), cb, None)
        if rc:
            raise OracleError(rc, "forward rejected its input")
        return out

    def dequantize_row(self, tensor: str, row: int, width: int) -> np.ndarray:
        out = np.zeros(width, dtype=np.float32)
        rc = lib().or_dequantize_row(self._h, tensor.encode(), row, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), width)
        if rc:
            raise OracleError(rc, f"cannot dequantize {tensor}[{row}]")
        return out


def _trace_cb(trace):
    if trace is None:
        return TRACE_FN(0)

    def _cb(name, data, n, user):
        trace[name.decode()] = np.ctypeslib.as_array(data, shape=(n,)).copy()
    return TRACE_FN(_cb)


class OracleVision:
    """CPUVisionReference over an mmproj file: one image per `forward` call."""

    def __init__(self, path: str):
        L = lib()
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = L.or_vision_open(path.encode(), ctypes.byref(h), err, 512)
        if rc:
            raise OracleError(rc, err.value.decode())
        self._h = h
        info = OrVisionInfo()
        L.or_vision_get_info(h, ctypes.byref(info))
        self.info = info

    def close(self):
        if self._h:
            lib().or_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, patches, grid_x: int, grid_y: int, trace: dict | None = None) -> np.ndarray:
        """The projected rows ([tokens][projection_dim]) of one prepared image."""
        pt = np.ascontiguousarray(patches, dtype=np.float32)
        m = self.info.merge
        out = np.zeros(((grid_x // m) * (grid_y // m), self.info.projection_dim), dtype=np.float32)
        cb = _trace_cb(trace)
        rc = lib().or_vision_forward(self._h, pt.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), grid_x, grid_y,
                                     out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), cb, None)
        if rc:
            raise OracleError(rc, "vision forward rejected its input")
        return out

    def prepare(self, rgb, max_image_tokens: int = 256):
        """ImagePreprocessor.prepare on a decoded image: (patches, grid_x, grid_y)."""
        i = self.info
        align = i.patch * i.merge
        h, w = rgb.shape[:2]
        tw, th = target_size(w, h, align, 70 * align * align, max_image_tokens * align * align)
        img = fit_image(rgb, tw, th)
        return patchify(img, i.patch, list(i.mean), list(i.std)), tw // i.patch, th // i.patch


class OracleAudio:
    """CPUAudioReference over an mmproj file: one 30-second chunk per `forward` call."""

    CHUNK_SAMPLES = 30 * 16000

    def __init__(self, path: str):
        L = lib()
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = L.or_audio_open(path.encode(), ctypes.byref(h), err, 512)
        if rc:
            raise OracleError(rc, err.value.decode())
        self._h = h
        info = OrAudioInfo()
        L.or_audio_get_info(h, ctypes.byref(info))
        self.info = info

    def close(self):
        if self._h:
            lib().or_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, mel, trace: dict | None = None) -> np.ndarray:
        """The projected rows ([tokens][projection_dim]) of one chunk's log-mel frames ([frames][mel_bins])."""
        m = np.ascontiguousarray(mel, dtype=np.float32)
        frames = m.shape[0]
        out = np.zeros((tokens_for_frames(frames), self.info.projection_dim), dtype=np.float32)
        cb = _trace_cb(trace)
        rc = lib().or_audio_forward(self._h, m.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), frames,
                                    out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), cb, None)
        if rc:
            raise OracleError(rc, "audio forward rejected its input")
        return out

    def prepare(self, samples) -> list:
        """AudioFrontEnd.prepare: the log-mel frames of each 30-second chunk of a 16 kHz clip."""
        return [log_mel(c, self.info.mel_bins) for c in chunks(samples)]

    def embed_rows(self, samples) -> np.ndarray:
        """All of a clip's projected rows, chunk after chunk."""
        return np.concatenate([self.forward(m) for m in self.prepare(samples)], axis=0)


def chunks(samples) -> list:
    s = np.ascontiguousarray(samples, dtype=np.float32)
    n = OracleAudio.CHUNK_SAMPLES
    return [s[i:i + n] for i in range(0, len(s), n)]


def frame_count(samples: int) -> int:
    return lib().or_audio_frame_count(samples)


def tokens_for_frames(frames: int) -> int:
    return lib().or_audio_tokens_for_frames(frames)


def audio_token_count(samples: int) -> int:
    return lib().or_audio_token_count(samples)


def audio_tables(mel_bins: int = 128) -> dict:
    f32 = ctypes.POINTER(ctypes.c_float)
    i32 = ctypes.POINTER(ctypes.c_int32)
    t = dict(hann=np.zeros(512, np.float32), sin=np.zeros(512, np.float32), cos=np.zeros(512, np.float32),
             filters=np.zeros((mel_bins, 257), np.float32), lo=np.zeros(mel_bins, np.int32),
             hi=np.zeros(mel_bins, np.int32), bitrev=np.zeros(512, np.int32))
    lib().or_audio_tables(mel_bins, t["hann"].ctypes.data_as(f32), t["sin"].ctypes.data_as(f32),
                          t["cos"].ctypes.data_as(f32), t["filters"].ctypes.data_as(f32), t["lo"].ctypes.data_as(i32),
                          t["hi"].ctypes.data_as(i32), t["bitrev"].ctypes.data_as(i32))
    return t


def log_mel(samples, mel_bins: int = 128) -> np.ndarray:
    """AudioFrontEnd.logMel of one chunk (at most 480000 samples): [frames][mel_bins]."""
    s = np.ascontiguousarray(samples, dtype=np.float32)
    frames = frame_count(len(s))
    if frames < 1:
        raise OracleError(16, f"the clip has {len(s)} samples at 16 kHz; at least 2 are needed for one frame")
    out = np.zeros((frames, mel_bins), np.float32)
    f32 = ctypes.POINTER(ctypes.c_float)
    lib().or_audio_log_mel(s.ctypes.data_as(f32), len(s), mel_bins, out.ctypes.data_as(f32))
    return out


def frames_after_resampling(rate_in: int, frames: int, rate_out: int = 16000) -> int:
    return int(lib().or_audio_frames_after_resampling(rate_out, rate_in, frames))


def to_mono16k(samples, rate: int, channels: int = 1) -> np.ndarray:
    """MiniaudioConverter.toMono16k: interleaved float samples at `rate` Hz to 16 kHz mono."""
    s = np.ascontiguousarray(samples, dtype=np.float32).reshape(-1)
    frames = s.size // channels
    n = frames_after_resampling(rate, frames) if rate != 16000 else frames
    out = np.zeros(max(n, 1), np.float32)
    f32 = ctypes.POINTER(ctypes.c_float)
    got = lib().or_audio_to_mono16k(s.ctypes.data_as(f32), frames, channels, rate, out.ctypes.data_as(f32))
    return out[:got]


def audio_sinusoid(position: int, width: int) -> np.ndarray:
    out = np.zeros(width, np.float32)
    lib().or_audio_sinusoid(position, width, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out


def target_size(width, height, alignment, min_pixels, max_pixels):
    tw, th = ctypes.c_int32(0), ctypes.c_int32(0)
    lib().or_target_size(width, height, alignment, min_pixels, max_pixels, ctypes.byref(tw), ctypes.byref(th))
    return tw.value, th.value


def fit_image(rgb, tw: int, th: int) -> np.ndarray:
    a = np.ascontiguousarray(rgb, dtype=np.uint8)
    out = np.zeros((th, tw, 3), dtype=np.uint8)
    u8 = ctypes.POINTER(ctypes.c_uint8)
    lib().or_fit_image(a.ctypes.data_as(u8), a.shape[1], a.shape[0], tw, th, out.ctypes.data_as(u8))
    return out


def patchify(rgb, patch: int, mean, std) -> np.ndarray:
    a = np.ascontiguousarray(rgb, dtype=np.uint8)
    h, w = a.shape[:2]
    out = np.zeros(((h // patch) * (w // patch), 3 * patch * patch), dtype=np.float32)
    mn = np.array(mean, np.float32)
    sd = np.array(std, np.float32)
    f32 = ctypes.POINTER(ctypes.c_float)
    lib().or_patchify(a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), w, h, patch, mn.ctypes.data_as(f32),
                      sd.ctypes.data_as(f32), out.ctypes.data_as(f32))
    return out


def tensor(handle, name: str) -> np.ndarray:
    """A whole tensor of an open oracle file, dequantised, as [rows][contiguous dimension]."""
    shape = np.zeros(4, np.int64)
    nd = ctypes.c_int32(0)
    rc = lib().or_tensor_shape(handle, name.encode(), shape.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                               ctypes.byref(nd))
    if rc:
        raise OracleError(rc, f"no tensor {name}")
    cols = int(shape[0])
    rows = int(np.prod(shape)) // cols
    out = np.zeros((rows, cols), np.float32)
    f32 = ctypes.POINTER(ctypes.c_float)
    for r in range(rows):
        lib().or_dequantize_row(handle, name.encode(), r, out[r].ctypes.data_as(f32), cols)
    return out


def round_f16(x: float) -> float:
    return lib().or_round_f16(x)


def matmul(x, w):
    x, xp = _f32(x)
    w, wp = _f32(w)
    y = np.zeros((x.shape[0], w.shape[0]), dtype=np.float32)
    lib().or_matmul(xp, x.shape[0], x.shape[1], wp, w.shape[0], y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return y


def rmsnorm(x, weight, eps=1e-6):
    x, xp = _f32(x)
    out = np.zeros_like(x)
    wp = None
    if weight is not None:
        weight, wp = _f32(weight)
    lib().or_rmsnorm(xp, x.shape[0], x.shape[1], wp, eps, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out


def gelu_tanh(x: float) -> float:
    return lib().or_gelu_tanh(x)


def rope_table(head_dim: int, base: float, positions: int) -> np.ndarray:
    out = np.zeros(positions * head_dim, dtype=np.float32)
    lib().or_rope_table(head_dim, base, positions, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out.reshape(positions, head_dim // 2, 2)


def attention(q, k, v, tokens, heads, kv_heads, hd, window=0, scale=1.0):
    q, qp = _f32(q)
    k, kp = _f32(k)
    v, vp = _f32(v)
    out = np.zeros(tokens * heads * hd, dtype=np.float32)
    lib().or_attention(qp, kp, vp, tokens, heads, kv_heads, hd, scale, window,
                       out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out


def batches(costs, batch_size, budgets):
    """EmbeddingModel.batches: a list of (start, end) ranges."""
    n = len(costs)
    ncost = len(budgets)
    c = np.ascontiguousarray(np.array(costs, dtype=np.int64).reshape(n, ncost) if n else np.zeros((0, ncost), np.int64))
    b = np.ascontiguousarray(np.array(budgets, dtype=np.int64))
    out = np.zeros(max(2 * n, 2), dtype=np.int32)
    cnt = lib().or_batches(c.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), n, ncost,
                           0 if batch_size is None else batch_size, b.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                           out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(cnt)]


def finish(v, dims, normalise):
    v, vp = _f32(v)
    out = np.zeros(min(dims, len(v)), dtype=np.float32)
    lib().or_finish(vp, len(v), dims, 1 if normalise else 0, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out


def seeded_draws(seed: int, n: int) -> list:
    state = ctypes.c_uint64((seed + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF)
    return [lib().or_seeded_next(ctypes.byref(state)) for _ in range(n)]


def set_threads(n: int) -> None:
    lib().or_set_threads(n)


def threads() -> int:
    return lib().or_threads()
