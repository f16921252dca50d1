"""ctypes binding of libgemma_embed_cuda.so (the C ABI in include/gemma_embed.h).

The library is required: importing the package without it raises, and there is no
CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgemma_embed_cuda.so")

P = ctypes.POINTER
i32p, i64p, f32p, u16p, i8p = P(ctypes.c_int32), P(ctypes.c_int64), P(ctypes.c_float), P(ctypes.c_uint16), P(ctypes.c_int8)


class GeSeq(ctypes.Structure):
    _fields_ = [("start", ctypes.c_uint32), ("length", ctypes.c_uint32)]


class GeLoadOpts(ctypes.Structure):
    _fields_ = [("device_mask", ctypes.c_uint32), ("batch_token_budget", ctypes.c_int32), ("flags", ctypes.c_uint32),
                ("image_encoder_path", ctypes.c_char_p), ("image_patch_budget", ctypes.c_int32),
                ("audio_encoder_path", ctypes.c_char_p), ("audio_frame_budget", ctypes.c_int32)]


class GeAudio(ctypes.Structure):
    _fields_ = [("samples", ctypes.POINTER(ctypes.c_float)), ("count", ctypes.c_int64), ("sample_rate", ctypes.c_int32),
                ("channels", ctypes.c_int32), ("wav", ctypes.POINTER(ctypes.c_uint8)), ("wav_bytes", ctypes.c_int64)]


class GeAudioOpts(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("dimensions", "normalise", "max_tokens", "batch_size")]


class GeImage(ctypes.Structure):
    _fields_ = [("rgb", ctypes.POINTER(ctypes.c_uint8)), ("width", ctypes.c_int32), ("height", ctypes.c_int32)]


class GePart(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("text", ctypes.c_char_p), ("text_len", ctypes.c_int64), ("image", GeImage),
                ("audio", GeAudio)]


class GeMultimodalInput(ctypes.Structure):
    _fields_ = [("parts", ctypes.POINTER(GePart)), ("count", ctypes.c_int32)]


class GeMultimodalOpts(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("max_tokens", "dimensions", "normalise", "max_image_tokens", "batch_size")]


class GeImageOpts(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("dimensions", "normalise", "max_image_tokens", "batch_size")]


class GeEmbedOpts(ctypes.Structure):
    _fields_ = [("max_tokens", ctypes.c_int32), ("dimensions", ctypes.c_int32), ("normalise", ctypes.c_int32),
                ("batch_size", ctypes.c_int32)]


class GeInfo(ctypes.Structure):
    _fields_ = [("architecture", ctypes.c_char * 64), ("name", ctypes.c_char * 128)] + [
        (n, ctypes.c_int32) for n in ("layer_count", "hidden_size", "output_dimensions", "feed_forward_size",
                                      "per_layer_input_size", "head_count", "vocabulary_size", "sliding_window",
                                      "max_tokens")] + [
        ("norm_epsilon", ctypes.c_float), ("quantization", ctypes.c_char * 16), ("file_size", ctypes.c_int64),
        ("device_count", ctypes.c_int32), ("eos_id", ctypes.c_int32), ("bos_id", ctypes.c_int32),
        ("device_name", ctypes.c_char * 128), ("kernel_launches", ctypes.c_int64),
        ("host_to_device_bytes", ctypes.c_int64), ("device_to_host_bytes", ctypes.c_int64)] + [
        (n, ctypes.c_int32) for n in ("image_layer_count", "image_hidden_size", "image_patch_size",
                                      "image_projection_dim", "audio_layer_count", "audio_hidden_size",
                                      "audio_head_count", "audio_feed_forward_size", "audio_mel_bins",
                                      "audio_projection_dim")] + [("graph_captures", ctypes.c_int64)]


class GeKernelTime(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("ms_per_launch", ctypes.c_double), ("flops_per_launch", ctypes.c_double),
                ("bytes_per_launch", ctypes.c_double), ("launches_per_forward", ctypes.c_int32)]


class GeTokenizerInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("bos_id", "eos_id", "pad_id", "unknown_id", "vocabulary_size",
                                             "add_bos", "add_eos")]


PROGRESS_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p)

# Every entry point of include/gemma_embed.h with its argument and result types.
SIGNATURES = {
    "ge_load_opts_default": ([P(GeLoadOpts)], None),
    "ge_embed_opts_default": ([P(GeEmbedOpts)], None),
    "ge_load": ([ctypes.c_char_p, P(GeLoadOpts), P(ctypes.c_void_p)], ctypes.c_int),
    "ge_free": ([ctypes.c_void_p], None),
    "ge_last_error": ([ctypes.c_void_p], ctypes.c_char_p),
    "ge_info_get": ([ctypes.c_void_p, P(GeInfo)], ctypes.c_int),
    "ge_forward_packed": ([ctypes.c_void_p, i32p, i32p, ctypes.c_int32, P(GeSeq), ctypes.c_int32, f32p], ctypes.c_int),
    "ge_forward_device": ([ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32, P(GeSeq), ctypes.c_int32,
                           ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "ge_forward_trace": ([ctypes.c_void_p, i32p, ctypes.c_int32, ctypes.c_int32, f32p], ctypes.c_int),
    "ge_embed_tokens": ([ctypes.c_void_p, P(i32p), i32p, ctypes.c_int32, P(GeEmbedOpts), f32p, i32p, i32p,
                         PROGRESS_FN, ctypes.c_void_p], ctypes.c_int),
    "ge_profile": ([ctypes.c_void_p, i32p, ctypes.c_int32, P(GeSeq), ctypes.c_int32, ctypes.c_int32, P(GeKernelTime),
                    ctypes.c_int32, i32p], ctypes.c_int),
    "ge_pool_head_noalloc": ([ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                              ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "ge_batches": ([i64p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, i64p, i32p, i32p], ctypes.c_int),
    "ge_finish": ([f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, f32p], ctypes.c_int),
    "ge_tokenizer_load": ([ctypes.c_char_p, P(ctypes.c_void_p)], ctypes.c_int),
    "ge_tokenizer_free": ([ctypes.c_void_p], None),
    "ge_model_tokenizer": ([ctypes.c_void_p], ctypes.c_void_p),
    "ge_tokenizer_get_info": ([ctypes.c_void_p, P(GeTokenizerInfo)], ctypes.c_int),
    "ge_tokenize": ([ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int64, ctypes.c_uint32, i32p, ctypes.c_int64, i64p],
                    ctypes.c_int),
    "ge_detokenize": ([ctypes.c_void_p, i32p, ctypes.c_int64, P(ctypes.c_char), ctypes.c_int64, i64p], ctypes.c_int),
    "ge_token_piece": ([ctypes.c_void_p, ctypes.c_int32, P(ctypes.c_char), ctypes.c_int64, i64p], ctypes.c_int),
    "ge_token_is_control": ([ctypes.c_void_p, ctypes.c_int32], ctypes.c_int),
    "ge_task_prefix": ([ctypes.c_int32, ctypes.c_char_p, P(ctypes.c_char), ctypes.c_int64, i64p], ctypes.c_int),
    "ge_image_opts_default": ([P(GeImageOpts)], None),
    "ge_multimodal_opts_default": ([P(GeMultimodalOpts)], None),
    "ge_embed_multimodal": ([ctypes.c_void_p, P(GeMultimodalInput), ctypes.c_int32, ctypes.c_char_p, P(GeMultimodalOpts),
                             f32p, i32p, i32p, PROGRESS_FN, ctypes.c_void_p], ctypes.c_int),
    "ge_embed_images": ([ctypes.c_void_p, P(GeImage), ctypes.c_int32, P(GeImageOpts), f32p, i32p, PROGRESS_FN,
                         ctypes.c_void_p], ctypes.c_int),
    "ge_image_forward_device": ([ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, P(GeImage), ctypes.c_int32,
                                 ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "ge_profile_images": ([ctypes.c_void_p, P(GeImage), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                           P(GeKernelTime), ctypes.c_int32, i32p], ctypes.c_int),
    "ge_image_tokens": ([ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32], ctypes.c_int32),
    "ge_image_vectors": ([ctypes.c_void_p, P(GeImage), ctypes.c_int32, ctypes.c_int32, f32p, ctypes.c_int64, i32p],
                         ctypes.c_int),
    "ge_audio_opts_default": ([P(GeAudioOpts)], None),
    "ge_audio_tokens": ([ctypes.c_int64], ctypes.c_int64),
    "ge_audio_convert": ([P(GeAudio), f32p, ctypes.c_int64, i64p], ctypes.c_int),
    "ge_audio_decode_wav": ([ctypes.POINTER(ctypes.c_uint8), ctypes.c_int64, f32p, ctypes.c_int64, i64p,
                             ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)], ctypes.c_int),
    "ge_embed_audios": ([ctypes.c_void_p, P(GeAudio), ctypes.c_int32, P(GeAudioOpts), f32p, i32p, PROGRESS_FN,
                         ctypes.c_void_p], ctypes.c_int),
    "ge_audio_vectors": ([ctypes.c_void_p, P(GeAudio), ctypes.c_int32, f32p, ctypes.c_int64, i32p], ctypes.c_int),
    "ge_audio_forward_device": ([ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, P(GeAudio), ctypes.c_int32,
                                 ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "ge_profile_audios": ([ctypes.c_void_p, P(GeAudio), ctypes.c_int32, ctypes.c_int32, P(GeKernelTime),
                           ctypes.c_int32, i32p], ctypes.c_int),
    "ge_embed_texts": ([ctypes.c_void_p, P(ctypes.c_char_p), i64p, ctypes.c_int32, ctypes.c_char_p, P(GeEmbedOpts),
                        f32p, i32p, i32p, PROGRESS_FN, ctypes.c_void_p], ctypes.c_int),
}

# Kernel-level entry points of include/gemma_embed_testing.h.
TEST_SIGNATURES = {
    "ge_test_gemm_time": ([ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                           ctypes.c_int32, P(ctypes.c_double)], ctypes.c_int),
    "ge_test_gemm": ([u16p, ctypes.c_int32, ctypes.c_int32, P(ctypes.c_uint8), ctypes.c_int32, ctypes.c_int32,
                      ctypes.c_int32, f32p, f32p], ctypes.c_int),
    "ge_test_gemm_residual": ([u16p, ctypes.c_int32, ctypes.c_int32, P(ctypes.c_uint8), ctypes.c_int32, ctypes.c_int32,
                               f32p, f32p, ctypes.c_float, f32p, ctypes.c_float, f32p, f32p], ctypes.c_int),
    "ge_test_attention": ([u16p, u16p, u16p, ctypes.c_int32, P(GeSeq), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                           ctypes.c_int32, ctypes.c_int32, u16p], ctypes.c_int),
    "ge_test_shard": ([P(GeSeq), ctypes.c_int32, ctypes.c_int32, P(ctypes.c_int32)], ctypes.c_int),
    "ge_test_attention_schedule": ([P(GeSeq), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                    ctypes.c_int32, P(ctypes.c_uint32), ctypes.c_int32, P(ctypes.c_int32),
                                    P(ctypes.c_int32)], ctypes.c_int),
    "ge_test_image_prepare": ([ctypes.c_int32] * 3 + [P(ctypes.c_uint8), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                               P(ctypes.c_uint8), ctypes.c_int64, i32p, i32p], ctypes.c_int),
    "ge_test_patchify": ([P(ctypes.c_uint8), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, f32p, f32p, u16p,
                          ctypes.c_int32], ctypes.c_int),
    "ge_test_multimodal_sequence": ([ctypes.c_char_p, i32p, P(ctypes.c_char_p), ctypes.c_int32, i32p] +
                                    [ctypes.c_int32] * 7 + [i32p, ctypes.c_int32, i32p, i32p], ctypes.c_int),
    "ge_test_log_mel": ([f32p, ctypes.c_int64, ctypes.c_int32, f32p, i32p], ctypes.c_int),
    "ge_test_last_error": ([], ctypes.c_char_p),
}

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python gemma-embed-swift_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in {**SIGNATURES, **TEST_SIGNATURES}.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib
