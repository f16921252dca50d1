"""The library's host-side image sizing and resampling (csrc/image.cpp) against the oracle's
restatement of ImageResizer / ImagePreprocessor, byte for byte, on CPU (no GPU needed)."""
import ctypes
from importlib import import_module

import numpy as np

from oracle import binding as B


def product_prepare(img, max_tokens, patch=16, merge=3, min_tokens=70):
    L = import_module("gemma-embed-swift_b200._lib").lib()
    h, w = img.shape[:2]
    cap = 8192 * 48 * 48 * 3
    out = np.zeros(cap, np.uint8)
    tw, th = ctypes.c_int32(0), ctypes.c_int32(0)
    u8 = ctypes.POINTER(ctypes.c_uint8)
    a = np.ascontiguousarray(img)
    rc = L.ge_test_image_prepare(patch, merge, min_tokens, a.ctypes.data_as(u8), w, h, max_tokens,
                                 out.ctypes.data_as(u8), cap, ctypes.byref(tw), ctypes.byref(th))
    assert rc == 0, L.ge_test_last_error()
    return out[:tw.value * th.value * 3].reshape(th.value, tw.value, 3)


def test_prepare_matches_oracle(ge):
    rng = np.random.default_rng(7)
    sizes = [(768, 768, 256), (1600, 1600, 256), (640, 640, 256), (800, 400, 256), (200, 150, 256), (37, 901, 256),
             (1024, 768, 1120), (96, 96, 70), (5, 3, 1)]
    for _ in range(10):
        sizes.append((int(rng.integers(4, 1200)), int(rng.integers(4, 1200)), int(rng.integers(1, 1121))))
    for w, h, mt in sizes:
        img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
        got = product_prepare(img, mt)
        tw, th = B.target_size(w, h, 48, 70 * 2304, mt * 2304)
        assert got.shape == (th, tw, 3), (w, h, mt)
        assert np.array_equal(got, B.fit_image(img, tw, th)), (w, h, mt)
