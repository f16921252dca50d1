"""Kernel parity on the GPU through the C ABI (include/gemma_embed_testing.h), mirroring the
reference's KernelTests (Tests/GemmaEmbedTests/KernelTests.swift): every model GEMM shape, the
fused epilogues, Q8-in-shared-memory vs fp16-resident weights bit for bit, and attention over
packed sequences with no cross-sequence leakage."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# Kernel tolerance: max |got - want| / max |want| (TestSupport.maxRelDiff). The reference
# asserts 1e-4 for fp32 GEMM outputs (KernelTests.swift:105-110); fp32 outputs here meet the
# same bound; fp16 outputs add one fp16 rounding (2^-11 relative).
TOL_F32 = 1e-4
TOL_F16 = 2e-3


def max_rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert not np.isnan(got).any()
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def gemm(ge, a16, wq, n, epi, use_q8, aux=None):
    """use_q8: False/0 fp16 weights on single CTAs, True/1 Q8 dequantised in shared memory,
    2 fp16 weights on CTA pairs."""
    from importlib import import_module
    L = import_module("gemma-embed-swift_b200._lib").lib()
    m, k = a16.shape
    cols = n // 2 if epi == 2 else n
    out = np.zeros((m, cols), np.float32)
    a = np.ascontiguousarray(a16.view(np.uint16))
    w = np.ascontiguousarray(wq)
    auxp = None
    if aux is not None:
        aux = np.ascontiguousarray(aux, np.float32)
        auxp = aux.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    rc = L.ge_test_gemm(a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), m, k,
                        w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), n, epi, int(use_q8), auxp,
                        out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == 0, L.ge_test_last_error()
    return out


def make_case(synth, m, k, n, seed):
    rng = np.random.default_rng(seed)
    a = rng.uniform(-1, 1, size=(m, k)).astype(np.float16)
    w = synth.floats(seed, n * k, (3.0 / k) ** 0.5).reshape(n, k)
    wq = synth.quantize_q8_0(w)
    wd = synth.dequantize_q8_0(wq, k).astype(np.float16).astype(np.float64)  # the fp16 operand
    return a, wq, wd


SHAPES = [(768, 1280), (768, 768), (768, 2304), (1152, 768),      # gemma-embedding: qkv, o, gate|up, down
          (512, 2048), (512, 3072), (1024, 512), (512, 4096), (2048, 512), (512, 512)]  # gemma-embedding2


@pytest.mark.parametrize("k,n", SHAPES)
@pytest.mark.parametrize("m", [128, 200, 1000])
def test_gemm_shapes_fp32(ge, synth, cuda_device, m, k, n):
    a, wq, wd = make_case(synth, m, k, n, seed=k + n + m)
    want = a.astype(np.float64) @ wd.T
    got16 = gemm(ge, a, wq, n, 0, use_q8=False)
    got8 = gemm(ge, a, wq, n, 0, use_q8=True)
    gotp = gemm(ge, a, wq, n, 0, use_q8=2)
    gotn = gemm(ge, a, wq, n, 0, use_q8=3)
    assert max_rel(got16, want) < TOL_F32
    # The Q8 path dequantises in shared memory to the very same fp16 operand: identical bits.
    assert got8.tobytes() == got16.tobytes()
    # CTA pairs multiply the same operands with 256-row instructions: identical bits.
    assert gotp.tobytes() == got16.tobytes()
    # 128-wide tiles: the same per-element accumulation order, identical bits.
    assert gotn.tobytes() == got16.tobytes()


@pytest.mark.parametrize("use_q8", [False, True, 2])
def test_gemm_epilogues(ge, synth, oracle, cuda_device, use_q8):
    m, k, ff = 300, 768, 1152
    a, wq_gate, wd_gate = make_case(synth, m, k, ff, seed=11)
    _, wq_up, wd_up = make_case(synth, m, k, ff, seed=12)
    a64 = a.astype(np.float64)
    # fp16 store
    n = 1280
    _, wq, wd = make_case(synth, m, k, n, seed=13)
    got = gemm(ge, a, wq, n, 1, use_q8)
    assert max_rel(got, a64 @ wd.T) < TOL_F16
    if use_q8 is False:
        assert gemm(ge, a, wq, n, 1, 3).tobytes() == got.tobytes()
    # GeGLU over rows interleaved in blocks of 128 (gate block j, up block j, ...)
    rows = []
    for j in range(ff // 128):
        rows.append(wq_gate[j * 128:(j + 1) * 128])
        rows.append(wq_up[j * 128:(j + 1) * 128])
    wq_gu = np.concatenate(rows)
    gate = a64 @ wd_gate.T
    up = a64 @ wd_up.T
    gelu = np.vectorize(oracle.gelu_tanh)
    want = gelu(gate.astype(np.float32)).astype(np.float64) * up
    got = gemm(ge, a, wq_gu, 2 * ff, 2, use_q8)
    assert got.shape == (m, ff)
    assert max_rel(got, want) < TOL_F16
    # gelu(acc) * aux
    aux = np.random.default_rng(5).normal(size=(m, ff)).astype(np.float32)
    got = gemm(ge, a, wq_gate[:1024], 1024, 3, use_q8, aux=aux[:, :1024])
    want = gelu(gate[:, :1024].astype(np.float32)).astype(np.float64) * aux[:, :1024]
    assert max_rel(got, want) < TOL_F16


# (k, n, m) on 148 SMs: 150 tiles of 128 x 256 (two past the full round) and 153 GeGLU tiles
# (five past it) run their last round as half-width pieces; 3, 18 and 40 tiles (one round with
# SMs to spare) run every tile as 2, 4 or 8 pieces.
SPLIT_CASES = [(768, 768, 128 * 50), (1152, 768, 128 * 50), (768, 1280, 128 * 30), (768, 2304, 128 * 17),
               (768, 768, 128), (768, 2304, 256), (1152, 768, 1024), (768, 1280, 1024)]


@pytest.mark.parametrize("k,n,m", SPLIT_CASES)
def test_gemm_split_tiles_match_whole_tiles(ge, synth, cuda_device, k, n, m):
    """Path 4 runs tiles as narrower pieces where that would shorten the persistent schedule (a
    GeGLU piece: part of the gate rows and the up rows they pair with); path 0 keeps every tile
    whole.  The pieces multiply the same rows over the same K steps, so every epilogue gives
    identical bits, and the results match float64."""
    a, wq, wd = make_case(synth, m, k, n, seed=k * 7 + n + m)
    a64 = a.astype(np.float64)
    for epi in (0, 1):
        split = gemm(ge, a, wq, n, epi, use_q8=4)
        whole = gemm(ge, a, wq, n, epi, use_q8=0)
        assert split.tobytes() == whole.tobytes(), epi
    assert max_rel(split, a64 @ wd.T) < TOL_F16
    assert max_rel(gemm(ge, a, wq, n, 0, use_q8=4), a64 @ wd.T) < TOL_F32
    if n % 256 == 0 and n >= 1024:
        aux = np.random.default_rng(n).normal(size=(m, n)).astype(np.float32)
        assert gemm(ge, a, wq, n, 3, 4, aux=aux).tobytes() == gemm(ge, a, wq, n, 3, 0, aux=aux).tobytes()
    if n == 2304:  # gate/up interleaved in blocks of 128 rows, as the loader lays them out
        split = gemm(ge, a, wq, n, 2, use_q8=4)
        assert split.tobytes() == gemm(ge, a, wq, n, 2, use_q8=0).tobytes()
        g = np.concatenate([a64 @ wd[j * 256:j * 256 + 128].T for j in range(n // 256)], axis=1)
        u = np.concatenate([a64 @ wd[j * 256 + 128:(j + 1) * 256].T for j in range(n // 256)], axis=1)
        want = 0.5 * g * (1 + np.tanh(0.7978845608028654 * (g + 0.044715 * g ** 3))) * u  # GELU (tanh form)
        assert max_rel(split, want) < TOL_F16


def test_gemm_rows_are_independent_of_the_batch(ge, synth, cuda_device):
    """A row's result does not depend on the other rows of the batch or the tile it lands in
    (KernelTests.swift:323-339, MetalForwardTests.swift:75-97)."""
    k, n = 768, 2304
    a, wq, _ = make_case(synth, 700, k, n, seed=21)
    full = gemm(ge, a, wq, n, 0, use_q8=False)
    for lo, hi in [(0, 1), (5, 133), (128, 256), (699, 700)]:
        part = gemm(ge, np.ascontiguousarray(a[lo:hi]), wq, n, 0, use_q8=(hi - lo) < 64)
        assert part.tobytes() == full[lo:hi].tobytes()


def attention(ge, q, k, v, lens, heads, kvh, hd, hw):
    from importlib import import_module
    lib_mod = import_module("gemma-embed-swift_b200._lib")
    L = lib_mod.lib()
    ntok = sum(lens)
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
    seqs = (lib_mod.GeSeq * len(lens))(*[lib_mod.GeSeq(int(s), int(n)) for s, n in zip(starts, lens)])
    out = np.zeros((ntok, heads, hd), np.float16)
    args = [np.ascontiguousarray(x).view(np.uint16) for x in (q, k, v)]
    rc = L.ge_test_attention(*[x.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)) for x in args], ntok, seqs,
                             len(lens), heads, kvh, hd, hw, out.view(np.uint16).ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)))
    assert rc == 0, L.ge_test_last_error()
    return out.astype(np.float32)


CONFIGS = [(3, 1, 256, 512), (3, 1, 256, 0), (4, 2, 256, 512), (4, 1, 512, 0), (4, 1, 512, 512),
           (3, 1, 512, 0), (4, 2, 512, 512)]  # head dim 512: 64-row items, 63 live rows for 3 heads
# The last case packs more work items than the GPU has SMs, so the tensor-core kernel's
# persistent CTAs each take several items of different lengths.
LENGTHS = [[1, 7, 64], [1024, 5], [2048], [2048, 3, 1024, 7],
           [int(x) for x in np.random.default_rng(17).integers(1, 600, 48)]]


@pytest.mark.parametrize("heads,kvh,hd,hw", CONFIGS)
@pytest.mark.parametrize("lens", LENGTHS)
def test_attention_packed_sequences(ge, oracle, cuda_device, heads, kvh, hd, hw, lens):
    """Packed attention equals per-sequence CPU attention, with no leakage across sequence
    boundaries, for global and sliding-window layers (KernelTests.swift:552-656)."""
    rng = np.random.default_rng(hd + hw + len(lens))
    ntok = sum(lens)
    scale = 1 / np.sqrt(hd)
    q = rng.uniform(-2 * scale, 2 * scale, size=(ntok, heads, hd)).astype(np.float16)
    k = rng.uniform(-2 * scale, 2 * scale, size=(ntok, kvh, hd)).astype(np.float16)
    v = rng.uniform(-1, 1, size=(ntok, kvh, hd)).astype(np.float16)
    got = attention(ge, q, k, v, lens, heads, kvh, hd, hw)
    s = 0
    for n in lens:
        want = oracle.attention(q[s:s + n].astype(np.float32), k[s:s + n].astype(np.float32),
                                v[s:s + n].astype(np.float32), n, heads, kvh, hd, window=2 * hw).reshape(n, heads, hd)
        g = got[s:s + n]
        assert not np.isnan(g).any()
        assert max_rel(g, want) < TOL_F16, (n, heads, kvh, hd, hw)
        s += n


def gemm_residual(ge, a16, wq, n, path, x, w_post, scale, w_next, eps, want_h=True, want_y=True):
    from importlib import import_module
    L = import_module("gemma-embed-swift_b200._lib").lib()
    m, k = a16.shape
    fp = ctypes.POINTER(ctypes.c_float)
    a = np.ascontiguousarray(a16.view(np.uint16))
    w = np.ascontiguousarray(wq)
    x = np.array(x, np.float32, copy=True)
    w_post = np.ascontiguousarray(w_post, np.float32)
    wn = None if w_next is None else np.ascontiguousarray(w_next, np.float32)
    h = np.zeros((m, n), np.float32) if want_h else None
    y = np.zeros((m, n), np.float32) if want_y else None
    rc = L.ge_test_gemm_residual(a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), m, k,
                                 w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), n, path,
                                 x.ctypes.data_as(fp), w_post.ctypes.data_as(fp), scale,
                                 None if wn is None else wn.ctypes.data_as(fp), eps,
                                 None if h is None else h.ctypes.data_as(fp),
                                 None if y is None else y.ctypes.data_as(fp))
    assert rc == 0, L.ge_test_last_error()
    return x, h, y


def residual_reference(t16, x, w_post, scale, w_next, eps):
    """k_residual_norm in float64 on the fp16-rounded projection (CPUReference.swift:239-243)."""
    t = t16.astype(np.float64)
    inv = 1.0 / np.sqrt((t * t).mean(axis=1, keepdims=True) + eps)
    v = (x.astype(np.float64) + t * inv * w_post) * scale
    y = None
    if w_next is not None:
        inv2 = 1.0 / np.sqrt((v * v).mean(axis=1, keepdims=True) + eps)
        y = v * inv2 * w_next
    return v, y


@pytest.mark.parametrize("k,n,scale", [(768, 768, 1.0), (1152, 768, 1.0), (512, 512, 1.0), (2048, 512, 0.7)])
def test_gemm_residual_epilogue(ge, synth, cuda_device, k, n, scale):
    """The projection fused with the residual step and the next norm, on row clusters of n / 256
    CTAs: the residual stream to 1e-5, the next norm's fp32 output to 1e-5 and fp16 output to
    one fp16 rounding, against float64 on the fp16 projection the unfused path stores; fp16
    and Q8 weights bit for bit."""
    m = 700
    a, wq, _ = make_case(synth, m, k, n, seed=31)
    rng = np.random.default_rng(32)
    x = rng.normal(scale=3.0, size=(m, n)).astype(np.float32)
    w_post = rng.uniform(0.5, 1.5, size=n).astype(np.float32)
    w_next = rng.uniform(0.5, 1.5, size=n).astype(np.float32)
    t16 = gemm(ge, a, wq, n, 1, False)  # the fp16 projection
    want_x, want_y = residual_reference(t16, x, w_post, scale, w_next, 1e-6)
    got_x, got_h, got_y = gemm_residual(ge, a, wq, n, 0, x, w_post, scale, w_next, 1e-6)
    assert max_rel(got_x, want_x) < 1e-5
    assert max_rel(got_y, want_y) < 1e-5
    assert max_rel(got_h, want_y) < TOL_F16
    assert np.array_equal(got_h, got_y.astype(np.float16).astype(np.float32))
    qx, qh, qy = gemm_residual(ge, a, wq, n, 1, x, w_post, scale, w_next, 1e-6)
    assert qx.tobytes() == got_x.tobytes() and qh.tobytes() == got_h.tobytes() and qy.tobytes() == got_y.tobytes()
    # without the next norm only the residual stream changes
    nx, _, _ = gemm_residual(ge, a, wq, n, 0, x, w_post, scale, None, 1e-6, want_h=False, want_y=False)
    assert nx.tobytes() == got_x.tobytes()
    # rows do not depend on the batch around them
    sx, sh, _ = gemm_residual(ge, np.ascontiguousarray(a[130:131]), wq, n, 0, x[130:131], w_post, scale, w_next, 1e-6,
                              want_y=False)
    assert sx.tobytes() == got_x[130:131].tobytes() and sh.tobytes() == got_h[130:131].tobytes()
