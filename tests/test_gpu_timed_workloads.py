"""Oracle parity on the workloads that bench.py times, at their full size.

The measured 24-layer gemma-embedding model (seed-0 weights), with the batch shapes bench.py
runs: the config-2 batch (64 texts of 32..512 tokens, 19,516 tokens) embedded in ONE packed call
on the fp16-weight GEMM path with the captured CUDA graph replayed, and the config-3 batch
(16 x 2048 + 4 x 8192 = 65,536 tokens) in one call.  Every vector is held to the reference's
long-input bar (MetalForwardTests.swift:198-216) on L2-normalised vectors: cosine > 0.99999 and
max abs diff against the CPU oracle (the restated CPUReference.forward); hidden states after
every layer of a 2048-token sequence within 1e-2 relative (the north star's per-layer bound).
Measured values are printed (pytest -rA shows them).

The reference's max-abs bar is 1e-4 for its fp32 Metal forward against its fp32 CPU forward.
Here the tensor cores multiply fp16 operands, and the Q8_0 weights rounded to fp16 (q x scale
needs 18 significant bits) alone move the normalised vectors by about 1e-4:
test_precision_budget.py shows on the CPU that every other 16-bit rounding together stays under
1e-4 and that the weight rounding accounts for the rest.  Measured on a B200: config 2 up to
1.28e-4, config 3 up to 1.13e-4, cosine 0.9999997.  The bar here is therefore 2e-4.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

COSINE_MIN = 0.99999   # MetalForwardTests.swift:213 (and the north star)
MAX_ABS_DIFF = 2e-4    # MetalForwardTests.swift:214 has 1e-4 for fp32 x fp32; fp16 weights add ~1e-4
LAYER_REL_TOL = 1e-2   # per-layer hidden state, max |got - want| / max |want|
BUDGET = 65536         # one packed batch per call, as bench.py loads the model


def normalised(v):
    v = np.asarray(v, np.float64)
    return v / np.linalg.norm(v)


def compare(got, want):
    g, w = normalised(got), normalised(want)
    return float(g @ w), float(np.abs(g - w).max())


@pytest.fixture(scope="module")
def measured(ge, synth, oracle, cuda_device):
    path = synth.model_path("gemma-embedding", seed=0)
    model = ge.EmbeddingModel.load(path, ge.LoadOptions(batch_token_budget=BUDGET))
    ref = oracle.OracleModel(path)
    yield model, ref
    model.close()
    ref.close()


def test_config2_batch_in_one_pack_matches_oracle(measured, ge, synth):
    import torch

    model, ref = measured
    seqs = synth.config_sequences(2, seed=0)
    toks, pos, ranges = ge.pack(seqs)
    assert len(toks) == 19516 and len(ranges) == 64
    first = model.forward_packed(toks, pos, ranges)    # a new batch shape: direct launches
    second = model.forward_packed(toks, pos, ranges)   # seen before: captured as a CUDA graph
    got = model.forward_packed(toks, pos, ranges)      # replayed
    assert first.tobytes() == second.tobytes() == got.tobytes()
    # the device-resident entry bench.py times as `value`
    d_tokens = torch.from_numpy(toks).cuda()
    d_out = torch.full((len(ranges), model.info.output_dimensions), float("nan"), device="cuda")
    model.forward_device(d_tokens, ranges, d_out)
    torch.cuda.synchronize()
    assert d_out.cpu().numpy().tobytes() == got.tobytes()
    worst_cos, worst_diff = 1.0, 0.0
    for i, (s, g) in enumerate(zip(seqs, got)):
        c, d = compare(g, ref.forward(s))
        worst_cos, worst_diff = min(worst_cos, c), max(worst_diff, d)
        assert c > COSINE_MIN, (i, len(s), c)
        assert d < MAX_ABS_DIFF, (i, len(s), d)
    print(f"config 2, 64 texts, 19516 tokens in one pack: min cosine {worst_cos:.9f}, max abs diff {worst_diff:.3g}")


def test_config3_long_sequences_match_oracle(measured, ge, synth):
    """The 65,536-token config-3 batch in one call; its first 2048-token and first 8192-token
    sequences (global layers attend over all 8192 positions) against the oracle."""
    model, ref = measured
    seqs = synth.config_sequences(3, seed=0)
    toks, pos, ranges = ge.pack(seqs)
    assert len(toks) == 65536
    got = model.forward_packed(toks, pos, ranges)
    assert np.isfinite(got).all()
    for i in (0, 16):
        c, d = compare(got[i], ref.forward(seqs[i]))
        print(f"config 3, sequence {i} ({len(seqs[i])} tokens) in the 65536-token pack: cosine {c:.9f}, max abs diff {d:.3g}")
        assert c > COSINE_MIN, (i, c)
        assert d < MAX_ABS_DIFF, (i, d)


def test_per_layer_hidden_states_at_2048_tokens(measured, synth):
    model, ref = measured
    toks = synth.config_sequences(3, seed=0)[1]
    names = {f"l_out-{l}" for l in range(model.info.layer_count)} | {"result_norm"}
    trace = {}
    ref.forward(toks, trace=trace, trace_names=names)
    worst = 0.0
    for layer in range(model.info.layer_count):
        got = model.trace(toks, layer)
        want = trace[f"l_out-{layer}"].reshape(len(toks), -1)
        rel = float(np.abs(got - want).max() / np.abs(want).max())
        worst = max(worst, rel)
        assert rel <= LAYER_REL_TOL, (layer, rel)
    got = model.trace(toks, -1)
    want = trace["result_norm"].reshape(len(toks), -1)
    rel = float(np.abs(got - want).max() / np.abs(want).max())
    print(f"2048 tokens, 24 layers: worst per-layer relative error {worst:.3g}, result_norm {rel:.3g}")
    assert rel <= LAYER_REL_TOL
