"""Where the CUDA forward's difference from the fp32 oracle comes from (CPU).

The reference holds its fp32 Metal forward to cosine > 0.99999 and max abs diff < 1e-4 against
its fp32 CPU reference (MetalForwardTests.swift:198-216).  The CUDA path multiplies fp16
operands; on the measured config-2 batch it reaches cosine 0.9999997 but max abs differences up
to 1.3e-4.  With the float emulation in fp16_rounding.py, on the config-2 batch's first text
(318 tokens, 24 layers, seed-0 weights), this test shows that the fp16 rounding of the Q8_0
weights (q x scale needs 18 significant bits; fp16 keeps 11) accounts for most of it: every
other 16-bit rounding point together stays under the reference's 1e-4, and the weight rounding
alone exceeds them all together.  That rounding is inherent to 16-bit tensor-core operands,
which the timed workloads' parity tests therefore allow for (max abs diff < 2e-4).
"""
import importlib

import numpy as np

from fp16_rounding import ALL, Emulator


def normalised(v):
    v = np.asarray(v, np.float64)
    return v / np.linalg.norm(v)


def test_fp16_weight_rounding_dominates_the_difference(oracle):
    synth = importlib.import_module("gemma-embed-swift_b200.synthetic")
    path = synth.model_path("gemma-embedding", seed=0)
    ids = synth.config_sequences(2, seed=0)[0]
    em = Emulator(oracle, path)
    try:
        want = normalised(em.model.forward(ids))

        def diff(rounding):
            got = normalised(em.forward(ids, rounding))
            return float(np.abs(got - want).max()), float(got @ want)

        exact, _ = diff(())
        assert exact < 1e-6  # the emulation without rounding is the oracle
        every, cos = diff(ALL)
        but_w, _ = diff(ALL - {"W"})
        only_w, _ = diff({"W"})
        print(f"max abs diff: every rounding {every:.3g} (cosine {cos:.9f}), all but the weights {but_w:.3g}, "
              f"weights alone {only_w:.3g}")
        assert cos > 0.99999 and every < 2e-4
        assert but_w < 1e-4
        assert only_w > but_w
    finally:
        em.close()
