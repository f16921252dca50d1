"""A float emulation of the CUDA forward's 16-bit rounding points (test helper, CPU only).

The CUDA path multiplies fp16 operands on the tensor cores and accumulates in fp32; the oracle
(the restated CPUReference.forward) is fp32 throughout.  This numpy restatement of the
gemma-embedding forward (Model/CPUReference.swift:183-283 for the layer loop, with the dense
head after the mean) can round to fp16 at each point where the CUDA path stores or multiplies a
16-bit value, so the tests can say which rounding the difference between the two comes from:

  "W"      the Q8_0 weights, q x scale rounded once to fp16 (the tensor-core B operand)
  "A"      GEMM inputs h and the attention output (the tensor-core A operand)
  "act"    the GeGLU output (the down projection's A operand)
  "qkvout" the q/k/v projection outputs, stored fp16
  "qkv"    q, k, v after their norms and RoPE, stored fp16 for the attention kernel
  "P"      the softmax numerators, fp16 operands of P.V
  "tout"   the o and down projection outputs, stored fp16 for the residual step

Everything else is fp32 with float64 dot products.  Weights come from the oracle's own Q8_0
dequantisation (Model/Weights.swift:19-43), and the RoPE table from its double-precision
restatement of RopeTable.swift:16-31.
"""
import numpy as np

ALL = frozenset({"W", "A", "act", "qkvout", "qkv", "P", "tout"})


def _f16(a):
    return a.astype(np.float16).astype(np.float32)


def _rms(x, w, eps):
    r = (1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + eps)).astype(np.float32)
    y = x * r
    return y * w if w is not None else y


def _gelu(x):
    return 0.5 * x * (1 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


class Emulator:
    """gemma-embedding forward over one sequence of at most 512 tokens (inside the sliding
    window, so every layer attends to the whole sequence)."""

    def __init__(self, binding, path):
        self.B = binding
        self.model = binding.OracleModel(path)
        info = self.model.info
        self.d, self.layers, self.eps = info.hidden, info.layers, 1e-6
        self.w = {}
        self.rope = {base: binding.rope_table(256, base, 512) for base in (1e4, 1e6)}

    def close(self):
        self.model.close()

    def _t(self, name):
        if name not in self.w:
            self.w[name] = self.B.tensor(self.model._h, name)
        return self.w[name]

    def _rope(self, x, base):
        tab = self.rope[base][: x.shape[0]]
        c, s = tab[:, None, :, 0], tab[:, None, :, 1]
        a, b = x[..., :128], x[..., 128:]
        return np.concatenate([a * c - b * s, a * s + b * c], -1)

    def forward(self, ids, rounding=ALL):
        R = set(rounding)
        n, d = len(ids), self.d
        emb = np.stack([self.model.dequantize_row("token_embd.weight", int(t), d) for t in ids])
        x = emb * np.float32(np.sqrt(float(d)))

        def mm(a, name, operand="A"):
            w = self._t(name)
            if "W" in R:
                w = _f16(w)
            if operand in R:
                a = _f16(a)
            return (a.astype(np.float64) @ w.T.astype(np.float64)).astype(np.float32)

        for l in range(self.layers):
            base = 1e6 if l % 6 == 5 else 1e4
            blk = f"blk.{l}."
            h = _rms(x, self._t(blk + "attn_norm.weight")[0], self.eps)
            q, k, v = (mm(h, blk + f"attn_{p}.weight") for p in "qkv")
            if "qkvout" in R:
                q, k, v = _f16(q), _f16(k), _f16(v)
            q = _rms(q.reshape(n, -1, 256), self._t(blk + "attn_q_norm.weight")[0], self.eps)
            k = _rms(k.reshape(n, -1, 256), self._t(blk + "attn_k_norm.weight")[0], self.eps)
            v = _rms(v.reshape(n, -1, 256), None, self.eps)
            q, k = self._rope(q, base), self._rope(k, base)
            if "qkv" in R:
                q, k, v = _f16(q), _f16(k), _f16(v)
            heads = q.shape[1]
            kk = np.repeat(k, heads // k.shape[1], 1)
            vv = np.repeat(v, heads // v.shape[1], 1)
            s = np.einsum("thd,shd->hts", q.astype(np.float64), kk.astype(np.float64)).astype(np.float32)
            p = np.exp(s - s.max(-1, keepdims=True))
            den = p.sum(-1, keepdims=True)
            if "P" in R:
                p = _f16(p)
            o = np.einsum("hts,shd->thd", p.astype(np.float64), vv.astype(np.float64)) / den.transpose(1, 0, 2)
            t = mm(o.astype(np.float32).reshape(n, -1), blk + "attn_output.weight")
            if "tout" in R:
                t = _f16(t)
            x = x + _rms(t, self._t(blk + "post_attention_norm.weight")[0], self.eps)
            h = _rms(x, self._t(blk + "ffn_norm.weight")[0], self.eps)
            act = _gelu(mm(h, blk + "ffn_gate.weight")) * mm(h, blk + "ffn_up.weight")
            t = mm(act, blk + "ffn_down.weight", operand="act")
            if "tout" in R:
                t = _f16(t)
            x = x + _rms(t, self._t(blk + "post_ffw_norm.weight")[0], self.eps)
        h = _rms(x, self._t("output_norm.weight")[0], self.eps)
        mid = self._t("dense_2.weight").astype(np.float64) @ h.mean(0).astype(np.float64)
        return (self._t("dense_3.weight").astype(np.float64) @ mid).astype(np.float32)
