"""Test infrastructure only: the reference's decode step evaluated in float64.

Every engine under test (the reference's scalar and SIMD kernels, the C
restatement, the CUDA engine) computes the same step in FP32 with its own
summation order. On models that amplify rounding (activation outliers) those
orders disagree by more than a fixed logit tolerance, so the tests measure each
engine's distance to this float64 evaluation of the same arithmetic instead.

The step follows src/model.cpp:258-329 operation by operation:

* embedding row: int8 value times the row's scale (model.cpp:262-266);
* RoPE angles exactly as the reference forms them, in FP32: the inverse
  frequencies of model.cpp:223-224 (taken from the C restatement) times
  float(pos) (model.cpp:269-272); only cos/sin and the rotation run in float64;
* rmsnorm: x * (1 / sqrt(sum(x^2) / n + eps)) * w (src/kernels.cpp:132-137);
* int8 matvec: (row . x) * row scale, the scale applied after the sum
  (src/kernels.cpp:27);
* biases, rotation (model.cpp:283-291), KV append, attention with max
  subtraction and 1/sqrt(dim) scaling (src/kernels.cpp:150-180), the O
  projection and residual, SiLU(gate) * up (model.cpp:302), down projection and
  residual, final rmsnorm and the tied LM head (model.cpp:307-310).

Weights are widened to float64 once (about 4 GB for the Qwen2.5-0.5B shape).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from . import _synthetic, inverse_frequency


class Exact64:
    """float64 decode over a model directory, with its own float64 KV cache."""

    def __init__(self, directory: Path | str, capacity: int):
        self.dims, t = _synthetic().load_model(directory)
        d = self.dims
        self.capacity = capacity
        self.pos = 0

        def mat(name):
            return np.asarray(t[name], np.float64), np.asarray(t[name + ".scales"], np.float64)

        def vec(name):
            return np.asarray(t[name], np.float64)
        self.embed, self.embed_scales = mat("model.embed_tokens.weight")
        self.final_norm = vec("model.norm.weight")
        self.layers = []
        for l in range(d.layers):
            b = f"model.layers.{l}."
            self.layers.append({
                "q": mat(b + "self_attn.q_proj.weight"), "k": mat(b + "self_attn.k_proj.weight"),
                "v": mat(b + "self_attn.v_proj.weight"), "o": mat(b + "self_attn.o_proj.weight"),
                "gate": mat(b + "mlp.gate_proj.weight"), "up": mat(b + "mlp.up_proj.weight"),
                "down": mat(b + "mlp.down_proj.weight"),
                "qb": vec(b + "self_attn.q_proj.bias"), "kb": vec(b + "self_attn.k_proj.bias"),
                "vb": vec(b + "self_attn.v_proj.bias"),
                "in_norm": vec(b + "input_layernorm.weight"), "post_norm": vec(b + "post_attention_layernorm.weight"),
            })
        self.keys = np.zeros((d.layers, capacity, d.kv_heads, d.head_dim))
        self.values = np.zeros_like(self.keys)
        self.inv_freq = inverse_frequency(d.head_dim, d.theta)

    def _norm(self, x, w):
        return x * (1.0 / np.sqrt(np.dot(x, x) / x.size + self.dims.epsilon)) * w

    @staticmethod
    def _mv(m, x):
        w, s = m
        return (w @ x) * s

    def _rotate(self, a, cos, sin):
        half = a.shape[-1] // 2
        first, second = a[:, :half].copy(), a[:, half:].copy()
        a[:, :half] = first * cos - second * sin
        a[:, half:] = second * cos + first * sin

    def step(self, token: int, head: bool = True) -> np.ndarray | None:
        d = self.dims
        if not 0 <= token < d.vocab:
            raise RuntimeError("token ID outside vocabulary")
        if self.pos >= self.capacity:
            raise RuntimeError("context capacity exceeded")
        pos, D = self.pos, d.head_dim
        x = self.embed[token] * self.embed_scales[token]
        angle = (np.float32(pos) * self.inv_freq).astype(np.float64)
        cos, sin = np.cos(angle), np.sin(angle)
        group = d.heads // d.kv_heads
        for li, L in enumerate(self.layers):
            h = self._norm(x, L["in_norm"])
            q = (self._mv(L["q"], h) + L["qb"]).reshape(d.heads, D)
            k = (self._mv(L["k"], h) + L["kb"]).reshape(d.kv_heads, D)
            v = (self._mv(L["v"], h) + L["vb"]).reshape(d.kv_heads, D)
            self._rotate(q, cos, sin)
            self._rotate(k, cos, sin)
            self.keys[li, pos] = k
            self.values[li, pos] = v
            keys, values = self.keys[li, :pos + 1], self.values[li, :pos + 1]
            attn = np.empty((d.heads, D))
            for hh in range(d.heads):
                g = hh // group
                s = keys[:, g] @ q[hh] * (1.0 / np.sqrt(D))
                p = np.exp(s - s.max())
                attn[hh] = (p / p.sum()) @ values[:, g]
            x = x + self._mv(L["o"], attn.reshape(-1))
            h = self._norm(x, L["post_norm"])
            gate, up = self._mv(L["gate"], h), self._mv(L["up"], h)
            x = x + self._mv(L["down"], gate / (1.0 + np.exp(-gate)) * up)
        self.pos += 1
        if not head:
            return None
        return self._mv((self.embed, self.embed_scales), self._norm(x, self.final_norm))
