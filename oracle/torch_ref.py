"""f32 CPU encoder in torch (MKL GEMMs).  TEST / BASELINE INFRASTRUCTURE ONLY.

The same restatement of the reference's default `t5-quantized` CPU path as
oracle.c (Q4_K weights dequantised to f32 at load, src/quantized_t5.rs:39-49;
RMSNorm :162-173; gated-GELU FF :231-252; attention without scaling plus the
relative-position bias :374-503; final RMSNorm + projection :669-700), but
with optimised CPU GEMMs, which is closer to the speed of the reference's
candle f32 matmuls than oracle.c's plain loops.  bench.py times it as the
CPU baseline and as the `--impl reference` arm; the parity tests use
oracle.c (and check this module against it on CPU).
"""
from __future__ import annotations

import os

import numpy as np
import torch

from . import oracle as O


class TorchCPUEncoder:
    def __init__(self, model, threads: int | None = None):
        torch.set_num_threads(threads or os.cpu_count() or 1)
        cfg = model.config
        self.cfg = cfg
        q = lambda n: torch.from_numpy(O.q4k_dequant_matrix(model.q4k[n]))  # noqa: E731
        f = lambda n: torch.from_numpy(np.ascontiguousarray(model.f32[n]))  # noqa: E731
        self.embed = q("encoder.embed_tokens.weight")
        self.rel_bias = f("encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight")
        self.layers = []
        for i in range(cfg.num_layers):
            p = f"encoder.block.{i}.layer"
            self.layers.append(dict(
                ln0=f(f"{p}.0.layer_norm.weight"),
                wq=q(f"{p}.0.SelfAttention.q.weight"), wk=q(f"{p}.0.SelfAttention.k.weight"),
                wv=q(f"{p}.0.SelfAttention.v.weight"), wo=q(f"{p}.0.SelfAttention.o.weight"),
                ln1=f(f"{p}.1.layer_norm.weight"),
                wi0=q(f"{p}.1.DenseReluDense.wi_0.weight"), wi1=q(f"{p}.1.DenseReluDense.wi_1.weight"),
                wff=q(f"{p}.1.DenseReluDense.wo.weight")))
        self.final_ln = f("encoder.final_layer_norm.weight")
        self.proj = q("linear.weight")
        self._lut = {}

    def _bias(self, L: int) -> torch.Tensor:
        if L not in self._lut:
            lut = torch.tensor([O.bucket(0, d) if d >= 0 else O.bucket(-d, 0) for d in range(-(L - 1), L)])
            delta = torch.arange(L)[None, :] - torch.arange(L)[:, None]
            self._lut[L] = self.rel_bias[lut[delta + L - 1]].permute(2, 0, 1).contiguous()  # H, L, L
        return self._lut[L]

    @torch.no_grad()
    def encode_one(self, ids: np.ndarray) -> np.ndarray:
        """One sequence (batch 1, as the reference's Embedder runs it) -> raw [L, 128]."""
        cfg = self.cfg
        H, eps = cfg.num_heads, cfg.layer_norm_epsilon
        L = len(ids)
        x = self.embed[torch.from_numpy(np.asarray(ids, np.int64))]

        def rms(t, w):
            return t / torch.sqrt((t * t).mean(-1, keepdim=True) + eps) * w

        bias = self._bias(L)
        for w in self.layers:
            xn = rms(x, w["ln0"])
            q = (xn @ w["wq"].T).view(L, H, 64).transpose(0, 1)
            k = (xn @ w["wk"].T).view(L, H, 64).transpose(0, 1)
            v = (xn @ w["wv"].T).view(L, H, 64).transpose(0, 1)
            a = torch.softmax(q @ k.transpose(-1, -2) + bias, -1) @ v
            x = x + a.transpose(0, 1).reshape(L, H * 64) @ w["wo"].T
            xn = rms(x, w["ln1"])
            g = xn @ w["wi0"].T
            h = 0.5 * g * (1 + torch.tanh(0.7978845608 * (g + 0.044715 * g ** 3))) * (xn @ w["wi1"].T)
            x = x + h @ w["wff"].T
        return (rms(x, self.final_ln) @ self.proj.T).numpy()
