"""Generates the committed golden fixtures under tests/golden/.

Run in a container that has gguf-py and transformers (this build's dev
container does); the fixtures are then plain .npz files the tests read
without either package.

  q4k_golden.npz     Q4_K blocks and their dequantised values from gguf-py
                     0.19.0 (`gguf.quants.dequantize(..., Q4_K)`), the
                     published restatement of candle's k_quants BlockQ4K.
  buckets_golden.npz HF transformers' T5Attention._relative_position_bucket
                     (bidirectional, 32 buckets, max distance 128) for every
                     key - query in [-2047, 2047].
  t5_tiny_golden.npz a tiny T5 v1.1-shaped encoder (seeded synthetic Q4_K
                     checkpoint from witchcraft_b200.synth) run through HF
                     transformers' T5EncoderModel in f32 with the same
                     dequantised weights plus a bias-free 256->128 Linear
                     (the XTR architecture of downloadweights.py:10-33).
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from witchcraft_b200.synth import T5Config, make_synthetic_model, quantize_q4k  # noqa: E402

TINY = dict(vocab_size=512, d_model=256, d_ff=512, num_heads=4, num_layers=2)
TINY_SEED = 7


def q4k_fixture():
    import gguf
    from gguf.quants import dequantize
    rng = np.random.default_rng(11)
    parts = []
    # blocks from this project's quantizer over varied scales
    for std in (1e-3, 0.02, 1.0, 30.0):
        parts.append(quantize_q4k(rng.standard_normal((4, 512)).astype(np.float32) * std).reshape(-1, 144))
    # random bytes with finite f16 d / dmin (normal and subnormal)
    rb = rng.integers(0, 256, (96, 144), dtype=np.uint8)
    d = rng.standard_normal(96).astype(np.float16) * np.float16(0.01)
    d[::7] = np.float16(3e-6)     # subnormal half
    d[3::11] = np.float16(-0.5)   # negative scale
    dm = np.abs(rng.standard_normal(96)).astype(np.float16) * np.float16(0.01)
    rb[:, 0:2] = d.view(np.uint8).reshape(96, 2)
    rb[:, 2:4] = dm.view(np.uint8).reshape(96, 2)
    parts.append(rb)
    # fully random bytes (may hold inf / NaN halves)
    parts.append(rng.integers(0, 256, (16, 144), dtype=np.uint8))
    blocks = np.concatenate(parts)
    deq = dequantize(blocks, gguf.GGMLQuantizationType.Q4_K).reshape(-1, 256).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q4k_golden.npz"), blocks=blocks, values=deq)


def bucket_fixture():
    import torch
    from transformers.models.t5.modeling_t5 import T5Attention
    rel = torch.arange(-2047, 2048)
    b = T5Attention._relative_position_bucket(rel, bidirectional=True, num_buckets=32, max_distance=128)
    np.savez_compressed(os.path.join(HERE, "buckets_golden.npz"), delta=rel.numpy().astype(np.int32),
                        bucket=b.numpy().astype(np.int32))


def tiny_fixture():
    import torch
    from transformers import T5Config as HFConfig, T5EncoderModel
    cfg = T5Config(**TINY)
    m = make_synthetic_model(cfg, seed=TINY_SEED)
    hf = HFConfig(vocab_size=cfg.vocab_size, d_model=cfg.d_model, d_kv=64, d_ff=cfg.d_ff,
                  num_layers=cfg.num_layers, num_heads=cfg.num_heads, relative_attention_num_buckets=32,
                  relative_attention_max_distance=128, dropout_rate=0.0, layer_norm_epsilon=1e-6,
                  feed_forward_proj="gated-gelu", is_encoder_decoder=False, use_cache=False)
    enc = T5EncoderModel(hf).eval().float()
    sd = {}
    for name, blocks in m.q4k.items():
        if name == "linear.weight":
            continue
        sd[name] = torch.from_numpy(m.dequantized(name))
    for name, arr in m.f32.items():
        sd[name] = torch.from_numpy(arr)
    sd["shared.weight"] = sd["encoder.embed_tokens.weight"]
    missing, unexpected = enc.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("embed_tokens" in k or k == "shared.weight" for k in missing), missing
    proj = torch.from_numpy(m.dequantized("linear.weight"))
    rng = np.random.default_rng(3)
    lengths = [24, 17, 5, 1]
    outs = []
    ids = rng.integers(3, cfg.vocab_size, (len(lengths), 24)).astype(np.uint32)
    with torch.no_grad():
        for b, n in enumerate(lengths):
            h = enc(input_ids=torch.from_numpy(ids[b:b + 1, :n].astype(np.int64))).last_hidden_state
            o = torch.zeros(1, 24, 128)
            o[:, :n] = h @ proj.T
            outs.append(o.numpy())
    np.savez_compressed(os.path.join(HERE, "t5_tiny_golden.npz"), ids=ids, lengths=np.array(lengths, np.int32),
                        out=np.concatenate(outs), gguf_sha256=np.frombuffer(hashlib.sha256(m.gguf).digest(), np.uint8),
                        seed=TINY_SEED)


if __name__ == "__main__":
    q4k_fixture()
    bucket_fixture()
    tiny_fixture()
    print("wrote fixtures to", HERE)
