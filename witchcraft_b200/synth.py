"""Seeded synthetic XTR-base checkpoints in the reference's GGUF format.

The real `assets/xtr.gguf` is produced by `tools/quantize-tool/src/main.rs:12-24`
from the HF `google/xtr-base-en` encoder plus its `2_Dense` 768->128 projection
(`downloadweights.py:10-40`): every rank-2 tensor whose inner dimension is a
multiple of 256 becomes Q4_K, everything else F32.  This module writes files
with the same tensor names, shapes and dtypes from seeded random weights, so
the encoder can be exercised without the (absent) real checkpoint.

The Q4_K quantizer here is this project's own (a per-sub-block min/max fit);
byte identity with candle's quantizer is not needed because the Q4_K bytes are
the common input of the CUDA path and the CPU oracle.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field

import numpy as np

QK_K = 256
Q4K_BLOCK_BYTES = 144

GGML_TYPE_F32 = 0
GGML_TYPE_F16 = 1
GGML_TYPE_Q4_K = 12


@dataclass
class T5Config:
    vocab_size: int = 32128
    d_model: int = 768
    d_kv: int = 64
    d_ff: int = 2048
    num_layers: int = 12
    num_heads: int = 12
    relative_attention_num_buckets: int = 32
    relative_attention_max_distance: int = 128
    layer_norm_epsilon: float = 1e-6
    feed_forward_proj: str = "gated-gelu"
    d_proj: int = 128

    def to_json(self) -> str:
        """config.json in the HF T5 schema the reference deserialises
        (`src/quantized_t5.rs:90-115`)."""
        return json.dumps({
            "vocab_size": self.vocab_size, "d_model": self.d_model, "d_kv": self.d_kv,
            "d_ff": self.d_ff, "num_layers": self.num_layers, "num_decoder_layers": self.num_layers,
            "num_heads": self.num_heads,
            "relative_attention_num_buckets": self.relative_attention_num_buckets,
            "relative_attention_max_distance": self.relative_attention_max_distance,
            "dropout_rate": 0.1, "layer_norm_epsilon": self.layer_norm_epsilon,
            "initializer_factor": 1.0, "feed_forward_proj": self.feed_forward_proj,
            "tie_word_embeddings": False, "is_decoder": False, "is_encoder_decoder": True,
            "pad_token_id": 0, "eos_token_id": 1, "decoder_start_token_id": 0,
            "model_type": "t5",
        })


# ---------------------------------------------------------------------------
# Q4_K quantizer (own algorithm) and reference-layout packing
# ---------------------------------------------------------------------------

def quantize_q4k(w: np.ndarray) -> np.ndarray:
    """Quantize a float matrix [N, K] (K % 256 == 0) to Q4_K blocks.

    Returns uint8 [N, K/256, 144] in the GGML Q4_K layout: f16 d, f16 dmin,
    12 bytes of packed 6-bit (scale, min) pairs for 8 sub-blocks of 32,
    then 128 bytes of nibbles where byte l of 32-byte chunk c holds element
    l of sub-block 2c (low nibble) and element l of sub-block 2c+1 (high).

    Fit: each sub-block gets scale = (max - min)/15 and offset = -min (min
    clamped to <= 0); the super-block stores d = max(scale)/63 and
    dmin = max(offset)/63 as f16 and 6-bit multipliers of them.
    """
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % QK_K == 0, "Q4_K needs the inner dimension to be a multiple of 256"
    nb = k // QK_K
    x = w.reshape(n, nb, 8, 32)
    mn = np.minimum(x.min(axis=-1), 0.0)          # [n, nb, 8]
    mx = x.max(axis=-1)
    scale = (mx - mn) / 15.0
    offs = -mn
    d = (scale.max(axis=-1) / 63.0).astype(np.float16)       # [n, nb]
    dmin = (offs.max(axis=-1) / 63.0).astype(np.float16)
    d32 = d.astype(np.float32)[..., None]
    dm32 = dmin.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32 > 0, np.rint(scale / d32), 0.0)
        mi = np.where(dm32 > 0, np.rint(offs / dm32), 0.0)
    sc = np.clip(sc, 0, 63).astype(np.uint8)
    mi = np.clip(mi, 0, 63).astype(np.uint8)
    d1 = (d32 * sc.astype(np.float32))[..., None]              # [n, nb, 8, 1]
    m1 = (dm32 * mi.astype(np.float32))[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(d1 > 0, np.rint((x + m1) / d1), 0.0)
    q = np.clip(q, 0, 15).astype(np.uint8)                     # [n, nb, 8, 32]

    out = np.zeros((n, nb, Q4K_BLOCK_BYTES), dtype=np.uint8)
    out[..., 0:2] = d.view(np.uint8).reshape(n, nb, 2)
    out[..., 2:4] = dmin.view(np.uint8).reshape(n, nb, 2)
    s = np.zeros((n, nb, 12), dtype=np.uint8)
    s[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    s[..., 4:8] = (mi[..., 0:4] & 63) | ((mi[..., 4:8] >> 4) << 6)
    s[..., 8:12] = (sc[..., 4:8] & 0x0F) | ((mi[..., 4:8] & 0x0F) << 4)
    out[..., 4:16] = s
    qq = q.reshape(n, nb, 4, 2, 32)
    out[..., 16:] = (qq[:, :, :, 0, :] | (qq[:, :, :, 1, :] << 4)).reshape(n, nb, 128)
    return out


def dequantize_q4k_np(blocks: np.ndarray) -> np.ndarray:
    """Vectorised numpy dequant of [..., 144] Q4_K blocks -> float32 [..., 256].

    Same arithmetic as gguf-py's Q4_K.dequantize_blocks (products rounded to
    f32, then the difference).  Host-side convenience for building oracle
    weights; the bit-exact pin is tests/test_oracle_golden.py.
    """
    b = np.asarray(blocks, dtype=np.uint8)
    lead = b.shape[:-1]
    b = b.reshape(-1, Q4K_BLOCK_BYTES)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    s = b[:, 4:16]
    sc = np.empty((b.shape[0], 8), np.uint8)
    mi = np.empty((b.shape[0], 8), np.uint8)
    sc[:, 0:4] = s[:, 0:4] & 63
    mi[:, 0:4] = s[:, 4:8] & 63
    sc[:, 4:8] = (s[:, 8:12] & 0x0F) | ((s[:, 0:4] >> 6) << 4)
    mi[:, 4:8] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    d1 = (d * sc.astype(np.float32))[:, :, None]
    m1 = (dmin * mi.astype(np.float32))[:, :, None]
    qs = b[:, 16:].reshape(-1, 4, 1, 32) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)
    q = (qs & 0x0F).reshape(-1, 8, 32).astype(np.float32)
    return (d1 * q - m1).reshape(*lead, QK_K)


# ---------------------------------------------------------------------------
# GGUF writer (v3)
# ---------------------------------------------------------------------------

def _gguf_str(s: str) -> bytes:
    e = s.encode()
    return struct.pack("<Q", len(e)) + e


def write_gguf(tensors: list[tuple[str, int, tuple[int, ...], bytes]], alignment: int = 32) -> bytes:
    """Serialise tensors to GGUF v3.  Each entry: (name, ggml_type, shape in
    row-major order [rows, cols], raw bytes).  GGUF stores dims innermost
    first, so shape is reversed on write."""
    header = bytearray()
    header += b"GGUF" + struct.pack("<I", 3)
    header += struct.pack("<QQ", len(tensors), 1)
    header += _gguf_str("general.alignment") + struct.pack("<I", 4) + struct.pack("<I", alignment)
    offset = 0
    infos = bytearray()
    offsets = []
    for name, typ, shape, data in tensors:
        infos += _gguf_str(name) + struct.pack("<I", len(shape))
        for dim in reversed(shape):
            infos += struct.pack("<Q", dim)
        infos += struct.pack("<IQ", typ, offset)
        offsets.append(offset)
        offset += len(data)
        offset = (offset + alignment - 1) // alignment * alignment
    out = bytearray(header + infos)
    pad = (-len(out)) % alignment
    out += b"\0" * pad
    base = len(out)
    for (name, typ, shape, data), off in zip(tensors, offsets):
        out += b"\0" * (base + off - len(out))
        out += data
    return bytes(out)


@dataclass
class SyntheticModel:
    """A seeded XTR-base-shaped checkpoint: GGUF bytes plus the f32 weights
    the oracle uses (dequantised from the very same Q4_K bytes)."""
    config: T5Config
    gguf: bytes
    q4k: dict = field(default_factory=dict)     # name -> uint8 [N, K/256, 144]
    f32: dict = field(default_factory=dict)     # name -> float32 (F32 tensors)

    def dequantized(self, name: str) -> np.ndarray:
        blocks = self.q4k[name]
        n = blocks.shape[0]
        return dequantize_q4k_np(blocks).reshape(n, -1)


def make_synthetic_model(cfg: T5Config | None = None, seed: int = 0, std: float = 0.02,
                         bias_std: float = 0.1, norm_weight: float = 1.0,
                         ff_norm_weight: float | None = None) -> SyntheticModel:
    """Random-init N(0, std) weights quantized to Q4_K, RMSNorm weights
    `norm_weight` (the feed-forward sub-layers' norms `ff_norm_weight` when
    given: a large value drives the gated-GELU output past the f16 range),
    relative-attention bias N(0, bias_std); tensor names as in the reference
    checkpoint (`src/quantized_t5.rs:514-516,582-590,639-646,682-690`)."""
    cfg = cfg or T5Config()
    rng = np.random.default_rng(seed)
    D, F, inner, H = cfg.d_model, cfg.d_ff, cfg.num_heads * cfg.d_kv, cfg.num_heads
    tensors = []
    m = SyntheticModel(config=cfg, gguf=b"")

    def add_q4k(name, rows, cols):
        w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)
        blocks = quantize_q4k(w)
        m.q4k[name] = blocks
        tensors.append((name, GGML_TYPE_Q4_K, (rows, cols), blocks.tobytes()))

    def add_f32(name, arr):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        m.f32[name] = arr
        tensors.append((name, GGML_TYPE_F32, arr.shape, arr.tobytes()))

    add_q4k("encoder.embed_tokens.weight", cfg.vocab_size, D)
    for i in range(cfg.num_layers):
        p = f"encoder.block.{i}.layer"
        for t in ("q", "k", "v"):
            add_q4k(f"{p}.0.SelfAttention.{t}.weight", inner, D)
        add_q4k(f"{p}.0.SelfAttention.o.weight", D, inner)
        if i == 0:
            add_f32(f"{p}.0.SelfAttention.relative_attention_bias.weight",
                    rng.standard_normal((cfg.relative_attention_num_buckets, H), dtype=np.float32) * np.float32(bias_std))
        add_f32(f"{p}.0.layer_norm.weight", np.full(D, norm_weight, np.float32))
        add_q4k(f"{p}.1.DenseReluDense.wi_0.weight", F, D)
        add_q4k(f"{p}.1.DenseReluDense.wi_1.weight", F, D)
        add_q4k(f"{p}.1.DenseReluDense.wo.weight", D, F)
        add_f32(f"{p}.1.layer_norm.weight",
                np.full(D, norm_weight if ff_norm_weight is None else ff_norm_weight, np.float32))
    add_f32("encoder.final_layer_norm.weight", np.full(D, norm_weight, np.float32))
    add_q4k("linear.weight", cfg.d_proj, D)
    m.gguf = write_gguf(tensors)
    return m
