"""The CPU oracle against the golden fixtures (tests/golden/make_golden.py):
gguf-py's Q4_K dequant, HF's relative-position buckets and HF's T5 encoder."""
import hashlib
import os

import numpy as np

from conftest import GOLDEN
from oracle import oracle as O
from witchcraft_b200.synth import dequantize_q4k_np, quantize_q4k


def _same_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    both_nan = np.isnan(a) & np.isnan(b)
    return np.all((a.view(np.uint32) == b.view(np.uint32)) | both_nan)


def test_q4k_dequant_matches_gguf_py_bit_exact():
    g = np.load(os.path.join(GOLDEN, "q4k_golden.npz"))
    assert _same_bits(O.q4k_dequant(g["blocks"]), g["values"])


def test_numpy_dequant_matches_oracle():
    g = np.load(os.path.join(GOLDEN, "q4k_golden.npz"))
    assert _same_bits(dequantize_q4k_np(g["blocks"]), O.q4k_dequant(g["blocks"]))


def test_quantizer_roundtrip_error_bounded():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((64, 768)).astype(np.float32) * 0.02
    deq = O.q4k_dequant_matrix(quantize_q4k(w))
    # one 4-bit step of a sub-block is at most range/15; rounding costs half of it
    step = (w.reshape(64, -1, 32).max(-1) - np.minimum(w.reshape(64, -1, 32).min(-1), 0)) / 15
    err = np.abs(deq - w).reshape(64, -1, 32).max(-1)
    assert np.all(err <= step * 0.75 + 1e-4)


def test_buckets_match_hf():
    g = np.load(os.path.join(GOLDEN, "buckets_golden.npz"))
    mine = np.array([O.bucket(0, d) if d >= 0 else O.bucket(-d, 0) for d in g["delta"]])
    assert np.array_equal(mine, g["bucket"])


def test_tiny_encoder_matches_hf(tiny_model):
    g = np.load(os.path.join(GOLDEN, "t5_tiny_golden.npz"))
    assert hashlib.sha256(tiny_model.gguf).digest() == g["gguf_sha256"].tobytes(), \
        "synthetic checkpoint generator changed; regenerate the fixtures"
    out = O.OracleEncoder(tiny_model).encode(g["ids"], g["lengths"])
    np.testing.assert_allclose(out, g["out"], atol=1e-4, rtol=1e-4)


def test_padded_batch_equals_single_rows(tiny_model):
    enc = O.OracleEncoder(tiny_model)
    rng = np.random.default_rng(4)
    ids = rng.integers(3, 512, (3, 40)).astype(np.uint32)
    lens = np.array([40, 23, 2], np.int32)
    batch = enc.encode(ids, lens)
    for b in range(3):
        single = enc.encode(ids[b:b + 1, :lens[b]])
        np.testing.assert_array_equal(batch[b, :lens[b]], single[0])
        assert np.all(batch[b, lens[b]:] == 0)


def test_torch_cpu_restatement_matches_oracle(tiny_model):
    """The torch-CPU f32 encoder bench.py times equals the C oracle."""
    from oracle.torch_ref import TorchCPUEncoder
    ids = np.random.default_rng(5).integers(3, 512, 37).astype(np.uint32)
    got = TorchCPUEncoder(tiny_model, threads=2).encode_one(ids)
    ref = O.OracleEncoder(tiny_model).encode(ids[None])[0]
    np.testing.assert_allclose(got, ref, atol=2e-4, rtol=1e-4)
