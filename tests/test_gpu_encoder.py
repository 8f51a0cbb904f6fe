"""End-to-end parity of the CUDA encoder through the C ABI (wc_t5_forward)
against the CPU oracle and the HF-pinned golden output.

Tolerance (per token, on the L2-normalised 128-d output, which is what the
Embedder returns): cosine >= 0.999 and max-abs <= 2e-2."""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import oracle as O
from witchcraft_b200._lib import WcError
from witchcraft_b200.t5cuda import Embedder, T5EncoderModel

from gpu_util import cosine_rows

pytestmark = pytest.mark.gpu

COS_MIN = 0.999
MAX_ABS = 2e-2


def _normalise(v):
    n = np.linalg.norm(v, axis=-1, keepdims=True)
    return v / np.where(n > 0, n, 1)


def _check(gpu_raw, ref_raw, lengths):
    for b, n in enumerate(lengths):
        g, r = gpu_raw[b, :n], ref_raw[b, :n]
        cos = cosine_rows(g, r)
        assert cos.min() >= COS_MIN, (b, cos.min())
        assert np.abs(_normalise(g) - _normalise(r)).max() <= MAX_ABS, b
        assert np.all(gpu_raw[b, n:] == 0)


@pytest.fixture(scope="module")
def tiny_gpu(tiny_model):
    m = T5EncoderModel(tiny_model.gguf, tiny_model.config.to_json(), 0)
    yield m
    m.close()


@pytest.fixture(scope="module")
def xtr_gpu(xtr_model):
    m = T5EncoderModel(xtr_model.gguf, xtr_model.config.to_json(), 0)
    yield m
    m.close()


@pytest.fixture(scope="module")
def xtr_oracle(xtr_model):
    return O.OracleEncoder(xtr_model)


def test_tiny_matches_hf_golden(tiny_gpu):
    g = np.load(os.path.join(GOLDEN, "t5_tiny_golden.npz"))
    out = tiny_gpu.forward(g["ids"], g["lengths"])
    _check(out, g["out"], g["lengths"])


def test_xtr_config1_shape_matches_oracle(xtr_gpu, xtr_oracle):
    """Config 1 shape (L = 128, no padding) on 2 of its 16 rows, plus norms
    and normalised outputs."""
    ids = np.random.default_rng(1).integers(3, 32128, (2, 128)).astype(np.uint32)
    raw, norms, outn = xtr_gpu.forward_full(ids)
    ref = xtr_oracle.encode(ids)
    _check(raw, ref, [128, 128])
    np.testing.assert_allclose(norms, np.linalg.norm(raw, axis=-1), rtol=1e-5)
    np.testing.assert_allclose(outn, _normalise(raw), atol=1e-6)


def test_xtr_ragged_padded_batch(xtr_gpu, xtr_oracle):
    rng = np.random.default_rng(6)
    lengths = [300, 1, 64, 65, 129, 200]
    L = 300
    ids = rng.integers(3, 32128, (len(lengths), L)).astype(np.uint32)
    out = xtr_gpu.forward(ids, lengths)
    ref = xtr_oracle.encode(ids, lengths)
    _check(out, ref, lengths)
    # each row equals the unpadded single-sequence forward
    for b in (1, 3):
        single = xtr_gpu.forward(ids[b:b + 1, :lengths[b]])
        cos = cosine_rows(single[0], out[b, :lengths[b]])
        assert cos.min() > 0.9999


def test_xtr_query_shapes(xtr_gpu, xtr_oracle):
    """Config 5 shapes: 32-token padded queries, lengths U[4, 32]."""
    rng = np.random.default_rng(6)
    lengths = rng.integers(4, 33, 8).tolist()
    ids = rng.integers(3, 32128, (8, 32)).astype(np.uint32)
    _check(xtr_gpu.forward(ids, lengths), xtr_oracle.encode(ids, lengths), lengths)


@pytest.mark.parametrize("B,L,lengths", [(1, 32, [32]), (1, 20, [13]), (2, 16, [16, 5])])
def test_xtr_small_batch_path(xtr_gpu, xtr_oracle, B, L, lengths):
    """B * L <= 32 tokens: the small-M layer path (split-K GEMV kernels, the
    residual add in the RMSNorm that follows, small-L attention)."""
    ids = np.random.default_rng(B * 100 + L).integers(3, 32128, (B, L)).astype(np.uint32)
    _check(xtr_gpu.forward(ids, lengths), xtr_oracle.encode(ids, lengths), lengths)


def test_long_window_tiny(tiny_gpu, tiny_model):
    ids = np.random.default_rng(8).integers(3, 512, (1, 2048)).astype(np.uint32)
    _check(tiny_gpu.forward(ids), O.OracleEncoder(tiny_model).encode(ids), [2048])


def test_embedder_multi_window_tiny(tiny_gpu, tiny_model):
    """Embedder over a 2600-token document: two overlapping windows summed,
    min-norm filter, L2 (src/embedder.rs:22-102), CUDA vs oracle."""
    ids = np.random.default_rng(9).integers(3, 512, 2600).astype(np.uint32)
    got, offs = Embedder(tiny_gpu).embed_ids(ids)
    orc = O.OracleEncoder(tiny_model)

    class _OracleModel:
        d_proj = 128

        def forward(self, x, lengths=None):
            return orc.encode(np.atleast_2d(x), lengths)
    ref, roffs = Embedder(_OracleModel()).embed_ids(ids)
    assert offs == roffs
    assert cosine_rows(got[0], ref[0]).min() >= COS_MIN
    assert np.abs(got - ref).max() <= MAX_ABS


def test_embed_batch_matches_single(tiny_gpu):
    rng = np.random.default_rng(10)
    docs = [rng.integers(3, 512, n).astype(np.uint32) for n in (3, 40, 41, 300, 2100, 17)]
    e = Embedder(tiny_gpu)
    for (b, _), d in zip(e.embed_ids_batch(docs, max_batch_tokens=2048), docs):
        s, _ = e.embed_ids(d)
        assert cosine_rows(b[0], s[0]).min() > 0.9999


def test_forward_rejects_bad_input(tiny_gpu):
    with pytest.raises(WcError) as ei:
        tiny_gpu.forward(np.array([[1, 2, 99999]], np.uint32))
    assert ei.value.code == -1
    with pytest.raises(WcError):
        tiny_gpu.forward(np.zeros((2, 8), np.uint32), [8, 9])
    with pytest.raises(WcError):
        tiny_gpu.forward(np.zeros((1, 2049), np.uint32))


def test_two_handles_on_one_device(tiny_model):
    a = T5EncoderModel(tiny_model.gguf, tiny_model.config.to_json(), 0)
    b = T5EncoderModel(tiny_model.gguf, tiny_model.config.to_json(), 0)
    ids = np.random.default_rng(2).integers(3, 512, (2, 50)).astype(np.uint32)
    np.testing.assert_array_equal(a.forward(ids), b.forward(ids))
    a.close()
    np.testing.assert_array_equal(b.forward(ids), b.forward(ids))
    b.close()


def test_graph_replay_matches_eager(xtr_gpu, xtr_oracle):
    """Small batches replay a captured CUDA graph from their second call on;
    every call must still see its own inputs."""
    rng = np.random.default_rng(12)
    lengths = [32, 9]
    runs = []
    for i in range(4):
        ids = rng.integers(3, 32128, (2, 32)).astype(np.uint32)
        runs.append((ids, xtr_gpu.forward(ids, lengths)))
    for ids, out in runs:
        _check(out, xtr_oracle.encode(ids, lengths), lengths)
    again = xtr_gpu.forward(runs[0][0], lengths)
    np.testing.assert_array_equal(again, runs[0][1])


def test_forward_many_equals_single_calls(tiny_gpu):
    """The pipelined entry point gives each batch exactly its wc_t5_forward result."""
    rng = np.random.default_rng(21)
    batches = []
    for B, L in [(3, 40), (1, 7), (64, 20), (2, 300), (5, 33), (40, 64), (1, 1)]:
        ids = rng.integers(3, 512, (B, L)).astype(np.uint32)  # tiny model: vocab 512
        lens = rng.integers(1, L + 1, B).astype(np.int32)
        batches.append((ids, lens))
    for n in (len(batches), 2, 1):  # odd, even and single batch counts
        got, gn = tiny_gpu.forward_many(batches[:n], with_norms=True)
        for (ids, lens), o, nr in zip(batches[:n], got, gn):
            ref, rn, _ = tiny_gpu.forward_full(ids, lens)
            np.testing.assert_array_equal(o, ref)
            np.testing.assert_array_equal(nr, rn)


def test_forward_many_two_lanes(tiny_gpu):
    """Batches past the graph size alternate between two compute streams with
    separate activation buffers; every batch still equals its single call,
    including a small batch on the second lane."""
    rng = np.random.default_rng(22)
    batches = []
    for B, L in [(40, 128), (9, 600), (33, 160), (3, 25), (70, 64)]:
        ids = rng.integers(3, 512, (B, L)).astype(np.uint32)
        lens = rng.integers(1, L + 1, B).astype(np.int32)
        batches.append((ids, lens))
    got, gn = tiny_gpu.forward_many(batches, with_norms=True)
    for (ids, lens), o, nr in zip(batches, got, gn):
        ref, rn, _ = tiny_gpu.forward_full(ids, lens)
        np.testing.assert_array_equal(o, ref)
        np.testing.assert_array_equal(nr, rn)


def _check_rows(got, ids, lens, rows, oracle):
    """Rows `rows` of a padded batch against the oracle, each encoded alone
    at its own length (rows are independent under the padding mask)."""
    for b in rows:
        n = int(lens[b])
        ref = oracle.encode(ids[b:b + 1, :n])
        _check(got[b:b + 1, :n], ref, [n])
        assert np.all(got[b, n:] == 0)


def test_xtr_config1_full_batch(xtr_gpu, xtr_oracle):
    """Config 1 in full: B = 16, L = 128, no padding (M = 2048 takes the
    2-SM GEMM path on the resident f16 weights)."""
    ids = np.random.default_rng(1).integers(3, 32128, (16, 128)).astype(np.uint32)
    raw = xtr_gpu.forward(ids)
    _check(raw, xtr_oracle.encode(ids), [128] * 16)


def test_xtr_config3_lengths_through_encoder(xtr_gpu, xtr_oracle):
    """Config-3 lengths through the whole encoder: one padded batch of
    sequences of 512, 257 and 32 tokens (persistent tcgen05 attention with
    the key padding mask, M = 1536)."""
    lens = np.array([512, 257, 32], np.int32)
    ids = np.random.default_rng(31).integers(3, 32128, (3, 512)).astype(np.uint32)
    out = xtr_gpu.forward(ids, lens)
    _check_rows(out, ids, lens, range(3), xtr_oracle)


def test_xtr_config4_batches_two_lanes(xtr_gpu, xtr_oracle):
    """Real config-4 batches (about 16k padded tokens each) through the
    pipelined two-lane entry point wc_t5_forward_many, a seeded sample of 8
    rows per batch against the oracle.  Three batches put the first and third
    on one compute lane and the second on the other."""
    from witchcraft_b200 import shard
    lengths = shard.config4_lengths()
    batches = shard.plan_batches(lengths)
    Ls = np.array([b.L for b in batches])
    pick = [int(np.argmin(np.abs(Ls - 512))), int(np.argmin(np.abs(Ls - 128))), int(np.argmin(np.abs(Ls - 256)))]
    rng = np.random.default_rng(41)
    inputs = []
    for i in pick:
        b = batches[i]
        lens = lengths[b.docs].astype(np.int32)
        ids = np.zeros((len(b.docs), b.L), np.uint32)
        for r, n in enumerate(lens):
            ids[r, :n] = rng.integers(3, 32128, n)
        assert len(b.docs) * b.L > 12000
        inputs.append((ids, lens))
    outs = xtr_gpu.forward_many(inputs)
    for (ids, lens), out in zip(inputs, outs):
        rows = sorted(set(rng.choice(len(lens), 7, replace=False).tolist()) | {int(np.argmax(lens))})
        _check_rows(out, ids, lens, rows, xtr_oracle)


def test_forward_many_device_equals_single_calls(tiny_gpu):
    """wc_t5_forward_many_device (device-resident batches, two compute lanes
    joined back into the caller's stream) gives every batch exactly its
    wc_t5_forward_device result."""
    import torch
    rng = np.random.default_rng(23)
    shapes = [(40, 128), (9, 600), (33, 160), (3, 25), (70, 64)]
    dev, outs, refs = [], [], []
    for B, L in shapes:
        ids = torch.from_numpy(rng.integers(3, 512, (B, L)).astype(np.uint32)).cuda()
        lens = torch.from_numpy(rng.integers(1, L + 1, B).astype(np.int32)).cuda()
        o = torch.full((B * L, 128), float("nan"), device="cuda")
        nr = torch.full((B * L,), float("nan"), device="cuda")
        dev.append((ids, lens))
        outs.append((o, nr))
        refs.append((torch.empty_like(o), torch.empty_like(nr)))
    st = torch.cuda.Stream()
    tiny_gpu.forward_many_device([(i.data_ptr(), l.data_ptr(), i.shape[0], i.shape[1], o.data_ptr(), n.data_ptr())
                                  for (i, l), (o, n) in zip(dev, outs)], st.cuda_stream)
    tiny_gpu.sync(st.cuda_stream)
    for (i, l), (o, n) in zip(dev, refs):
        tiny_gpu.forward_device(i.data_ptr(), l.data_ptr(), i.shape[0], i.shape[1], o.data_ptr(), n.data_ptr(), None,
                                st.cuda_stream)
    tiny_gpu.sync(st.cuda_stream)
    for (o, n), (ro, rn) in zip(outs, refs):
        assert torch.equal(o, ro) and torch.equal(n, rn)


def test_fused_q4k_weights_handle_bitwise(xtr_model, xtr_gpu):
    """A handle created with WC_F16_WEIGHTS=0 keeps no f16 weight copies; its
    large-M GEMMs dequantise the Q4_K super-blocks in the kernel into the same
    f16 operand bits, so every output equals the default handle's."""
    os.environ["WC_F16_WEIGHTS"] = "0"
    try:
        fused = T5EncoderModel(xtr_model.gguf, xtr_model.config.to_json(), 0)
    finally:
        del os.environ["WC_F16_WEIGHTS"]
    try:
        rng = np.random.default_rng(51)
        for B, L in ((16, 128), (3, 300), (40, 200)):
            ids = rng.integers(3, 32128, (B, L)).astype(np.uint32)
            lens = rng.integers(1, L + 1, B).astype(np.int32)
            np.testing.assert_array_equal(fused.forward(ids, lens), xtr_gpu.forward(ids, lens))
    finally:
        fused.close()
