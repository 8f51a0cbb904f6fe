"""Host logic of the Embedder mirror (src/embedder.rs:22-102) and of the
bulk-embedding planner, with a fake encoder so no GPU is needed."""
import numpy as np
import pytest

from witchcraft_b200 import shard
from witchcraft_b200.t5cuda import MAX_LEN, STRIDE, Embedder, _windows


class FakeModel:
    """Row-wise deterministic stand-in: each output row depends on its own
    sequence's valid tokens only, like the real encoder."""
    d_proj = 128

    def __init__(self):
        self.table = np.random.default_rng(0).standard_normal((40000, 128)).astype(np.float32)
        self.calls = []

    def forward(self, ids, lengths=None):
        ids = np.atleast_2d(ids)
        B, L = ids.shape
        lens = np.full(B, L) if lengths is None else np.asarray(lengths)
        self.calls.append((B, L))
        out = np.zeros((B, L, 128), np.float32)
        for b in range(B):
            n = lens[b]
            scale = 1.0 + 0.1 * (int(ids[b, :n].astype(np.int64).sum()) % 7)
            out[b, :n] = self.table[ids[b, :n]] * scale
            out[b, 1:n:5] *= 0.01  # some rows fall below the min-norm filter
        return out


def _reference_embed(model, ids):
    """Literal restatement of src/embedder.rs:37-94 for comparison."""
    n = len(ids)
    accum = [None] * n
    start = 0
    while True:
        end = min(start + MAX_LEN, n)
        chunk = model.forward(ids[start:end][None])[0]
        for i in range(chunk.shape[0]):
            g = start + i
            accum[g] = chunk[i].copy() if accum[g] is None else accum[g] + chunk[i]
        if end == n:
            break
        start = max(end - STRIDE, 0)
    kept = [v for v in accum if np.sqrt((v * v).sum()) >= 1.0]
    if not kept:
        raise ValueError
    m = np.stack(kept)[None]
    return m / np.sqrt((m * m).sum(axis=2, keepdims=True))


def test_windows_follow_reference_stride():
    assert list(_windows(10)) == [(0, 10)]
    assert list(_windows(2048)) == [(0, 2048)]
    assert list(_windows(2049)) == [(0, 2048), (1792, 2049)]
    assert list(_windows(5000)) == [(0, 2048), (1792, 3840), (3584, 5000)]


@pytest.mark.parametrize("n", [1, 7, 300, 2048, 2500, 5000])
def test_embed_ids_matches_reference_loop(n):
    m = FakeModel()
    ids = np.random.default_rng(n).integers(3, 40000, n).astype(np.uint32)
    got, offs = Embedder(m).embed_ids(ids)
    np.testing.assert_allclose(got, _reference_embed(m, ids), rtol=1e-6)
    assert len(offs) == got.shape[1]


def test_embed_batch_equals_single_docs():
    m = FakeModel()
    rng = np.random.default_rng(1)
    docs = [rng.integers(3, 40000, n).astype(np.uint32) for n in (5, 17, 300, 2100, 64, 64, 9, 4100)]
    e = Embedder(m)
    singles = [e.embed_ids(d)[0] for d in docs]
    batched = e.embed_ids_batch(docs, max_batch_tokens=4096)
    for s, (b, _) in zip(singles, batched):
        np.testing.assert_allclose(b, s, rtol=1e-5, atol=1e-6)
    assert all(B * L <= max(4096, L) for B, L in m.calls)


def test_all_filtered_is_an_error():
    class Tiny(FakeModel):
        def forward(self, ids, lengths=None):
            return super().forward(ids, lengths) * 1e-4
    with pytest.raises(ValueError):
        Embedder(Tiny()).embed_ids(np.array([5, 6, 7], np.uint32))


def test_plan_batches_cover_every_doc_once():
    lens = shard.config4_lengths(5000)
    batches = shard.plan_batches(lens, 16384)
    docs = np.concatenate([b.docs for b in batches])
    assert sorted(docs.tolist()) == list(range(5000))
    for b in batches:
        assert b.L == lens[b.docs].max()
        assert b.padded_tokens <= 16384
    owners = shard.assign_batches(batches, 8)
    assert sorted(sum(owners, [])) == list(range(len(batches)))
    loads = [sum(batches[i].padded_tokens for i in o) for o in owners]
    assert max(loads) - min(loads) <= 512 * 32


def test_config4_length_distribution():
    lens = shard.config4_lengths()
    assert lens.min() >= 16 and lens.max() <= 512
    assert 170 < lens.mean() < 195  # log-normal(5.0, 0.7) clipped
