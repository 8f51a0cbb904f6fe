"""Batched Gatherer / embed_chunks driver (src/lib.rs:901-1003, 1044-1135)
with the row-deterministic fake encoder, so no GPU is needed."""
import numpy as np
import pytest

from test_embedder_host import FakeModel
from witchcraft_b200.gather import Document, Gatherer, chunk_counts, embed_chunks
from witchcraft_b200.t5cuda import Embedder


def _reference_counts(offsets, lens):
    """Literal restatement of the reference loop (src/lib.rs:948-992)."""
    lengths = []
    for s in lens.split(","):
        try:
            if s.strip() != s or s.startswith("-"):
                raise ValueError
            lengths.append(int(s))
        except ValueError:
            pass
    for i in range(1, len(lengths)):
        lengths[i] += lengths[i - 1]
    i = j = 0
    count, done, flush, counts = 0, False, False, []
    while not done:
        o = offsets[i][1] if i < len(offsets) else 2**64 - 1
        l = lengths[j] if j < len(lengths) else 2**64 - 1
        if o <= l:
            i += 1
            count += 1
        else:
            j += 1
            flush = True
        done = i == len(offsets) and j == len(lengths)
        if flush or done:
            counts.append(count)
            count = 0
            flush = False
    return counts


def test_chunk_counts_cases():
    offs = [(0, 3), (4, 9), (10, 12), (13, 20), (21, 25)]
    assert chunk_counts(offs, "10,10,5") == [2, 2, 1]
    assert chunk_counts(offs, "12,13") == [3, 2]
    # a boundary no row reaches closes an empty sub-chunk
    assert chunk_counts(offs, "2,10,13") == [0, 3, 2]
    # rows past the last boundary form one trailing group
    assert chunk_counts(offs, "9") == [2, 3]
    # no sub-chunks: everything in one group; unparsable entries are skipped
    assert chunk_counts(offs, "") == [5]
    assert chunk_counts(offs, "x,10,,15") == [2, 3]
    assert chunk_counts([], "4,4") == [0, 0]
    with pytest.raises(ValueError):
        chunk_counts([], "")


def test_chunk_counts_match_reference_loop_random():
    rng = np.random.default_rng(7)
    for _ in range(300):
        n = int(rng.integers(0, 40))
        ends = np.sort(rng.integers(1, 400, n))
        offs = [(int(e) - 1, int(e)) for e in ends]
        k = int(rng.integers(0, 8))
        if n == 0 and k == 0:
            continue  # unreachable in the reference (its Embedder fails first)
        lens = ",".join(str(int(v)) for v in rng.integers(0, 120, k))
        got = chunk_counts(offs, lens)
        assert got == _reference_counts(offs, lens)
        assert sum(got) == n


def _docs(n, seed=3):
    rng = np.random.default_rng(seed)
    docs = []
    for d in range(n):
        L = int(rng.integers(3, 700)) if d % 7 else 2300  # some multi-window
        ids = rng.integers(3, 32128, L).astype(np.uint32)
        ends = np.cumsum(rng.integers(1, 6, L))
        offs = [(int(e) - 1, int(e)) for e in ends]
        parts = rng.integers(1, 4)
        cuts = np.sort(rng.integers(1, int(ends[-1]), parts))
        lens = ",".join(str(int(c)) for c in np.diff(np.concatenate([[0], cuts, [ends[-1]]])))
        docs.append(Document(f"h{d}", ids, offs, lens))
    return docs


def test_batched_gatherer_equals_per_document_path():
    emb = Embedder(FakeModel())
    docs = _docs(23)
    got = list(Gatherer(docs, emb, group_docs=5, max_batch_tokens=4096))
    assert [g[0] for g in got] == [d.hash for d in docs]
    for (h, e, counts), d in zip(got, docs):
        ref_e, ref_off = Embedder(FakeModel()).embed_ids(d.ids, d.offsets)
        np.testing.assert_allclose(e, ref_e[0], rtol=1e-5, atol=1e-6)
        assert counts == _reference_counts(ref_off, d.lens)
        assert sum(counts) == e.shape[0]


def test_embed_chunks_payload_and_counts_string():
    emb = Embedder(FakeModel())
    docs = _docs(4, seed=9)
    out = list(embed_chunks(docs, emb, pack=lambda e: e.shape, group_docs=3))
    assert [o[0] for o in out] == [d.hash for d in docs]
    for (_h, shape, cstr), d in zip(out, docs):
        assert shape[1] == 128
        assert sum(int(c) for c in cstr.split(",")) == shape[0]
