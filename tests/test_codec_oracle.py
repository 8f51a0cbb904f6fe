"""CPU oracle of the packed-embedding codec (oracle/codec.c, restating
src/packops.rs:172-438, src/haarops.rs, src/rans64.rs).  The reference pins
no vectors for it (its packops tests are commented out and the Rust cannot
be built here), so these are structural and round-trip properties."""
import numpy as np
import pytest

from oracle import oracle as O


def _rows(n, cols=128, seed=0):
    e = np.random.default_rng(seed).standard_normal((n, cols)).astype(np.float32)
    return e / np.linalg.norm(e, axis=1, keepdims=True)


def _parse(buf, cols):
    """Window headers of one packed document (layout of src/packops.rs:172-301)."""
    b = np.frombuffer(buf, np.uint8)
    rows = int(b[:4].view(np.uint32)[0])
    p, wins = 4, []
    for r in range(0, rows, 1024):
        perm = b[p:p + cols]
        p += cols
        m = int(b[p:p + 2].view(np.uint16)[0])
        p += 2
        pairs = b[p:p + 4 * m].view(np.uint16).reshape(m, 2)
        p += 4 * m
        n = int(b[p:p + 2].view(np.uint16)[0])
        p += 2 + n
        wins.append((perm.copy(), pairs.copy(), n))
    assert p == len(b)
    return rows, wins


@pytest.mark.parametrize("rows", [1, 2, 3, 31, 100, 1024, 1025, 2100])
def test_layout_and_round_trip(rows):
    e = _rows(rows, seed=rows)
    buf = O.pack_embeddings(e)
    n, wins = _parse(buf, 128)
    assert n == rows and len(wins) == (rows + 1023) // 1024
    for perm, pairs, _ in wins:
        assert sorted(perm.tolist()) == list(range(128))     # a permutation
        assert np.all(np.diff(pairs[:, 0].astype(int)) > 0)  # symbols ascending
        assert int(pairs[:, 1].astype(int).sum()) == 4096    # frequencies normalised to 2^12
        assert pairs[:, 1].min() >= 1
    d = O.unpack_embeddings(buf)
    assert d.shape == e.shape
    assert (d * e).sum(1).min() > 0.99
    np.testing.assert_allclose(np.linalg.norm(d, axis=1), 1.0, atol=1e-5)


def test_deterministic_and_column_order_by_sum():
    e = _rows(300, seed=5)
    assert O.pack_embeddings(e) == O.pack_embeddings(e.copy())
    _, wins = _parse(O.pack_embeddings(e), 128)
    inv = wins[0][0]
    sums = e.sum(0, dtype=np.float32)
    order = np.argsort(sums, kind="stable")  # ascending, ties by index
    assert np.array_equal(inv[order], np.arange(128))


@pytest.mark.parametrize("cols", [1, 2, 7, 255])
def test_other_widths(cols):
    e = _rows(40, cols=cols, seed=cols)
    d = O.unpack_embeddings(O.pack_embeddings(e), cols)
    assert d.shape == e.shape
    if cols > 2:
        assert (d * e).sum(1).min() > 0.95


def test_rejects_malformed_streams():
    buf = O.pack_embeddings(_rows(50))
    with pytest.raises(ValueError):
        O.unpack_embeddings(buf[:-1])
    with pytest.raises(ValueError):
        O.unpack_embeddings(buf + b"\\0")
    with pytest.raises(ValueError):
        O.pack_embeddings(np.zeros((2, 256), np.float32))
