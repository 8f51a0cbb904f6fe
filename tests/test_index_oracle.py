"""CPU oracle of the index-build steps (oracle/index.c; src/lib.rs:187-274,
1376) against direct numpy statements of the same loops."""
import numpy as np

from oracle import oracle as O


def _unit(n, d=128, seed=0):
    x = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)
    return x / np.linalg.norm(x, axis=1, keepdims=True)


def test_assign_matches_argmax():
    x, c = _unit(300, seed=1), _unit(77, seed=2)
    got = O.assign_centers(x, c)
    sim = x.astype(np.float64) @ c.astype(np.float64).T
    top2 = np.sort(sim, axis=1)[:, -2:]
    clear = top2[:, 1] - top2[:, 0] > 1e-5   # away from near-ties f32 may order differently
    assert np.array_equal(got[clear], sim.argmax(1)[clear])
    # exact ties resolve to the first center
    c2 = np.concatenate([c[:5], c[:5]])
    assert O.assign_centers(c[:5], c2).tolist() == list(range(5))


def test_kmeans_update_follows_reference_loop():
    x = _unit(500, seed=3)
    k = 40
    idx = np.random.default_rng(4).integers(0, k - 3, len(x)).astype(np.uint32)  # last 3 clusters empty
    empty = np.arange(k, dtype=np.int64) * 7
    got, counts = O.kmeans_update(x, idx, k, empty)
    for c in range(k):
        members = x[idx == c]
        if len(members):
            s = np.zeros(128, np.float32)
            for r in members:
                s = (s + r).astype(np.float32)
        else:
            s = x[empty[c]]
        nrm = np.float32(np.sqrt(np.float32(sum(np.float32(v * v) for v in s))))
        np.testing.assert_allclose(got[c], s / nrm, rtol=1e-6, atol=1e-7)
        assert counts[c] == len(members)


def test_residual_codes():
    x, c = _unit(64, seed=5), _unit(8, seed=6)
    idx = O.assign_centers(x, c)
    got = O.residual_q4(x, idx, c)
    r = (x - c[idx]) * 4
    y = np.sign(r) * np.log1p(np.abs(r) * 255) / np.log(256)
    q = np.clip(np.round(y * 7.5 + 7.5), 0, 15).astype(np.uint8)
    want = (q[:, 0::2] << 4) | q[:, 1::2]
    assert (got == want).mean() > 0.999  # float64 numpy vs f32 ops: rare rounding flips only
