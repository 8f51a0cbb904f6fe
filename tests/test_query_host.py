"""match_centroids host logic (witchcraft_b200/query.py) with the CPU scorer
against a literal restatement of the reference loop (src/lib.rs:600-887)."""
import numpy as np

from oracle import oracle as O
from witchcraft_b200 import query as Qm


def _unit(n, d=128, seed=0):
    x = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)
    return x / np.linalg.norm(x, axis=1, keepdims=True)


def make_index(seed=0, n_docs=40, n_cent=24, gens=2):
    rng = np.random.default_rng(seed)
    idx = Qm.Index()
    for g in range(gens):
        centers = _unit(n_cent, seed=seed * 10 + g)
        buckets = []
        emb = _unit(400, seed=seed * 10 + g + 100)
        assign = O.assign_centers(emb, centers)
        codes = O.residual_q4(emb, assign, centers)
        for c in range(n_cent):
            rows = np.nonzero(assign == c)[0]
            keys = [(int(rng.integers(0, n_docs)), int(rng.integers(0, 3))) for _ in rows]
            buckets.append(Qm.Bucket(keys, codes[rows]))
        idx.generations.append(Qm.Generation(centers, buckets))
    for d in range(3):
        idx.unindexed.append((n_docs + d, _unit(5, seed=seed + 500 + d)))
    return idx


def reference_loop(index, q, threshold, top_k, k=32, t_prime=40000):
    """Literal restatement of match_centroids (no SQL filter), f32 throughout."""
    table = O.q4_table()
    m = q.shape[0]
    missing = np.zeros(m, np.float32)
    sims, all_ = [], []
    for gen in index.generations:
        n = len(gen.buckets)
        sim = (q @ gen.centers.T).astype(np.float32)
        sizes = [len(b.keys) for b in gen.buckets]
        top = []
        for i in range(m):
            order = np.argsort(-sim[i], kind="stable")
            cum = 0
            for j in range(min(n, k)):
                top.append(int(order[j]))
                cum += sizes[order[j]]
                if cum >= t_prime:
                    break
            if cum < t_prime:
                missing[i] = max(missing[i], sim[i, order[min(n, k) - 1]])
        for c in sorted(set(top)):
            b = gen.buckets[c]
            res = np.stack([np.concatenate([[table[x >> 4], table[x & 15]] for x in row]) for row in b.codes])
            for r, key in enumerate(b.keys[:len(res)]):
                sims.append((q @ res[r]).astype(np.float32) + sim[:, c])
                all_.append((key, len(all_)))
    for doc, emb in index.unindexed:
        for r in emb:
            sims.append((q @ r).astype(np.float32))
            all_.append(((doc, 0), len(all_)))
    if not all_:
        return []
    s = np.float32(0)
    for v in missing:
        s = np.float32(s + v)
    ms = np.float32(s / np.float32(m))
    cutoff = ms if ms > threshold else np.float32(threshold)
    all_.sort()
    sub, doc = missing.copy(), missing.copy()
    out, prev = [], None
    for i in range(len(all_) + 1):
        end = i == len(all_)
        key, pos = (None, None) if end else all_[i]
        if i > 0:
            if end or key != prev:
                sc = np.float32(np.float32(1) / np.float32(m)) * np.float32(sub.astype(np.float64).sum())
                if sc > cutoff:
                    out.append((float(sc), prev[0], prev[1]))
                doc = np.maximum(doc, sub)
                sub = doc.copy()
            if end or key[0] != prev[0]:
                doc, sub = missing.copy(), missing.copy()
        if end:
            break
        sub = np.maximum(sub, sims[pos])
        prev = key
    out.sort(key=lambda r: -r[0])
    return out[:top_k]


def _cpu_sim(q, c):
    return (q @ c.T).astype(np.float32)


def test_prepare_and_finish_match_reference_loop():
    index = make_index(seed=1)
    q = _unit(20, seed=77)
    c = Qm.prepare(index, q, sim_fn=_cpu_sim)
    scores = O.score_candidates(c.q, c.codes, c.cluster, c.cscores, O.q4_table(), c.raw, c.group_rows,
                                c.group_start, c.doc_start, c.missing)
    got = Qm.finish(c, scores, threshold=0.0, top_k=15)
    want = reference_loop(index, q, 0.0, 15)
    assert [(d, s) for _, d, s in got] == [(d, s) for _, d, s in want]
    np.testing.assert_allclose([g[0] for g in got], [w[0] for w in want], rtol=1e-5, atol=1e-6)


def test_small_bucket_sizes_raise_missing_floor():
    index = make_index(seed=2, n_cent=8)
    q = _unit(6, seed=5)
    c = Qm.prepare(index, q, sim_fn=_cpu_sim)
    # all 8 clusters together hold far fewer than t' rows: every token's floor is
    # its 8th-best centroid similarity (the smaller over the two generations kept by max)
    assert np.all(c.missing > -1.0)
    assert len(set(c.cluster.tolist())) == 16  # every cluster of both generations was read


def test_empty_index():
    assert Qm.prepare(Qm.Index(), _unit(3), sim_fn=_cpu_sim) is None
