"""Query-side scoring kernels (csrc/query.cu) against the CPU oracle
(oracle/query.c): similarities and sub-chunk scores bit-identical, and the
whole match_centroids search equal to the oracle-scored one."""
import numpy as np
import pytest

from oracle import oracle as O
from test_query_host import _unit, make_index
from witchcraft_b200 import query as Qm

pytestmark = pytest.mark.gpu


def test_q4_table_and_similarities():
    assert np.array_equal(Qm.q4_table().view(np.uint32), O.q4_table().view(np.uint32))
    q, c = _unit(37, seed=1), _unit(300, seed=2)
    assert np.array_equal(Qm.similarities(q, c).view(np.uint32), O.similarities(q, c).view(np.uint32))


@pytest.mark.parametrize("m", [1, 20, 32, 45, 128])
def test_scores_bit_identical(m):
    index = make_index(seed=m)
    q = _unit(m, seed=m + 1)
    c = Qm.prepare(index, q, sim_fn=O.similarities)
    got = Qm.score_gpu(c, Qm.q4_table())
    want = O.score_candidates(c.q, c.codes, c.cluster, c.cscores, O.q4_table(), c.raw, c.group_rows,
                              c.group_start, c.doc_start, c.missing)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_match_centroids_end_to_end():
    index = make_index(seed=9, n_docs=200, n_cent=64)
    q = _unit(24, seed=10)
    got = Qm.match_centroids(index, q, threshold=0.0, top_k=20)
    c = Qm.prepare(index, q, sim_fn=O.similarities)
    want = Qm.finish(c, O.score_candidates(c.q, c.codes, c.cluster, c.cscores, O.q4_table(), c.raw, c.group_rows,
                                           c.group_start, c.doc_start, c.missing), 0.0, 20)
    assert got == want
    assert len(got) == 20


@pytest.mark.parametrize("m", [7, 32, 33])
def test_scores_ragged_groups_bit_identical(m):
    """Sub-chunks of 0 to 19 rows (an empty one keeps the running maxima of
    the document's earlier sub-chunks), documents without sub-chunks, and
    indexed rows mixed with raw (unindexed) rows, for the register-resident
    path (m <= 32) and the general one."""
    rng = np.random.default_rng(m)
    n_idx, n_raw, n_cent = 3000, 300, 64
    q = _unit(m, seed=m + 7)
    codes = rng.integers(0, 256, (n_idx, 64), dtype=np.uint8)
    cluster = rng.integers(0, n_cent, n_idx).astype(np.uint32)
    cs = (rng.standard_normal((m, n_cent)) * 0.2).astype(np.float32)
    raw = _unit(n_raw, seed=m + 8)
    rows, gstart, dstart = [], [0], [0]
    for _ in range(400):
        for _ in range(int(rng.integers(0, 5))):
            k = int(rng.integers(0, 20))
            rows.extend(int(r) for r in rng.integers(0, n_idx + n_raw, k))
            gstart.append(len(rows))
        dstart.append(len(gstart) - 1)
    c = Qm.Candidates(q=q, codes=codes, cluster=cluster, cscores=cs, raw=raw,
                      group_rows=np.array(rows, np.int64), group_start=np.array(gstart, np.int64),
                      doc_start=np.array(dstart, np.int64), group_keys=[(0, 0)] * (len(gstart) - 1),
                      missing=(rng.standard_normal(m) * 0.1).astype(np.float32))
    got = Qm.score_gpu(c, Qm.q4_table())
    want = O.score_candidates(q, codes, cluster, cs, O.q4_table(), raw, c.group_rows, c.group_start, c.doc_start,
                              c.missing)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
