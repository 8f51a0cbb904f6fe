"""CUDA index-build kernels (csrc/index.cu) against the CPU oracle
(oracle/index.c): assignments and k-means centers bit-identical (same fused
multiply-add chains, same summation order), residual codes identical except
where logf's last bit differs between libm and CUDA."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from witchcraft_b200 import index as I

pytestmark = pytest.mark.gpu


def _unit(n, d=128, seed=0):
    x = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)
    return x / np.linalg.norm(x, axis=1, keepdims=True)


@pytest.mark.parametrize("m,k,d", [(1, 1, 128), (300, 77, 128), (1000, 1000, 128), (257, 129, 64), (5, 300, 4)])
def test_assign_bit_identical(m, k, d):
    x, c = _unit(m, d, seed=m), _unit(k, d, seed=k)
    got = I.assign(torch.from_numpy(x).cuda(), torch.from_numpy(c).cuda()).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, O.assign_centers(x, c))


def test_assign_ties_pick_first_center():
    c = _unit(50, seed=1)
    c2 = np.concatenate([c, c, c])
    got = I.assign(torch.from_numpy(c).cuda(), torch.from_numpy(c2).cuda()).cpu().numpy()
    assert got.tolist() == list(range(50))


def test_kmeans_update_bit_identical():
    x = _unit(3000, seed=2)
    k = 60
    idx = np.random.default_rng(3).integers(0, k - 4, len(x)).astype(np.uint32)
    empty = (np.arange(k) * 11).astype(np.int64)
    got, counts = I.kmeans_update(torch.from_numpy(x).cuda(), torch.from_numpy(idx.view(np.int32)).cuda(), k,
                                  torch.from_numpy(empty).cuda())
    want, wcounts = O.kmeans_update(x, idx, k, empty)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert np.array_equal(counts.cpu().numpy().view(np.uint32), wcounts)


def test_kmeans_loop_matches_oracle_loop():
    x = _unit(2000, seed=4)
    k, iters = 32, 3
    init = np.random.default_rng(5).choice(len(x), k, replace=False)
    got = I.kmeans(torch.from_numpy(x).cuda(), k, iters, init).cpu().numpy()
    c = x[init]
    for _ in range(iters):
        idx = O.assign_centers(x, c)
        c, _ = O.kmeans_update(x, idx, k, np.zeros(k, np.int64))
    assert np.array_equal(got.view(np.uint32), c.view(np.uint32))


def test_residual_codes():
    x, c = _unit(4000, seed=6), _unit(64, seed=7)
    idx = O.assign_centers(x, c)
    got = I.residual_q4(torch.from_numpy(x).cuda(), torch.from_numpy(idx.view(np.int32)).cuda(),
                        torch.from_numpy(c).cuda()).cpu().numpy()
    want = O.residual_q4(x, idx, c)
    assert (got == want).mean() > 0.9999
