"""match_centroids (src/lib.rs:600-887) over an in-memory index, scored on
the GPU (include/wc_query.h).

An index is a list of generations plus unindexed chunks:
  Generation(centers [n, 128] f32, buckets: list of Bucket), one bucket per
  center; Bucket(keys: list of (doc rowid, sub-chunk index), codes
  [rows, 64] u8 4-bit residual codes).  The bucket size is its row count
  (the reference's `sizes`).
  unindexed: list of (doc rowid, embeddings [rows, 128] f32).

`prepare` restates the reference's host logic: per generation the query-
centroid similarities, per query token the best clusters in descending
order until their sizes reach t' = 40000 (at most 32), the `missing` floor
when they do not, the union of the chosen buckets, and the candidates sorted
by (document, sub-chunk, position).  `finish` applies the cutoff
(max(threshold, mean missing)) and returns the top_k (score, doc, sub).
The scoring between them runs in `score_gpu`.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import WcError, lib

K_CLUSTERS = 32        # src/lib.rs:609
T_PRIME = 40000        # src/lib.rs:610


@dataclass
class Bucket:
    keys: list                 # [(doc rowid, sub index)] per row
    codes: np.ndarray          # [rows, dim / 2] u8


@dataclass
class Generation:
    centers: np.ndarray        # [n, dim] f32
    buckets: list              # Bucket per center


@dataclass
class Index:
    generations: list = field(default_factory=list)
    unindexed: list = field(default_factory=list)   # [(doc rowid, [rows, dim] f32)]


def _p(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def _check(rc: int) -> None:
    if rc != 0:
        msg = lib().wc_query_last_error()
        raise WcError(rc, msg.decode() if msg else "")


def similarities(q: np.ndarray, centers: np.ndarray) -> np.ndarray:
    dq, dc = torch.from_numpy(np.ascontiguousarray(q, np.float32)).cuda(), torch.from_numpy(
        np.ascontiguousarray(centers, np.float32)).cuda()
    out = torch.empty(q.shape[0], centers.shape[0], dtype=torch.float32, device="cuda")
    _check(lib().wc_similarities(_p(dq), q.shape[0], _p(dc), centers.shape[0], q.shape[1], _p(out),
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return out.cpu().numpy()


@dataclass
class Candidates:
    q: np.ndarray
    codes: np.ndarray
    cluster: np.ndarray        # global cluster column into cscores
    cscores: np.ndarray        # [m, total clusters]
    raw: np.ndarray
    group_rows: np.ndarray
    group_start: np.ndarray
    doc_start: np.ndarray
    group_keys: list           # (doc, sub) per group
    missing: np.ndarray


def prepare(index: Index, q: np.ndarray, sim_fn=similarities) -> Candidates | None:
    q = np.ascontiguousarray(q, np.float32)
    m, dim = q.shape
    missing = np.zeros(m, np.float32)
    codes, clusters, keys = [], [], []
    cs_cols, col0 = [], 0
    for gen in index.generations:
        n = len(gen.buckets)
        if n == 0:
            continue
        sim = sim_fn(q, gen.centers)                     # [m, n]
        sizes = np.array([len(b.keys) for b in gen.buckets])
        chosen = []
        for i in range(m):
            order = np.argsort(-sim[i], kind="stable")
            cum = 0
            for j in range(min(n, K_CLUSTERS)):
                chosen.append(int(order[j]))
                cum += int(sizes[order[j]])
                if cum >= T_PRIME:
                    break
            if cum < T_PRIME:
                missing[i] = max(missing[i], sim[i, order[min(n, K_CLUSTERS) - 1]])
        for c in sorted(set(chosen)):
            b = gen.buckets[c]
            rows = b.codes.shape[0]
            codes.append(b.codes)
            clusters.extend([col0 + c] * rows)
            keys.extend(b.keys[:rows])
        cs_cols.append(sim)
        col0 += n
    n_idx = len(keys)
    raws = []
    for doc, emb in index.unindexed:
        raws.append(np.asarray(emb, np.float32))
        keys.extend([(doc, 0)] * len(emb))
    if not keys:
        return None
    pos = sorted(range(len(keys)), key=lambda p: (keys[p], p))
    group_rows, group_start, doc_start, group_keys = [], [0], [0], []
    for p in pos:
        k = keys[p]
        if not group_keys or group_keys[-1] != k:
            if group_keys:
                group_start.append(len(group_rows))
                if group_keys[-1][0] != k[0]:
                    doc_start.append(len(group_keys))
            group_keys.append(k)
        group_rows.append(p)
    group_start.append(len(group_rows))
    doc_start.append(len(group_keys))
    return Candidates(
        q=q,
        codes=np.concatenate(codes) if codes else np.zeros((0, dim // 2), np.uint8),
        cluster=np.asarray(clusters, np.uint32),
        cscores=np.concatenate(cs_cols, axis=1) if cs_cols else np.zeros((m, 1), np.float32),
        raw=np.concatenate(raws) if raws else np.zeros((0, dim), np.float32),
        group_rows=np.asarray(group_rows, np.int64), group_start=np.asarray(group_start, np.int64),
        doc_start=np.asarray(doc_start, np.int64), group_keys=group_keys, missing=missing)


def q4_table() -> np.ndarray:
    """make_q4_dequant_table (src/packops.rs:14-24), from the library."""
    t = np.empty(16, np.float32)
    _check(lib().wc_q4_table(ctypes.c_void_p(t.ctypes.data)))
    return t


def score_gpu(c: Candidates, table: np.ndarray) -> np.ndarray:
    dev = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dt)).cuda()  # noqa: E731
    m, dim = c.q.shape
    dq, dcodes, dcl = dev(c.q, np.float32), dev(c.codes.reshape(-1), np.uint8), dev(c.cluster.view(np.int32), np.int32)
    dcs, dtab, draw = dev(c.cscores, np.float32), dev(table, np.float32), dev(c.raw.reshape(-1), np.float32)
    dgr, dgs, dds = (dev(a, np.int64) for a in (c.group_rows, c.group_start, c.doc_start))
    dmiss = dev(c.missing, np.float32)
    out = torch.empty(len(c.group_keys), dtype=torch.float32, device="cuda")
    nz = lambda t: _p(t) if t.numel() else None  # noqa: E731
    _check(lib().wc_score_candidates(_p(dq), m, dim, nz(dcodes), nz(dcl), _p(dcs), c.cscores.shape[1], _p(dtab),
                                     len(c.cluster), nz(draw), _p(dgr), _p(dgs), _p(dds), len(c.doc_start) - 1,
                                     _p(dmiss), _p(out), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return out.cpu().numpy()


def finish(c: Candidates, scores: np.ndarray, threshold: float, top_k: int):
    m = len(c.missing)
    s = np.float32(0.0)
    for v in c.missing:
        s = np.float32(s + v)
    missing_score = np.float32(s / np.float32(m))
    cutoff = missing_score if missing_score > threshold else np.float32(threshold)
    res = [(float(sc), int(k[0]), int(k[1])) for sc, k in zip(scores, c.group_keys) if sc > cutoff]
    res.sort(key=lambda r: -r[0])
    return res[:top_k]


def match_centroids(index: Index, q: np.ndarray, threshold: float, top_k: int):
    """[(score, doc rowid, sub index)] best first (src/lib.rs:600-887, no SQL filter)."""
    c = prepare(index, q)
    if c is None:
        return []
    return finish(c, score_gpu(c, q4_table()), threshold, top_k)
