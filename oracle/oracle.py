"""ctypes front end of the CPU oracle (oracle.c).  TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU legs (the
cpu_baseline measurement and `--impl reference`), always as the checker or
the timed CPU restatement of the reference, never as part of the product
path.  See oracle.c's header for the reference lines each function follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
_lib = None

_fp = ctypes.POINTER(ctypes.c_float)


def lib():
    global _lib
    if _lib is None:
        srcs = [os.path.join(HERE, f) for f in ("oracle.c", "codec.c", "index.c", "query.c", "Makefile")]
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(os.path.getmtime(f) for f in srcs):
            subprocess.run(["make", "-C", HERE, "CC=gcc"], check=True, capture_output=True)
        l = ctypes.CDLL(LIB_PATH)
        l.oracle_q4k_dequant.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        l.oracle_t5_bucket.argtypes = [ctypes.c_int] * 4
        l.oracle_t5_bucket.restype = ctypes.c_int
        l.oracle_attention.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        l.oracle_t5_encode.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_void_p]
        l.oracle_gemm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3
        l.oracle_pack.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64]
        l.oracle_pack.restype = ctypes.c_int64
        l.oracle_unpack.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64]
        l.oracle_unpack.restype = ctypes.c_int64
        l.oracle_packed_bound.argtypes = [ctypes.c_int64, ctypes.c_int]
        l.oracle_packed_bound.restype = ctypes.c_int64
        l.oracle_assign.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                    ctypes.c_void_p]
        l.oracle_kmeans_update.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                           ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        l.oracle_residual_q4.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p]
        l.oracle_q4_table.argtypes = [ctypes.c_void_p]
        l.oracle_similarities.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                          ctypes.c_void_p]
        l.oracle_score_candidates.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                              ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        l.oracle_num_threads.restype = ctypes.c_int
        l.oracle_set_threads.argtypes = [ctypes.c_int]
        _lib = l
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def num_threads() -> int:
    return lib().oracle_num_threads()


def q4k_dequant(blocks: np.ndarray) -> np.ndarray:
    """[..., 144] uint8 Q4_K blocks -> float32 [..., 256] (reference arithmetic)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    lead = b.shape[:-1]
    n = int(np.prod(lead)) if lead else 1
    out = np.empty((n, 256), np.float32)
    lib().oracle_q4k_dequant(_ptr(b), n, _ptr(out))
    return out.reshape(*lead, 256)


def q4k_dequant_matrix(blocks: np.ndarray) -> np.ndarray:
    """[N, K/256, 144] -> float32 [N, K]."""
    return q4k_dequant(blocks).reshape(blocks.shape[0], -1)


def bucket(i: int, j: int, num_buckets: int = 32, max_distance: int = 128) -> int:
    return lib().oracle_t5_bucket(i, j, num_buckets, max_distance)


def gemm(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """y = x w^T in f32."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty((x.shape[0], w.shape[0]), np.float32)
    lib().oracle_gemm(_ptr(x), _ptr(w), _ptr(y), x.shape[0], w.shape[0], x.shape[1])
    return y


def attention(qkv: np.ndarray, B: int, L: int, H: int, lengths, bias_tab: np.ndarray,
              num_buckets: int = 32, max_distance: int = 128) -> np.ndarray:
    """qkv f32 [B*L, 3*H*64] -> f32 [B*L, H*64]; rows past lengths[b] are 0."""
    qkv = np.ascontiguousarray(qkv, np.float32)
    lens = np.ascontiguousarray(lengths, np.int32)
    bias_tab = np.ascontiguousarray(bias_tab, np.float32)
    out = np.empty((B * L, H * 64), np.float32)
    lib().oracle_attention(_ptr(qkv), B, L, H, 64, _ptr(lens), _ptr(bias_tab), num_buckets, max_distance, _ptr(out))
    return out


class _Weights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("vocab", "d_model", "n_heads", "d_kv", "d_ff", "n_layers",
                                            "num_buckets", "max_distance", "d_proj")] + [
        ("eps", ctypes.c_float), ("embed", _fp), ("rel_bias", _fp),
        ("ln0", ctypes.POINTER(_fp)), ("wq", ctypes.POINTER(_fp)), ("wk", ctypes.POINTER(_fp)),
        ("wv", ctypes.POINTER(_fp)), ("wo_attn", ctypes.POINTER(_fp)), ("ln1", ctypes.POINTER(_fp)),
        ("wi0", ctypes.POINTER(_fp)), ("wi1", ctypes.POINTER(_fp)), ("wo_ff", ctypes.POINTER(_fp)),
        ("final_ln", _fp), ("proj", _fp)]


class OracleEncoder:
    """The reference's f32 CPU encoder over a SyntheticModel's Q4_K bytes
    (weights dequantised to f32 at load, as src/quantized_t5.rs:43-45 does)."""

    def __init__(self, model):
        cfg = model.config
        self.cfg = cfg
        keep = []

        def q(name):
            a = q4k_dequant_matrix(model.q4k[name])
            keep.append(a)
            return a.ctypes.data_as(_fp)

        def f(name):
            a = np.ascontiguousarray(model.f32[name], np.float32)
            keep.append(a)
            return a.ctypes.data_as(_fp)

        nl = cfg.num_layers
        arr = lambda: (_fp * nl)()  # noqa: E731
        ln0, wq, wk, wv, wo, ln1, wi0, wi1, wof = (arr() for _ in range(9))
        for i in range(nl):
            p = f"encoder.block.{i}.layer"
            wq[i] = q(f"{p}.0.SelfAttention.q.weight")
            wk[i] = q(f"{p}.0.SelfAttention.k.weight")
            wv[i] = q(f"{p}.0.SelfAttention.v.weight")
            wo[i] = q(f"{p}.0.SelfAttention.o.weight")
            ln0[i] = f(f"{p}.0.layer_norm.weight")
            wi0[i] = q(f"{p}.1.DenseReluDense.wi_0.weight")
            wi1[i] = q(f"{p}.1.DenseReluDense.wi_1.weight")
            wof[i] = q(f"{p}.1.DenseReluDense.wo.weight")
            ln1[i] = f(f"{p}.1.layer_norm.weight")
        self.w = _Weights(cfg.vocab_size, cfg.d_model, cfg.num_heads, cfg.d_kv, cfg.d_ff, nl,
                          cfg.relative_attention_num_buckets, cfg.relative_attention_max_distance, cfg.d_proj,
                          cfg.layer_norm_epsilon, q("encoder.embed_tokens.weight"),
                          f("encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight"),
                          ln0, wq, wk, wv, wo, ln1, wi0, wi1, wof,
                          f("encoder.final_layer_norm.weight"), q("linear.weight"))
        self._keep = (keep, ln0, wq, wk, wv, wo, ln1, wi0, wi1, wof)

    def encode(self, ids: np.ndarray, lengths=None) -> np.ndarray:
        """ids u32 [B, L] -> raw projection f32 [B, L, 128]; rows past lengths[b] are 0."""
        ids = np.ascontiguousarray(ids, np.uint32)
        B, L = ids.shape
        lens = np.ascontiguousarray(np.full(B, L) if lengths is None else lengths, np.int32)
        out = np.empty((B, L, self.cfg.d_proj), np.float32)
        lib().oracle_t5_encode(ctypes.addressof(self.w), _ptr(ids), _ptr(lens), B, L, _ptr(out))
        return out


def pack_embeddings(emb: np.ndarray) -> bytes:
    """embeddings_to_packed (src/packops.rs:172-301) of one [rows, cols] f32 matrix."""
    emb = np.ascontiguousarray(emb, np.float32)
    rows, cols = emb.shape
    cap = lib().oracle_packed_bound(rows, cols)
    out = np.empty(cap, np.uint8)
    n = lib().oracle_pack(emb.ctypes.data, rows, cols, out.ctypes.data, cap)
    if n < 0:
        raise ValueError("embeddings_to_packed failed")
    return out[:n].tobytes()


def unpack_embeddings(buf: bytes, cols: int = 128) -> np.ndarray:
    """embeddings_from_packed (src/packops.rs:303-438) -> [rows, cols] f32, L2-normalised."""
    b = np.frombuffer(buf, np.uint8)
    rows = int(b[:4].view(np.uint32)[0]) if len(b) >= 4 else 0
    out = np.empty(max(rows, 1) * cols, np.float32)
    n = lib().oracle_unpack(b.ctypes.data, len(b), cols, out.ctypes.data, out.size)
    if n < 0:
        raise ValueError("malformed packed embeddings")
    return out[: n * cols].reshape(n, cols)


def assign_centers(x: np.ndarray, centers: np.ndarray) -> np.ndarray:
    """matmul_argmax_batched (src/lib.rs:187-208): first argmax of x c^T per row."""
    x = np.ascontiguousarray(x, np.float32)
    c = np.ascontiguousarray(centers, np.float32)
    out = np.empty(len(x), np.uint32)
    lib().oracle_assign(x.ctypes.data, len(x), c.ctypes.data, len(c), x.shape[1], out.ctypes.data)
    return out


def kmeans_update(x: np.ndarray, idx: np.ndarray, k: int, empty_src: np.ndarray):
    """One k-means update (src/lib.rs:238-274) -> (centers [k, dim], counts)."""
    x = np.ascontiguousarray(x, np.float32)
    idx = np.ascontiguousarray(idx, np.uint32)
    es = np.ascontiguousarray(empty_src, np.int64)
    out = np.empty((k, x.shape[1]), np.float32)
    counts = np.empty(k, np.uint32)
    lib().oracle_kmeans_update(x.ctypes.data, len(x), x.shape[1], idx.ctypes.data, k, es.ctypes.data,
                               out.ctypes.data, counts.ctypes.data)
    return out, counts


def residual_q4(x: np.ndarray, idx: np.ndarray, centers: np.ndarray) -> np.ndarray:
    """4-bit companded residual codes (src/lib.rs:1376) -> [m, dim / 2] bytes."""
    x = np.ascontiguousarray(x, np.float32)
    idx = np.ascontiguousarray(idx, np.uint32)
    c = np.ascontiguousarray(centers, np.float32)
    out = np.empty((len(x), x.shape[1] // 2), np.uint8)
    lib().oracle_residual_q4(x.ctypes.data, len(x), x.shape[1], idx.ctypes.data, c.ctypes.data, out.ctypes.data)
    return out


def q4_table() -> np.ndarray:
    """make_q4_dequant_table (src/packops.rs:14-24)."""
    t = np.empty(16, np.float32)
    lib().oracle_q4_table(t.ctypes.data)
    return t


def score_candidates(q, codes, cluster, cscores, table, raw, group_rows, group_start, doc_start, missing):
    """match_centroids' sub-chunk scores over a prepared candidate set (src/lib.rs:715-808)."""
    q = np.ascontiguousarray(q, np.float32)
    m, dim = q.shape
    codes = np.ascontiguousarray(codes, np.uint8).reshape(-1, dim // 2)
    cluster = np.ascontiguousarray(cluster, np.uint32)
    cscores = np.ascontiguousarray(cscores, np.float32)
    raw = np.ascontiguousarray(raw, np.float32).reshape(-1, dim)
    gr, gs, ds = (np.ascontiguousarray(a, np.int64) for a in (group_rows, group_start, doc_start))
    miss = np.ascontiguousarray(missing, np.float32)
    out = np.empty(len(gs) - 1, np.float32)
    lib().oracle_score_candidates(q.ctypes.data, m, dim, codes.ctypes.data, cluster.ctypes.data, cscores.ctypes.data,
                                  cscores.shape[1] if cscores.ndim == 2 else 1, np.ascontiguousarray(table, np.float32).ctypes.data,
                                  len(codes), raw.ctypes.data, gr.ctypes.data, gs.ctypes.data, ds.ctypes.data,
                                  len(ds) - 1, miss.ctypes.data, out.ctypes.data)
    return out


def similarities(q: np.ndarray, c: np.ndarray) -> np.ndarray:
    """Query-centroid similarities (src/lib.rs:637-640) as fmaf chains."""
    q = np.ascontiguousarray(q, np.float32)
    c = np.ascontiguousarray(c, np.float32)
    out = np.empty((len(q), len(c)), np.float32)
    lib().oracle_similarities(q.ctypes.data, len(q), c.ctypes.data, len(c), q.shape[1], out.ctypes.data)
    return out
