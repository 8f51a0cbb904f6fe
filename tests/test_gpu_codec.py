"""CUDA packed-embedding codec (csrc/codec.cu) against the CPU oracle
(src/packops.rs:172-438): the packed bytes of every document identical, the
decoded rows bit-identical."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from witchcraft_b200._lib import lib

pytestmark = pytest.mark.gpu


def _docs(lengths, cols=128, seed=0, scale=None):
    rng = np.random.default_rng(seed)
    out = []
    for n in lengths:
        e = rng.standard_normal((n, cols)).astype(np.float32)
        if scale is not None:  # a shared direction, like real embeddings
            e += scale * rng.standard_normal(cols).astype(np.float32)
        out.append(e / np.linalg.norm(e, axis=1, keepdims=True))
    return out


def _pack_gpu(docs, cols=128):
    rows = np.concatenate([[0], np.cumsum([len(d) for d in docs])]).astype(np.int64)
    emb = np.ascontiguousarray(np.concatenate(docs), np.float32)
    cap = lib().wc_packed_bound(rows.ctypes.data, len(docs), cols)
    out = np.empty(cap, np.uint8)
    offs = np.empty(len(docs) + 1, np.int64)
    rc = lib().wc_pack_embeddings(emb.ctypes.data, rows.ctypes.data, len(docs), cols, out.ctypes.data, cap,
                                  offs.ctypes.data, 0)
    assert rc == 0, lib().wc_codec_last_error()
    return [out[offs[i]:offs[i + 1]].tobytes() for i in range(len(docs))]


def _unpack_gpu(bufs, cols=128):
    offs = np.concatenate([[0], np.cumsum([len(b) for b in bufs])]).astype(np.int64)
    inp = np.frombuffer(b"".join(bufs), np.uint8).copy()
    total_rows = sum(int(np.frombuffer(b[:4], np.uint32)[0]) for b in bufs)
    out = np.empty((max(total_rows, 1), cols), np.float32)
    rows = np.empty(len(bufs) + 1, np.int64)
    rc = lib().wc_unpack_embeddings(inp.ctypes.data, offs.ctypes.data, len(bufs), cols, out.ctypes.data, total_rows,
                                    rows.ctypes.data, 0)
    return rc, out[:total_rows], rows


@pytest.mark.parametrize("lengths", [[1], [2, 3, 31], [1024, 1025, 7], [2100, 180, 64, 1023], list(range(1, 40))])
def test_packed_bytes_identical_to_oracle(lengths):
    docs = _docs(lengths, seed=len(lengths))
    got = _pack_gpu(docs)
    for d, g in zip(docs, got):
        assert g == O.pack_embeddings(d)


def test_packed_bytes_with_a_shared_direction():
    docs = _docs([300, 900, 40], seed=9, scale=0.8)
    for d, g in zip(docs, _pack_gpu(docs)):
        assert g == O.pack_embeddings(d)


@pytest.mark.parametrize("cols", [1, 7, 128, 255])
def test_other_widths(cols):
    docs = _docs([5, 130], cols=cols, seed=cols)
    for d, g in zip(docs, _pack_gpu(docs, cols)):
        assert g == O.pack_embeddings(d)


def test_unpack_bit_identical_to_oracle():
    docs = _docs([1, 17, 1024, 1500, 333], seed=4)
    bufs = [O.pack_embeddings(d) for d in docs]
    rc, out, rows = _unpack_gpu(bufs)
    assert rc == 0, lib().wc_codec_last_error()
    for i, b in enumerate(bufs):
        ref = O.unpack_embeddings(b)
        got = out[rows[i]:rows[i + 1]]
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_unpack_rejects_malformed_input():
    b = O.pack_embeddings(_docs([50])[0])
    rc, _, _ = _unpack_gpu([b[:-1]])
    assert rc != 0
    rc, _, _ = _unpack_gpu([b + b"\x00"])
    assert rc != 0


def test_device_entry_and_empty_call():
    docs = _docs([10, 20], seed=1)
    rows = np.array([0, 10, 30], np.int64)
    d_emb = torch.from_numpy(np.concatenate(docs)).cuda()
    cap = lib().wc_packed_bound(rows.ctypes.data, 2, 128)
    d_out = torch.empty(cap, dtype=torch.uint8, device="cuda")
    offs = np.empty(3, np.int64)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib().wc_pack_embeddings_device(ctypes.c_void_p(d_emb.data_ptr()), rows.ctypes.data, 2, 128,
                                           ctypes.c_void_p(d_out.data_ptr()), cap, offs.ctypes.data, st) == 0
    host = d_out.cpu().numpy()
    for i, d in enumerate(docs):
        assert host[offs[i]:offs[i + 1]].tobytes() == O.pack_embeddings(d)
    z = np.zeros(1, np.int64)
    assert lib().wc_pack_embeddings(None, z.ctypes.data, 0, 128, None, 0, z.ctypes.data, 0) == 0
