"""Host front end of the packed-embedding codec (include/wc_codec.h): the
reference's `embeddings_to_packed` / `embeddings_from_packed`
(src/packops.rs:172-438) for many documents in one GPU call."""
from __future__ import annotations

import numpy as np

from ._lib import WcError, lib


def _check(rc: int) -> None:
    if rc != 0:
        msg = lib().wc_codec_last_error()
        raise WcError(rc, msg.decode() if msg else "")


def pack_many(docs, device: int = 0) -> list[bytes]:
    """[f32 [rows_i, cols] L2-normalised, rows_i >= 1] -> the packed bytes of
    each document (byte-identical to the reference's stream), one
    wc_pack_embeddings call for all of them."""
    if not docs:
        return []
    cols = docs[0].shape[1]
    rows = np.concatenate([[0], np.cumsum([len(d) for d in docs])]).astype(np.int64)
    emb = np.ascontiguousarray(np.concatenate(docs), np.float32)
    cap = lib().wc_packed_bound(rows.ctypes.data, len(docs), cols)
    if cap < 0:
        raise WcError(-1, "invalid document row counts")
    out = np.empty(cap, np.uint8)
    offs = np.empty(len(docs) + 1, np.int64)
    _check(lib().wc_pack_embeddings(emb.ctypes.data, rows.ctypes.data, len(docs), cols, out.ctypes.data, cap,
                                    offs.ctypes.data, device))
    return [out[offs[i]:offs[i + 1]].tobytes() for i in range(len(docs))]


def unpack_many(bufs, cols: int = 128, device: int = 0) -> list[np.ndarray]:
    """Packed bytes per document -> L2-normalised rows [rows_i, cols] each."""
    if not bufs:
        return []
    offs = np.concatenate([[0], np.cumsum([len(b) for b in bufs])]).astype(np.int64)
    inp = np.frombuffer(b"".join(bufs), np.uint8).copy()
    total = sum(int(np.frombuffer(b[:4], np.uint32)[0]) if len(b) >= 4 else 0 for b in bufs)
    out = np.empty((max(total, 1), cols), np.float32)
    rows = np.empty(len(bufs) + 1, np.int64)
    _check(lib().wc_unpack_embeddings(inp.ctypes.data, offs.ctypes.data, len(bufs), cols, out.ctypes.data, total,
                                      rows.ctypes.data, device))
    return [out[rows[i]:rows[i + 1]].copy() for i in range(len(bufs))]
