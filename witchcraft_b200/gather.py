"""Batched embedding driver: the reference's `Gatherer` / `embed_chunks` loop
(src/lib.rs:901-1003, 1044-1135) feeding many documents per encoder call.

The reference embeds one document per `Embedder::embed` call (batch 1) and
then maps the kept token rows onto the document's sub-chunks.  Here
documents are grouped, their windows packed into length-bucketed padded
batches (`Embedder.embed_ids_batch`), and each document comes out exactly
as the per-document path gives it: the same kept rows (within the encoder
tolerance) and the same sub-chunk counts, in input order.

A document is (hash, token ids, token char offsets, lens) where `lens` is the
reference's comma-separated list of sub-chunk character lengths
(`document.lens`).  No tokenizer is needed when ids and offsets are given.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, Iterator, Sequence

import numpy as np


def chunk_counts(kept_offsets: Sequence[tuple[int, int]], lens: str) -> list[int]:
    """Kept embedding rows per sub-chunk (src/lib.rs:946-992).

    Row i belongs to the sub-chunk whose cumulative character end is the
    first one at or after the row's token end offset; a boundary that no row
    reaches closes a sub-chunk with 0 rows, and rows past the last boundary
    form one trailing group.  The counts sum to the number of kept rows.
    """
    lengths = [int(s) for s in lens.split(",") if _is_uint(s)]
    for i in range(1, len(lengths)):
        lengths[i] += lengths[i - 1]
    big = 1 << 64
    i = j = 0
    i_end, j_end = len(kept_offsets), len(lengths)
    if i_end == 0 and j_end == 0:
        # the reference loop never terminates here; its Embedder has already
        # failed ("all token embeddings below minimum norm threshold")
        raise ValueError("no kept rows and no sub-chunk lengths")
    count = 0
    counts: list[int] = []
    done = False
    while not done:
        o = kept_offsets[i][1] if i < i_end else big
        ln = lengths[j] if j < j_end else big
        flush = False
        if o <= ln:
            i += 1
            count += 1
        else:
            j += 1
            flush = True
        done = i == i_end and j == j_end
        if flush or done:
            counts.append(count)
            count = 0
    assert sum(counts) == i_end
    return counts


def _is_uint(s: str) -> bool:
    """`s.parse::<usize>().ok()` is Some: ASCII digits, optional leading '+'."""
    t = s[1:] if s.startswith("+") else s
    return len(t) > 0 and t.isascii() and t.isdigit()


@dataclass
class Document:
    hash: str
    ids: np.ndarray                    # u32 token ids (with the trailing </s>)
    offsets: list[tuple[int, int]]     # char (start, end) per token
    lens: str                          # comma-separated sub-chunk char lengths


class Gatherer:
    """Iterator of (hash, embeddings [kept, 128] f32, counts) per document,
    in input order; documents are embedded `group_docs` at a time through
    length-bucketed batches of at most `max_batch_tokens` padded tokens."""

    def __init__(self, documents: Iterable[Document], embedder, group_docs: int = 256,
                 max_batch_tokens: int = 16384):
        self._docs = iter(documents)
        self._embedder = embedder
        self._group = max(1, group_docs)
        self._max_tokens = max_batch_tokens
        self._ready: list[tuple[str, np.ndarray, list[int]]] = []

    def __iter__(self) -> Iterator[tuple[str, np.ndarray, list[int]]]:
        return self

    def next_group(self) -> list[tuple[str, np.ndarray, list[int]]]:
        """The next up to `group_docs` documents' results, in input order
        (empty at the end)."""
        group = []
        for d in self._docs:
            group.append(d)
            if len(group) == self._group:
                break
        if not group:
            return []
        results = self._embedder.embed_ids_batch([d.ids for d in group], [d.offsets for d in group],
                                                 max_batch_tokens=self._max_tokens)
        return [(d.hash, emb[0], chunk_counts(kept, d.lens)) for d, (emb, kept) in zip(group, results)]

    def __next__(self) -> tuple[str, np.ndarray, list[int]]:
        if not self._ready:
            self._ready = self.next_group()
            if not self._ready:
                raise StopIteration
            self._ready.reverse()
        return self._ready.pop()


def embed_chunks(documents: Iterable[Document], embedder, pack=None, pack_many=None, **kw):
    """The reference's embed_chunks loop without the database: yields
    (hash, payload, counts string) per document, in input order.  The payload
    is `add_chunk`'s blob: with pack_many (e.g. `codec.pack_many`, one
    wc_pack_embeddings call per document group) or pack (one document at a
    time) the packed codec bytes, otherwise the f32 rows."""
    g = Gatherer(documents, embedder, **kw)
    while True:
        group = g.next_group()
        if not group:
            return
        if pack_many is not None:
            payloads = pack_many([emb for _, emb, _ in group])
        else:
            payloads = [pack(emb) if pack is not None else emb for _, emb, _ in group]
        for (h, _, counts), p in zip(group, payloads):
            yield h, p, ",".join(str(c) for c in counts)
