"""The batched embedding driver end to end on the GPU: `embed_chunks` over
config-4-length documents with the CUDA encoder (windows packed into
length-bucketed batches, one wc_t5_forward_many call per document group) and
the GPU codec (one wc_pack_embeddings call per group), against the same
driver over the CPU oracle encoder.  The per-document sub-chunk counts
strings must be identical, and the decoded payload rows must match the
oracle's rows (the codec is lossy: cosine >= 0.99 per row, as its round-trip
tests use)."""
import numpy as np
import pytest

from oracle import oracle as O
from witchcraft_b200 import codec, shard
from witchcraft_b200.gather import Document, embed_chunks
from witchcraft_b200.t5cuda import Embedder, T5EncoderModel

from gpu_util import cosine_rows

pytestmark = pytest.mark.gpu


def _documents(n, seed):
    rng = np.random.default_rng(seed)
    lengths = shard.config4_lengths(n, seed=seed)
    docs = []
    for i, nt in enumerate(lengths):
        ids = rng.integers(3, 32128, int(nt)).astype(np.uint32)
        widths = rng.integers(1, 9, int(nt))
        ends = np.cumsum(widths)
        offsets = [(int(e - w), int(e)) for e, w in zip(ends, widths)]
        total = int(ends[-1])
        cuts = np.sort(rng.choice(np.arange(1, total), size=min(3, total - 1), replace=False))
        parts = np.diff(np.concatenate([[0], cuts, [total]]))
        docs.append(Document(f"doc{i}", ids, offsets, ",".join(str(int(p)) for p in parts)))
    return docs


class _OracleModel:
    d_proj = 128

    def __init__(self, model):
        self.enc = O.OracleEncoder(model)

    def forward(self, ids, lengths=None):
        ids = np.atleast_2d(ids)
        out = np.zeros((ids.shape[0], ids.shape[1], 128), np.float32)
        for b in range(ids.shape[0]):
            n = ids.shape[1] if lengths is None else int(lengths[b])
            out[b, :n] = self.enc.encode(ids[b:b + 1, :n])[0]
        return out


def test_embed_chunks_gpu_matches_oracle_driver(xtr_model):
    docs = _documents(40, seed=12)
    enc = T5EncoderModel(xtr_model.gguf, xtr_model.config.to_json(), 0)
    try:
        got = list(embed_chunks(docs, Embedder(enc), pack_many=codec.pack_many, group_docs=16))
    finally:
        enc.close()
    ref = list(embed_chunks(docs, Embedder(_OracleModel(xtr_model)), group_docs=16))
    assert [g[0] for g in got] == [d.hash for d in docs]
    rows = codec.unpack_many([g[1] for g in got])
    for (h, payload, counts), (rh, remb, rcounts), dec in zip(got, ref, rows):
        assert h == rh
        assert counts == rcounts
        assert dec.shape == remb.shape
        assert cosine_rows(dec, remb).min() >= 0.99
