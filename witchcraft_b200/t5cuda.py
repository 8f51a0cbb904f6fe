"""Python mirror of the reference's encoder backend and Embedder, over the
native library (no CPU fallback: every forward runs the sm_100a kernels).

  T5ModelBuilder.load / build_encoder    src/quantized_t5.rs:708-749
  T5EncoderModel.forward / device        src/quantized_t5.rs:698-705
  Embedder.embed                         src/embedder.rs:22-102

`Embedder.embed_ids_batch` is this backend's addition: it packs the windows of
many documents into length-bucketed padded batches (one forward per batch
instead of one per window) and returns, per document, exactly what
`embed_ids` returns for it alone.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

from ._lib import WC_OK, WcError, check, lib

MAX_LEN = 2048      # window (src/embedder.rs:27)
STRIDE = 256        # overlap (src/embedder.rs:28)
MIN_NORM = 1.0      # src/embedder.rs:79
EMBEDDING_DIM = 128  # src/lib.rs:70


def _ptr(a: np.ndarray | None):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


class T5EncoderModel:
    """One encoder on one GPU (a `wc_t5` handle)."""

    def __init__(self, gguf: bytes, config_json: str, device: int = 0):
        h = ctypes.c_void_p()
        self._gguf = gguf  # kept alive only for the duration of create
        rc = lib().wc_t5_create(int(device), gguf, len(gguf), config_json.encode(), ctypes.byref(h))
        if rc != WC_OK:
            raise WcError(rc, lib().wc_t5_last_error(None).decode())
        self._h = h
        self._device = int(device)
        d = [ctypes.c_int() for _ in range(4)]
        check(lib().wc_t5_dims(h, *[ctypes.byref(x) for x in d]), h)
        self.d_model, self.n_layers, self.d_proj, self.vocab = (x.value for x in d)
        self._gguf = None

    @property
    def handle(self):
        return self._h

    def device(self) -> int:
        return self._device

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().wc_t5_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward_full(self, ids: np.ndarray, lengths=None):
        """ids u32 [B, L] (or [L]) -> (raw [B, L, 128], norms [B, L], normalised [B, L, 128])."""
        ids = np.ascontiguousarray(np.atleast_2d(ids), dtype=np.uint32)
        B, L = ids.shape
        lens = None if lengths is None else np.ascontiguousarray(lengths, dtype=np.int32)
        out = np.empty((B, L, self.d_proj), np.float32)
        norms = np.empty((B, L), np.float32)
        outn = np.empty((B, L, self.d_proj), np.float32)
        check(lib().wc_t5_forward(self._h, _ptr(ids), _ptr(lens), B, L, _ptr(out), _ptr(norms), _ptr(outn)),
              self._h)
        return out, norms, outn

    def forward(self, ids: np.ndarray, lengths=None) -> np.ndarray:
        """T5EncoderModel::forward: ids [1, L] -> raw projection f32 [1, L, 128]."""
        ids = np.ascontiguousarray(np.atleast_2d(ids), dtype=np.uint32)
        B, L = ids.shape
        lens = None if lengths is None else np.ascontiguousarray(lengths, dtype=np.int32)
        out = np.empty((B, L, self.d_proj), np.float32)
        check(lib().wc_t5_forward(self._h, _ptr(ids), _ptr(lens), B, L, _ptr(out), None, None), self._h)
        return out

    def forward_many(self, batches, with_norms: bool = False):
        """[(ids [B, L] u32, lengths [B] or None)] -> [raw [B, L, 128]] (and norms),
        pipelined through wc_t5_forward_many (copies overlap the compute when
        the arrays are page-locked)."""
        ids = [np.ascontiguousarray(np.atleast_2d(b[0]), dtype=np.uint32) for b in batches]
        outs = [np.empty((a.shape[0], a.shape[1], self.d_proj), np.float32) for a in ids]
        norms = [np.empty(a.shape, np.float32) for a in ids] if with_norms else None
        self.forward_many_into(batches, outs, norms)
        return (outs, norms) if with_norms else outs

    def forward_many_into(self, batches, outs, norms=None) -> None:
        """forward_many writing into caller-owned arrays: outs[i] f32 [B, L, 128]
        (C-contiguous, e.g. views of page-locked buffers), norms[i] f32 [B, L] or
        norms None."""
        n = len(batches)
        ids = [np.ascontiguousarray(np.atleast_2d(b[0]), dtype=np.uint32) for b in batches]
        lens = [None if b[1] is None else np.ascontiguousarray(b[1], dtype=np.int32) for b in batches]
        for a, o in zip(ids, outs):
            if o.dtype != np.float32 or not o.flags["C_CONTIGUOUS"] or o.size < a.size * self.d_proj:
                raise ValueError("output array must be C-contiguous f32 with B * L * 128 elements")
        vp = ctypes.c_void_p
        arr = lambda xs: (vp * n)(*[vp(x.ctypes.data) if x is not None else None for x in xs])  # noqa: E731
        Bs = (ctypes.c_int * n)(*[a.shape[0] for a in ids])
        Ls = (ctypes.c_int * n)(*[a.shape[1] for a in ids])
        check(lib().wc_t5_forward_many(self._h, n, arr(ids), arr(lens), Bs, Ls, arr(outs),
                                       arr(norms) if norms is not None else None), self._h)

    def forward_device(self, d_ids: int, d_lengths: int, B: int, L: int, d_out: int, d_norms: int | None = None,
                       d_outn: int | None = None, stream: int | None = None) -> None:
        """Enqueue a forward on device buffers (raw pointers) on `stream`."""
        check(lib().wc_t5_forward_device(self._h, ctypes.c_void_p(d_ids), ctypes.c_void_p(d_lengths), B, L,
                                         ctypes.c_void_p(d_out), ctypes.c_void_p(d_norms) if d_norms else None,
                                         ctypes.c_void_p(d_outn) if d_outn else None,
                                         ctypes.c_void_p(stream) if stream else None), self._h)

    def forward_many_device(self, batches, stream: int | None = None) -> None:
        """Enqueue device-resident batches [(d_ids, d_lengths, B, L, d_out, d_norms or None)]
        (raw device pointers) in one call on `stream` (wc_t5_forward_many_device)."""
        n = len(batches)
        vp = ctypes.c_void_p
        col = lambda k: (vp * n)(*[vp(b[k]) if b[k] else None for b in batches])  # noqa: E731
        Bs = (ctypes.c_int * n)(*[b[2] for b in batches])
        Ls = (ctypes.c_int * n)(*[b[3] for b in batches])
        norms = col(5) if any(b[5] for b in batches) else None
        check(lib().wc_t5_forward_many_device(self._h, n, col(0), col(1), Bs, Ls, col(4), norms,
                                              vp(stream) if stream else None), self._h)

    def sync(self, stream: int | None = None) -> None:
        check(lib().wc_t5_sync(self._h, ctypes.c_void_p(stream) if stream else None), self._h)


class HostBuffer:
    """Page-locked host memory from the library (wc_host_alloc), viewed as a
    numpy array; freed by close() or when collected."""

    def __init__(self, nbytes: int):
        self._p = lib().wc_host_alloc(int(nbytes))
        if not self._p:
            raise MemoryError(f"wc_host_alloc({nbytes}) failed")
        self.nbytes = int(nbytes)

    def array(self, shape, dtype=np.float32, offset: int = 0) -> np.ndarray:
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        if offset + n > self.nbytes:
            raise ValueError("view past the end of the buffer")
        raw = (ctypes.c_char * n).from_address(self._p + offset)
        return np.frombuffer(raw, dtype=dtype).reshape(shape)

    def close(self) -> None:
        if getattr(self, "_p", None):
            lib().wc_host_free(self._p)
            self._p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class T5ModelBuilder:
    """Reads config.json (and tokenizer.json when the `tokenizers` package is
    present) from an assets directory, like src/quantized_t5.rs:713-729."""

    def __init__(self, config_json: str):
        self.config_json = config_json

    @classmethod
    def load(cls, assets: str):
        path = os.path.join(assets, "config.json")
        if not os.path.exists(path):
            raise FileNotFoundError("failed to get bytes for CONFIG")
        builder = cls(open(path).read())
        tok = None
        tpath = os.path.join(assets, "tokenizer.json")
        if os.path.exists(tpath):
            try:
                from tokenizers import Tokenizer
                tok = Tokenizer.from_file(tpath)
            except ImportError:
                tok = None
        return builder, tok

    def build_encoder(self, device: int, assets: str) -> T5EncoderModel:
        path = os.path.join(assets, "xtr.gguf")
        if not os.path.exists(path):
            raise FileNotFoundError("failed to get bytes for MODEL")
        return T5EncoderModel(open(path, "rb").read(), self.config_json, device)


@dataclass
class _Window:
    doc: int
    start: int
    ids: np.ndarray


def _windows(n_tokens: int):
    """(start, end) windows of src/embedder.rs:37-63."""
    start = 0
    while True:
        end = min(start + MAX_LEN, n_tokens)
        yield start, end
        if end == n_tokens:
            break
        start = max(end - STRIDE, 0)


def _finish(accum: np.ndarray, offsets):
    """Min-norm filter and L2 normalisation (src/embedder.rs:75-94)."""
    norms = np.sqrt((accum * accum).sum(axis=1))
    keep = norms >= MIN_NORM
    if not keep.any():
        raise ValueError("all token embeddings below minimum norm threshold")
    kept = accum[keep]
    normalized = kept / np.sqrt((kept * kept).sum(axis=1, keepdims=True))
    kept_offsets = [o for o, k in zip(offsets, keep) if k] if offsets is not None else list(np.nonzero(keep)[0])
    return normalized[None].astype(np.float32), kept_offsets


class Embedder:
    """src/embedder.rs:10-102 over the CUDA encoder."""

    def __init__(self, model: T5EncoderModel, tokenizer=None):
        self.model = model
        self.tokenizer = tokenizer

    @classmethod
    def new(cls, device: int, assets: str) -> "Embedder":
        builder, tok = T5ModelBuilder.load(assets)
        return cls(builder.build_encoder(device, assets), tok)

    def embed(self, text: str):
        if self.tokenizer is None:
            raise RuntimeError("no tokenizer.json loaded")
        enc = self.tokenizer.encode(text, add_special_tokens=True)
        return self.embed_ids(np.asarray(enc.ids, np.uint32), list(enc.offsets))

    def embed_ids(self, ids: np.ndarray, offsets=None):
        """Token ids of one document -> ([1, kept, 128] normalised, kept offsets)."""
        ids = np.asarray(ids, np.uint32)
        n = len(ids)
        accum = np.zeros((n, self.model.d_proj), np.float32)
        for start, end in _windows(n):
            chunk = self.model.forward(ids[start:end][None])[0]
            accum[start:end] += chunk
        return _finish(accum, offsets)

    def embed_ids_batch(self, docs: list[np.ndarray], offsets=None, max_batch_tokens: int = 16384):
        """Many documents at once: windows sorted by length and packed into
        padded batches of at most max_batch_tokens (B * L) tokens."""
        wins: list[_Window] = []
        accums = []
        for d, ids in enumerate(docs):
            ids = np.asarray(ids, np.uint32)
            accums.append(np.zeros((len(ids), self.model.d_proj), np.float32))
            for start, end in _windows(len(ids)):
                wins.append(_Window(d, start, ids[start:end]))
        wins.sort(key=lambda w: len(w.ids))
        plan = []  # (windows, padded ids, lengths) per batch
        i = 0
        while i < len(wins):
            L = len(wins[i].ids)
            j = i
            # grow the batch while the padded size (count x longest) fits
            while j < len(wins) and (j - i + 1) * len(wins[j].ids) <= max(max_batch_tokens, len(wins[j].ids)):
                L = len(wins[j].ids)
                j += 1
            batch = wins[i:j]
            ids = np.zeros((len(batch), L), np.uint32)
            lens = np.empty(len(batch), np.int32)
            for b, w in enumerate(batch):
                ids[b, :len(w.ids)] = w.ids
                lens[b] = len(w.ids)
            plan.append((batch, ids, lens))
            i = j
        if hasattr(self.model, "forward_many"):
            # one pipelined call for all batches (copies overlap the compute)
            outs = self.model.forward_many([(ids, lens) for _, ids, lens in plan])
        else:
            outs = [self.model.forward(ids, lens) for _, ids, lens in plan]
        for (batch, _, _), out in zip(plan, outs):
            for b, w in enumerate(batch):
                accums[w.doc][w.start:w.start + len(w.ids)] += out[b, :len(w.ids)]
        return [_finish(a, None if offsets is None else offsets[d]) for d, a in enumerate(accums)]
