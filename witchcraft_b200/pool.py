"""Multi-GPU bulk encoder: one worker thread and one encoder handle per GPU.

The reference embeds a corpus document by document on one device
(`embed_chunks`, src/lib.rs:1044-1135; the napi `Indexer` loop,
src/napi.rs:353-372).  Documents are independent, so here padded batches
(`shard.plan_batches`) are dealt to the GPUs by longest-processing-time
(`shard.lpt_assign` on padded token counts) and every GPU runs its own
batches: a replica per device, no collective and no peer traffic.

Each worker owns a `wc_t5` handle on its device and a ring of page-locked
output buffers.  It takes its batches `chunk` at a time through
`wc_t5_forward_many` (which overlaps the host copies with the compute) and
hands every result to `sink(batch_index, raw [B, L, 128], norms [B, L])`,
from the worker's thread, before the buffers are reused: a sink that keeps a
result must copy it, and sinks run concurrently on different workers.

Failure handling: the first worker that raises sets a shared stop flag; the
other workers finish the chunk they are in (a `wc_t5_forward_many` call is
not interrupted) and return without starting another; `run` joins every
worker and re-raises the first error with its device.  No worker is left
running and no call hangs on a failed peer, because workers never wait on
each other.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Callable, Sequence

import numpy as np

from .shard import lpt_assign


class WorkerError(RuntimeError):
    def __init__(self, device, err: BaseException):
        super().__init__(f"encoder worker on device {device} failed: {err!r}")
        self.device = device
        self.error = err


@dataclass
class RunStats:
    devices: list                 # device of each worker, in worker order
    batches_per_worker: list
    padded_tokens_per_worker: list


def _pinned_alloc(nbytes: int):
    from .t5cuda import HostBuffer
    return HostBuffer(nbytes)


class _NumpyBuffer:
    """Pageable stand-in for HostBuffer (used by encoders that run on the host)."""

    def __init__(self, nbytes: int):
        self._b = np.empty(nbytes, np.uint8)

    def array(self, shape, dtype=np.float32, offset: int = 0):
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        return self._b[offset:offset + n].view(dtype).reshape(shape)

    def close(self):
        self._b = None


class EncoderPool:
    """Encoders on `devices`, built by `factory(device)` (for the CUDA
    encoder: `lambda d: T5EncoderModel(gguf, config_json, d)`).

    With close_encoders=False the encoders stay open when the pool closes
    (the caller owns them).  `chunk` batches go through one wc_t5_forward_many call; each worker keeps
    `chunk` page-locked output slots of `max_batch_tokens` rows (for 16,384
    tokens and a chunk of 8: 64 MiB of outputs plus norms per GPU)."""

    def __init__(self, factory: Callable, devices: Sequence[int], chunk: int = 8, max_batch_tokens: int = 16384,
                 d_proj: int = 128, pinned: bool = True, close_encoders: bool = True):
        if not devices:
            raise ValueError("no devices")
        self.devices = list(devices)
        self.chunk = max(1, int(chunk))
        self.max_rows = int(max_batch_tokens)
        self.d_proj = d_proj
        self._alloc = _pinned_alloc if pinned else _NumpyBuffer
        self._close_encoders = close_encoders
        self.encoders = []
        self._bufs = []
        try:
            for d in self.devices:
                self.encoders.append(factory(d))
                self._bufs.append([(self._alloc(self.max_rows * d_proj * 4), self._alloc(self.max_rows * 4))
                                   for _ in range(self.chunk)])
        except BaseException:
            self.close()
            raise

    def close(self) -> None:
        for e in self.encoders:
            if self._close_encoders and hasattr(e, "close"):
                e.close()
        for ring in self._bufs:
            for o, n in ring:
                o.close()
                n.close()
        self.encoders, self._bufs = [], []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def run(self, batches: Sequence[tuple], sink: Callable[[int, np.ndarray, np.ndarray], None]) -> RunStats:
        """Encode `batches` [(ids u32 [B, L], lengths i32 [B] or None)] on all
        devices; sink(i, raw, norms) receives batch i's results (views valid
        only during the call)."""
        shapes = []
        for ids, _ in batches:
            B, L = np.shape(ids)
            if B * L > self.max_rows:
                raise ValueError(f"batch of {B} x {L} tokens exceeds max_batch_tokens={self.max_rows}")
            shapes.append((B, L))
        owners = lpt_assign([B * L for B, L in shapes], len(self.devices))
        stop = threading.Event()
        errors: list[WorkerError] = []
        lock = threading.Lock()

        def work(w: int):
            enc, ring = self.encoders[w], self._bufs[w]
            mine = owners[w]
            try:
                for c0 in range(0, len(mine), self.chunk):
                    if stop.is_set():
                        return
                    idx = mine[c0:c0 + self.chunk]
                    outs = [ring[k][0].array((shapes[i][0], shapes[i][1], self.d_proj)) for k, i in enumerate(idx)]
                    norms = [ring[k][1].array(shapes[i]) for k, i in enumerate(idx)]
                    enc.forward_many_into([batches[i] for i in idx], outs, norms)
                    for k, i in enumerate(idx):
                        sink(i, outs[k], norms[k])
            except BaseException as e:  # noqa: BLE001 - reported to the caller
                with lock:
                    errors.append(WorkerError(self.devices[w], e))
                stop.set()

        threads = [threading.Thread(target=work, args=(w,), name=f"wc-encoder-{d}", daemon=True)
                   for w, d in enumerate(self.devices)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return RunStats(list(self.devices), [len(o) for o in owners],
                        [int(sum(shapes[i][0] * shapes[i][1] for i in o)) for o in owners])
