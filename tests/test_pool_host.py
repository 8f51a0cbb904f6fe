"""The multi-GPU bulk encoder pool (witchcraft_b200/pool.py) on the host,
with fake encoders: every batch reaches the sink exactly once with its own
results, batches are dealt by LPT, and a failing worker surfaces as an error
in the caller while the other workers stop without hanging."""
import threading
import time

import numpy as np
import pytest

from witchcraft_b200 import shard
from witchcraft_b200.pool import EncoderPool, WorkerError


class FakeEncoder:
    """Row-deterministic stand-in for T5EncoderModel.forward_many_into:
    raw[b, t, :] = ids[b, t] + arange(128) for t < length, 0 past it."""

    def __init__(self, device, fail_on_call=None, delay=0.0):
        self.device = device
        self.calls = 0
        self.fail_on_call = fail_on_call
        self.delay = delay
        self.closed = False

    def forward_many_into(self, batches, outs, norms=None):
        self.calls += 1
        if self.fail_on_call is not None and self.calls >= self.fail_on_call:
            raise RuntimeError(f"injected failure on device {self.device}")
        time.sleep(self.delay)
        for (ids, lens), o, n in zip(batches, outs, norms):
            B, L = ids.shape
            lens = np.full(B, L) if lens is None else lens
            o[...] = ids[..., None].astype(np.float32) + np.arange(128, dtype=np.float32)
            o[np.arange(L)[None, :] >= np.asarray(lens)[:, None]] = 0
            n[...] = np.linalg.norm(o, axis=-1)

    def close(self):
        self.closed = True


def _batches(seed=0, n_docs=3000):
    lengths = shard.config4_lengths(n_docs, seed=seed)
    rng = np.random.default_rng(seed)
    out = []
    for b in shard.plan_batches(lengths, 4096):
        lens = lengths[b.docs].astype(np.int32)
        ids = rng.integers(3, 32128, (len(lens), b.L)).astype(np.uint32)
        out.append((ids, lens))
    return out


def _expected(ids, lens):
    o = ids[..., None].astype(np.float32) + np.arange(128, dtype=np.float32)
    o[np.arange(ids.shape[1])[None, :] >= lens[:, None]] = 0
    return o


@pytest.mark.parametrize("n_dev,chunk", [(1, 1), (3, 4), (8, 2)])
def test_every_batch_once_with_its_results(n_dev, chunk):
    batches = _batches()
    seen = {}
    lock = threading.Lock()

    def sink(i, raw, norms):
        with lock:
            assert i not in seen
            seen[i] = (raw.copy(), norms.copy(), threading.current_thread().name)

    encs = {}

    def factory(d):
        encs[d] = FakeEncoder(d)
        return encs[d]
    with EncoderPool(factory, list(range(n_dev)), chunk=chunk, max_batch_tokens=4096, pinned=False) as pool:
        stats = pool.run(batches, sink)
    assert sorted(seen) == list(range(len(batches)))
    for i, (ids, lens) in enumerate(batches):
        raw, norms, _ = seen[i]
        np.testing.assert_array_equal(raw, _expected(ids, lens))
        np.testing.assert_allclose(norms, np.linalg.norm(raw, axis=-1), rtol=1e-6)
    # LPT on padded tokens: the same split as shard.lpt_assign
    owners = shard.lpt_assign([ids.size for ids, _ in batches], n_dev)
    assert stats.batches_per_worker == [len(o) for o in owners]
    loads = stats.padded_tokens_per_worker
    assert max(loads) - min(loads) <= max(ids.size for ids, _ in batches)
    assert all(e.closed for e in encs.values())


def test_failing_worker_raises_and_others_stop():
    batches = _batches(1)
    got = []

    def factory(d):
        # device 1 fails on its second chunk; the others are slow enough to
        # still be running when it does
        return FakeEncoder(d, fail_on_call=2 if d == 1 else None, delay=0.01)
    pool = EncoderPool(factory, [0, 1, 2, 3], chunk=1, max_batch_tokens=4096, pinned=False)
    t0 = time.perf_counter()
    with pytest.raises(WorkerError) as ei:
        pool.run(batches, lambda i, r, n: got.append(i))
    assert time.perf_counter() - t0 < 10
    assert ei.value.device == 1 and "injected failure" in str(ei.value)
    # the other workers stopped early instead of encoding their whole share
    assert len(got) < len(batches)
    assert not [t for t in threading.enumerate() if t.name.startswith("wc-encoder-")]
    pool.close()


def test_sink_error_is_reported():
    batches = _batches(2, 500)

    def sink(i, raw, norms):
        raise ValueError("sink refused")
    with EncoderPool(FakeEncoder, [0, 1], pinned=False, max_batch_tokens=4096) as pool:
        with pytest.raises(WorkerError, match="sink refused"):
            pool.run(batches, sink)


def test_factory_failure_closes_built_encoders():
    built = []

    def factory(d):
        if d == 2:
            raise RuntimeError("no device 2")
        built.append(FakeEncoder(d))
        return built[-1]
    with pytest.raises(RuntimeError, match="no device 2"):
        EncoderPool(factory, [0, 1, 2], pinned=False)
    assert len(built) == 2 and all(e.closed for e in built)


def test_oversized_batch_is_refused():
    with EncoderPool(FakeEncoder, [0], pinned=False, max_batch_tokens=1024) as pool:
        with pytest.raises(ValueError, match="max_batch_tokens"):
            pool.run([(np.zeros((4, 512), np.uint32), None)], lambda *a: None)
