"""The bulk encoder pool on real handles: every batch equals its
wc_t5_forward_many result.  With one GPU the pool runs two workers (two
handles) on device 0; with more it runs one worker per device."""
import threading

import numpy as np
import pytest

from witchcraft_b200 import shard
from witchcraft_b200._lib import lib
from witchcraft_b200.pool import EncoderPool
from witchcraft_b200.t5cuda import T5EncoderModel

pytestmark = pytest.mark.gpu


def test_pool_matches_forward_many(tiny_model):
    n = lib().wc_t5_device_count()
    devices = list(range(min(n, 4))) if n > 1 else [0, 0]
    lengths = shard.config4_lengths(600, seed=3)
    rng = np.random.default_rng(3)
    batches = []
    for b in shard.plan_batches(lengths, 8192):
        lens = lengths[b.docs].astype(np.int32)
        batches.append((rng.integers(3, 512, (len(lens), b.L)).astype(np.uint32), lens))
    cfg = tiny_model.config.to_json()
    got = {}
    lock = threading.Lock()

    def sink(i, raw, norms):
        with lock:
            got[i] = (raw.copy(), norms.copy())
    with EncoderPool(lambda d: T5EncoderModel(tiny_model.gguf, cfg, d), devices, chunk=3,
                     max_batch_tokens=8192) as pool:
        pool.run(batches, sink)
    ref = T5EncoderModel(tiny_model.gguf, cfg, 0)
    try:
        outs, norms = ref.forward_many(batches, with_norms=True)
    finally:
        ref.close()
    assert sorted(got) == list(range(len(batches)))
    for i in range(len(batches)):
        np.testing.assert_array_equal(got[i][0], outs[i])
        np.testing.assert_array_equal(got[i][1], norms[i])
