"""The no-allocation forward entry point against the regular one.

wc_t5_forward_device_noalloc exists for callers that cannot allocate GPU
memory while they run (a latency-critical query path that must not pay for
cudaMalloc's implicit device synchronisation, or a host application that
reserves all device memory up front).  It keeps its activations in one fixed
8 MiB device array instead of the handle's workspace and runs the same
kernels on the same shapes, so its results must be bitwise identical to
wc_t5_forward_device's.  This test calls it twice in a row, on different
inputs, and compares each result bit for bit against wc_t5_forward_device on
the same inputs; one case is also checked against the CPU oracle within the
encoder tolerance (cosine >= 0.999, max-abs <= 2e-2 per token).  The largest
batch that fits the array must run and match; one token more must be refused
with a clear error.  The file name makes pytest collect it last."""
import ctypes
import re

import numpy as np
import pytest
import torch

from oracle import oracle as O
from witchcraft_b200._lib import check, lib
from witchcraft_b200.t5cuda import T5EncoderModel

from gpu_util import cosine_rows

pytestmark = pytest.mark.gpu

P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731


def _run(fn, enc, ids, lens):
    B, L = ids.shape
    d_ids = torch.from_numpy(ids).cuda()
    d_len = torch.from_numpy(lens).cuda()
    out = torch.full((B * L, 128), float("nan"), device="cuda")
    norms = torch.full((B * L,), float("nan"), device="cuda")
    outn = torch.full((B * L, 128), float("nan"), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    check(fn(enc.handle, P(d_ids), P(d_len), B, L, P(out), P(norms), P(outn), ctypes.c_void_p(st)), enc.handle)
    enc.sync(st)
    return (out.view(B, L, 128).cpu().numpy(), norms.view(B, L).cpu().numpy(),
            outn.view(B, L, 128).cpu().numpy())


def _inputs(seed, B, L):
    rng = np.random.default_rng(seed)
    ids = rng.integers(3, 32128, (B, L)).astype(np.uint32)
    lens = rng.integers(1, L + 1, B).astype(np.int32)
    lens[0] = L
    return ids, lens


def _same_bits(got, ref):
    for g, r in zip(got, ref):
        np.testing.assert_array_equal(g.view(np.uint32), r.view(np.uint32))


@pytest.fixture(scope="module")
def enc(xtr_model):
    e = T5EncoderModel(xtr_model.gguf, xtr_model.config.to_json(), 0)
    yield e
    e.close()


def _limit(enc):
    """Largest B*L the array takes, read from the refusal message of a batch
    that is certainly too large."""
    ids = torch.zeros(1, 2048, dtype=torch.int32, device="cuda")
    lens = torch.full((1,), 2048, dtype=torch.int32, device="cuda")
    out = torch.empty(2048, 128, device="cuda")
    rc = lib().wc_t5_forward_device_noalloc(enc.handle, P(ids), P(lens), 1, 2048, P(out), None, None, None)
    assert rc == -1
    msg = lib().wc_t5_last_error(enc.handle).decode()
    m = re.search(r"at most (\d+) tokens per call", msg)
    assert m, msg
    return int(m.group(1))


def test_noalloc_bitwise_equal_to_regular_forward_twice(enc):
    for seed, (B, L) in ((1, (16, 32)), (2, (3, 150))):
        ids, lens = _inputs(seed, B, L)
        ref = _run(lib().wc_t5_forward_device, enc, ids, lens)
        got = _run(lib().wc_t5_forward_device_noalloc, enc, ids, lens)
        _same_bits(got, ref)
        for b in range(B):
            assert np.all(got[0][b, lens[b]:] == 0) and np.all(got[1][b, lens[b]:] == 0)


def test_noalloc_matches_oracle(enc, xtr_model):
    ids, lens = _inputs(3, 4, 96)
    got = _run(lib().wc_t5_forward_device_noalloc, enc, ids, lens)[0]
    ref = O.OracleEncoder(xtr_model).encode(ids, lens)
    for b, n in enumerate(lens):
        g, r = got[b, :n], ref[b, :n]
        assert cosine_rows(g, r).min() >= 0.999
        gn = g / np.linalg.norm(g, axis=1, keepdims=True)
        rn = r / np.linalg.norm(r, axis=1, keepdims=True)
        assert np.abs(gn - rn).max() <= 2e-2


def test_noalloc_at_its_limit_and_one_past(enc):
    n = _limit(enc)
    assert 256 <= n <= 2048
    ids, lens = _inputs(4, 1, n)
    _same_bits(_run(lib().wc_t5_forward_device_noalloc, enc, ids, lens),
               _run(lib().wc_t5_forward_device, enc, ids, lens))
    d_ids = torch.zeros(1, n + 1, dtype=torch.int32, device="cuda")
    d_len = torch.full((1,), n + 1, dtype=torch.int32, device="cuda")
    out = torch.empty(n + 1, 128, device="cuda")
    rc = lib().wc_t5_forward_device_noalloc(enc.handle, P(d_ids), P(d_len), 1, n + 1, P(out), None, None, None)
    assert rc == -1
    msg = lib().wc_t5_last_error(enc.handle).decode()
    assert "at most" in msg and "tokens per call" in msg
