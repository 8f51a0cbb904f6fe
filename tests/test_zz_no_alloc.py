"""The no-allocation forward entry point against the regular one.

wc_t5_forward_device_noalloc exists for callers that cannot allocate GPU
memory while they run (a latency-critical query path that must not pay for
cudaMalloc's implicit device synchronisation, or a host application that
reserves all device memory up front).  It keeps its activations in one fixed
8 MiB device array instead of the handle's workspace.  This test calls it
twice in a row, on different inputs, and checks each result against
wc_t5_forward_device on the same inputs; it also checks that a batch too
large for the array is refused with a clear error.  The file name makes
pytest collect it last."""
import ctypes

import numpy as np
import pytest
import torch

from witchcraft_b200._lib import check, lib
from witchcraft_b200.t5cuda import T5EncoderModel

from gpu_util import cosine_rows

pytestmark = pytest.mark.gpu


def _run(fn, enc, ids, lens):
    B, L = ids.shape
    d_ids = torch.from_numpy(ids).cuda()
    d_len = torch.from_numpy(lens).cuda()
    out = torch.full((B * L, 128), float("nan"), device="cuda")
    norms = torch.full((B * L,), float("nan"), device="cuda")
    outn = torch.full((B * L, 128), float("nan"), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
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


def test_noalloc_matches_regular_forward_twice(xtr_model):
    enc = T5EncoderModel(xtr_model.gguf, xtr_model.config.to_json(), 0)
    try:
        for seed, (B, L) in ((1, (16, 32)), (2, (3, 150))):
            ids, lens = _inputs(seed, B, L)
            ref = _run(lib().wc_t5_forward_device, enc, ids, lens)
            got = _run(lib().wc_t5_forward_device_noalloc, enc, ids, lens)
            for b in range(B):
                n = lens[b]
                assert cosine_rows(got[0][b, :n], ref[0][b, :n]).min() >= 0.999
                assert np.abs(got[2][b, :n] - ref[2][b, :n]).max() <= 2e-2
                np.testing.assert_allclose(got[1][b, :n], ref[1][b, :n], rtol=1e-4)
                assert np.all(got[0][b, n:] == 0) and np.all(got[1][b, n:] == 0)
    finally:
        enc.close()


def test_noalloc_rejects_batches_beyond_its_scratch(xtr_model):
    enc = T5EncoderModel(xtr_model.gguf, xtr_model.config.to_json(), 0)
    try:
        ids = np.zeros((8, 128), np.uint32)
        lens = np.full(8, 128, np.int32)
        d_ids = torch.from_numpy(ids).cuda()
        d_len = torch.from_numpy(lens).cuda()
        out = torch.empty(8 * 128, 128, device="cuda")
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        rc = lib().wc_t5_forward_device_noalloc(enc.handle, P(d_ids), P(d_len), 8, 128, P(out), None, None, None)
        assert rc == -1
        msg = lib().wc_t5_last_error(enc.handle).decode()
        assert "at most" in msg and "tokens per call" in msg
    finally:
        enc.close()
