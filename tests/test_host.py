"""Host-side checks of the native library that need no GPU: it loads, it
exports every function include/wc_t5cuda.h declares, the relative-position
bucket function equals the oracle, and wc_t5_create rejects bad inputs with
the documented error codes (config, GGUF, shape/dtype, no device)."""
import ctypes
import json
import os
import struct
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT
from oracle import oracle as O
from witchcraft_b200 import _lib
from witchcraft_b200.synth import GGML_TYPE_F32, write_gguf


def _create(lib, gguf: bytes, cfg: str):
    h = ctypes.c_void_p()
    rc = lib.wc_t5_create(0, gguf, len(gguf), cfg.encode() if cfg is not None else None, ctypes.byref(h))
    return rc, h, lib.wc_t5_last_error(None).decode()


def test_library_exports_every_header_symbol(cuda_lib):
    syms = _lib.header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(cuda_lib, s), s


def test_device_count_never_fails(cuda_lib):
    assert cuda_lib.wc_t5_device_count() >= 0


def test_relative_bucket_matches_oracle(cuda_lib):
    for d in range(-2047, 2048):
        q, k = (0, d) if d >= 0 else (-d, 0)
        assert cuda_lib.wc_t5_relative_bucket(q, k, 32, 128) == O.bucket(q, k, 32, 128), d
    # other bucket geometries
    for nb, md in ((16, 64), (64, 256), (8, 20)):
        for d in range(-300, 301, 7):
            q, k = (0, d) if d >= 0 else (-d, 0)
            assert cuda_lib.wc_t5_relative_bucket(q, k, nb, md) == O.bucket(q, k, nb, md)
    assert cuda_lib.wc_t5_relative_bucket(0, 5000, 32, 128) == -1


def test_create_rejects_bad_config(cuda_lib, tiny_model):
    rc, h, msg = _create(cuda_lib, tiny_model.gguf, None)
    assert rc == -6 and not h.value
    cfg = json.loads(tiny_model.config.to_json())
    del cfg["d_model"]
    rc, h, msg = _create(cuda_lib, tiny_model.gguf, json.dumps(cfg))
    assert rc == -6 and "d_model" in msg
    cfg = json.loads(tiny_model.config.to_json())
    cfg["feed_forward_proj"] = "relu"
    rc, h, msg = _create(cuda_lib, tiny_model.gguf, json.dumps(cfg))
    assert rc == -3


def test_create_rejects_bad_gguf(cuda_lib, tiny_model):
    cfg = tiny_model.config.to_json()
    rc, h, msg = _create(cuda_lib, b"", cfg)
    assert rc == -2
    rc, h, msg = _create(cuda_lib, b"XXXX" + tiny_model.gguf[4:], cfg)
    assert rc == -2 and "magic" in msg
    rc, h, msg = _create(cuda_lib, tiny_model.gguf[: len(tiny_model.gguf) // 2], cfg)
    assert rc == -2 and not h.value
    rc, h, msg = _create(cuda_lib, tiny_model.gguf[:200], cfg)
    assert rc == -2


def _rebuild(model, replace=None, drop=None):
    tensors = []
    for name, blocks in model.q4k.items():
        n = blocks.shape[0]
        tensors.append((name, 12, (n, blocks.shape[1] * 256), blocks.tobytes()))
    for name, arr in model.f32.items():
        tensors.append((name, GGML_TYPE_F32, arr.shape, arr.tobytes()))
    out = []
    for t in tensors:
        if drop and t[0] == drop:
            continue
        if replace and t[0] in replace:
            t = replace[t[0]]
        out.append(t)
    return write_gguf(out)


def test_create_rejects_missing_or_misshaped_tensor(cuda_lib, tiny_model):
    cfg = tiny_model.config.to_json()
    rc, h, msg = _create(cuda_lib, _rebuild(tiny_model, drop="linear.weight"), cfg)
    assert rc == -2 and "linear.weight" in msg
    name = "encoder.block.1.layer.0.SelfAttention.q.weight"
    f32 = np.zeros((256, 256), np.float32)
    rc, h, msg = _create(cuda_lib, _rebuild(tiny_model, replace={name: (name, GGML_TYPE_F32, f32.shape, f32.tobytes())}), cfg)
    assert rc == -3 and "Q4_K" in msg
    name = "encoder.final_layer_norm.weight"
    bad = np.ones(128, np.float32)
    rc, h, msg = _create(cuda_lib, _rebuild(tiny_model, replace={name: (name, GGML_TYPE_F32, bad.shape, bad.tobytes())}), cfg)
    assert rc == -3 and "shape" in msg


def test_create_without_visible_gpu_fails_cleanly(tiny_model, tmp_path):
    """A process with no visible GPU gets WC_E_CUDA from create (never a crash
    and never a CPU fallback)."""
    gg = tmp_path / "m.gguf"
    gg.write_bytes(tiny_model.gguf)
    code = f"""
import ctypes, sys
sys.path.insert(0, {ROOT!r})
from witchcraft_b200._lib import lib
l = lib()
b = open({str(gg)!r}, 'rb').read()
h = ctypes.c_void_p()
rc = l.wc_t5_create(0, b, len(b), {tiny_model.config.to_json()!r}.encode(), ctypes.byref(h))
print(rc, l.wc_t5_device_count(), l.wc_t5_last_error(None).decode())
"""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    rc, n, *msg = r.stdout.split()
    assert int(rc) == -4 and int(n) == 0
