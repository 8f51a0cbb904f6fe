"""Index-build helpers over the CUDA kernels of include/wc_index.h.

`kmeans` mirrors the reference's loop (src/lib.rs:210-280): start from the
given rows, then per iteration assign every row to its nearest center
(matmul_argmax_batched) and replace each center by the normalised sum of its
rows.  The reference draws the starting rows and the replacement row of an
empty cluster at random; here the caller supplies them (`init_rows`,
`empty_rows(iteration) -> [k] row indices`), so runs are reproducible.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._lib import WcError, lib


def _p(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def _check(rc: int) -> None:
    if rc != 0:
        msg = lib().wc_index_last_error()
        raise WcError(rc, msg.decode() if msg else "")


def assign(x: torch.Tensor, centers: torch.Tensor) -> torch.Tensor:
    """[m] u32 (as int32 storage) nearest center of each row of x (device f32)."""
    out = torch.empty(x.shape[0], dtype=torch.int32, device=x.device)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _check(lib().wc_assign_centers(_p(x), x.shape[0], _p(centers), centers.shape[0], x.shape[1], _p(out), st))
    return out


def kmeans_update(x: torch.Tensor, idx: torch.Tensor, k: int, empty_src: torch.Tensor):
    centers = torch.empty(k, x.shape[1], dtype=torch.float32, device=x.device)
    counts = torch.empty(k, dtype=torch.int32, device=x.device)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _check(lib().wc_kmeans_update(_p(x), x.shape[0], x.shape[1], _p(idx), k, _p(empty_src), _p(centers),
                                  _p(counts), st))
    return centers, counts


def residual_q4(x: torch.Tensor, idx: torch.Tensor, centers: torch.Tensor) -> torch.Tensor:
    out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=torch.uint8, device=x.device)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _check(lib().wc_residual_q4(_p(x), x.shape[0], x.shape[1], _p(idx), _p(centers), _p(out), st))
    return out


def kmeans(x: torch.Tensor, k: int, max_iter: int, init_rows: np.ndarray, empty_rows=None) -> torch.Tensor:
    """Centers [k, dim] after max_iter iterations (src/lib.rs:210-280)."""
    m = x.shape[0]
    centers = x[torch.as_tensor(np.asarray(init_rows, np.int64), device=x.device)].contiguous()
    for it in range(max_iter):
        idx = assign(x, centers)
        src = np.zeros(k, np.int64) if empty_rows is None else np.asarray(empty_rows(it), np.int64)
        if src.min(initial=0) < 0 or src.max(initial=0) >= m:
            raise ValueError("empty-cluster rows out of range")
        centers, _ = kmeans_update(x, idx, k, torch.as_tensor(src, device=x.device))
    return centers
