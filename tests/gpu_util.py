"""Helpers for the GPU tests: torch is used only for device memory and for
the fp32 reference of the floating-point kernels."""
import ctypes

import numpy as np
import torch

from witchcraft_b200._lib import check, lib


def dptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def q4k_to_device(blocks: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)).cuda()


def dequant_gpu(blocks: np.ndarray) -> torch.Tensor:
    d = q4k_to_device(blocks)
    n = d.numel() // 144
    out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
    check(lib().wc_q4k_dequant(dptr(d), n, dptr(out), stream_ptr()))
    torch.cuda.synchronize()
    return out


def gemm_gpu(x16: torch.Tensor, w_blocks: np.ndarray, epilogue: int, w_up_blocks=None, out=None):
    M, K = x16.shape
    N = w_blocks.shape[0]
    dw = q4k_to_device(w_blocks)
    du = q4k_to_device(w_up_blocks) if w_up_blocks is not None else None
    if out is None:
        dt = torch.float16 if epilogue in (0, 1) else torch.float32
        out = torch.empty(M, N, dtype=dt, device="cuda")
    check(lib().wc_gemm_q4k(dptr(x16), M, K, dptr(dw), dptr(du) if du is not None else None, N, epilogue,
                            dptr(out), stream_ptr()))
    torch.cuda.synchronize()
    return out


def cosine_rows(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = a.reshape(-1, a.shape[-1]).astype(np.float64)
    b = b.reshape(-1, b.shape[-1]).astype(np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1) + 1e-30)
