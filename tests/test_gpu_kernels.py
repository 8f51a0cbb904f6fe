"""Kernel-level parity on the GPU through the C ABI: bit-exact Q4_K dequant,
the tcgen05 Q4_K GEMM (all epilogues, config-2 shapes and ragged M) and the
encoder attention (config-3 shape, padding, long sequences)."""
import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import oracle as O
from witchcraft_b200._lib import check, lib
from witchcraft_b200.synth import quantize_q4k

from gpu_util import dequant_gpu, dptr, gemm_gpu, q4k_to_device, stream_ptr

pytestmark = pytest.mark.gpu


def _same_bits(a, b):
    a = np.asarray(a, np.float32).reshape(-1)
    b = np.asarray(b, np.float32).reshape(-1)
    both_nan = np.isnan(a) & np.isnan(b)
    return np.all((a.view(np.uint32) == b.view(np.uint32)) | both_nan)


def test_dequant_bit_exact_against_golden():
    g = np.load(os.path.join(GOLDEN, "q4k_golden.npz"))
    assert _same_bits(dequant_gpu(g["blocks"]).cpu().numpy(), g["values"])


def test_dequant_bit_exact_full_embedding_table(xtr_model):
    blocks = xtr_model.q4k["encoder.embed_tokens.weight"]
    assert _same_bits(dequant_gpu(blocks).cpu().numpy(), O.q4k_dequant(blocks))


def test_dequant_f16_is_rounded_f32_dequant(xtr_model):
    """The resident f16 weights equal the bit-exact f32 dequant rounded to f16."""
    g = np.load(os.path.join(GOLDEN, "q4k_golden.npz"))
    for blocks, ref32 in [(g["blocks"], g["values"]),
                          (xtr_model.q4k["encoder.block.0.layer.1.DenseReluDense.wi_0.weight"], None)]:
        if ref32 is None:
            ref32 = O.q4k_dequant(blocks)
        d = q4k_to_device(blocks)
        n = d.numel() // 144
        out = torch.empty(n * 256, dtype=torch.float16, device="cuda")
        check(lib().wc_q4k_dequant_f16(dptr(d), n, dptr(out), stream_ptr()))
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        want = np.asarray(ref32, np.float32).reshape(-1).astype(np.float16)
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan)
        assert np.array_equal(got[~nan].view(np.uint16), want[~nan].view(np.uint16))


def _gelu(g):
    return 0.5 * g * (1.0 + torch.tanh(0.7978845608 * (g + 0.044715 * g ** 3)))


def _weights(N, K, seed):
    w = np.random.default_rng(seed).standard_normal((N, K)).astype(np.float32) * 0.02
    blocks = quantize_q4k(w)
    wd = torch.from_numpy(O.q4k_dequant_matrix(blocks)).cuda()
    return blocks, wd


# M <= 32 runs the small-M kernel (except the residual epilogue), M >= 512 with N % 256 == 0 the
# 2-SM persistent kernel, the rest the 1-SM kernel
@pytest.mark.parametrize("M,K,N", [(8192, 768, 2304), (8192, 2048, 768), (1, 768, 768), (77, 768, 2304),
                                   (300, 2048, 768), (129, 256, 128), (2048, 768, 128), (511, 768, 768),
                                   (512, 768, 768), (1000, 2048, 768), (16384, 768, 256), (700, 256, 512),
                                   (5, 2048, 768), (16, 768, 2304), (32, 2048, 768), (9, 256, 128), (33, 768, 768)])
@pytest.mark.parametrize("epi", [0, 3])
def test_gemm_store(M, K, N, epi):
    blocks, wd = _weights(N, K, seed=M + N)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(2)).cuda().to(torch.float16)
    y = gemm_gpu(x, blocks, epi).float()
    # same f16-rounded operands, fp32 accumulation
    ref = x.float() @ wd.to(torch.float16).float().T
    tol = 2e-3
    err = (y - ref).abs().max().item() / ref.abs().max().item()
    assert err < tol, err
    # and against the unrounded f32 weights (the reference's numbers)
    ref32 = x.float() @ wd.T
    assert ((y - ref32).abs().max() / ref32.abs().max()).item() < 1e-2


@pytest.mark.parametrize("M,K,F", [(8192, 768, 2048), (200, 768, 2048), (64, 256, 512), (1300, 768, 2048),
                                   (600, 256, 512),
                                   (1, 768, 2048), (13, 768, 2048), (32, 256, 512)])
def test_gemm_geglu(M, K, F):
    b0, w0 = _weights(F, K, 10)
    b1, w1 = _weights(F, K, 11)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(3)).cuda().to(torch.float16)
    y = gemm_gpu(x, b0, 1, w_up_blocks=b1).float()
    xf = x.float()
    ref = _gelu(xf @ w0.to(torch.float16).float().T) * (xf @ w1.to(torch.float16).float().T)
    err = ((y - ref).abs().max() / ref.abs().max()).item()
    assert err < 5e-3, err


@pytest.mark.parametrize("M", [1, 7, 32, 333, 4000])
def test_gemm_residual_accumulates(M):
    K, N = 2048, 768
    blocks, wd = _weights(N, K, 12)
    x = torch.randn(M, K).cuda().to(torch.float16)
    base = torch.randn(M, N, device="cuda")
    out = base.clone()
    gemm_gpu(x, blocks, 2, out=out)
    ref = base + x.float() @ wd.to(torch.float16).float().T
    assert ((out - ref).abs().max() / ref.abs().max()).item() < 2e-3


def _dequant_f16(blocks):
    d = q4k_to_device(blocks)
    out = torch.empty(blocks.shape[0], blocks.shape[1] * 256, dtype=torch.float16, device="cuda")
    check(lib().wc_q4k_dequant_f16(dptr(d), d.numel() // 144, dptr(out), stream_ptr()))
    return out


def _gemm_f16_gpu(x16, w16, epi, w_up16=None, out=None):
    M, K = x16.shape
    N = w16.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.float16 if epi in (0, 1) else torch.float32, device="cuda")
    check(lib().wc_gemm_f16(dptr(x16), M, K, dptr(w16), dptr(w_up16) if w_up16 is not None else None, N, epi,
                            dptr(out), stream_ptr()))
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("M", [8192, 1300, 300, 1])
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_gemm_f16_weights(M, epi):
    """The forward's large-M GEMM on resident f16 weights: bitwise equal to the
    fused-dequant kernel where both run the 2-SM kernel (M >= 512), and within
    the GEMM tolerance of fp32 torch on the same operands everywhere."""
    K, N = (2048, 768) if epi in (2, 3) else (768, 512)
    b0, w0 = _weights(N, K, 20 + epi)
    b1, w1 = _weights(N, K, 30 + epi)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(4)).cuda().to(torch.float16)
    h0, h1 = _dequant_f16(b0), _dequant_f16(b1)
    base = torch.randn(M, N, generator=torch.Generator().manual_seed(5)).cuda() if epi == 2 else None
    y16 = _gemm_f16_gpu(x, h0, epi, h1 if epi == 1 else None, base.clone() if base is not None else None)
    xf = x.float()
    if epi == 1:
        ref = _gelu(xf @ h0.float().T) * (xf @ h1.float().T)
    else:
        ref = xf @ h0.float().T + (base if epi == 2 else 0)
    assert ((y16.float() - ref).abs().max() / ref.abs().max()).item() < 5e-3
    if M >= 512:
        yq = gemm_gpu(x, b0, epi, w_up_blocks=b1 if epi == 1 else None,
                      out=base.clone() if base is not None else None)
        assert torch.equal(y16, yq)


def test_gemm_rejects_bad_shapes():
    l = lib()
    x = torch.zeros(8, 300, dtype=torch.float16, device="cuda")
    assert l.wc_gemm_q4k(dptr(x), 8, 300, dptr(x), None, 128, 0, dptr(x), stream_ptr()) == -1
    assert l.wc_gemm_q4k(dptr(x), 8, 256, dptr(x), None, 100, 0, dptr(x), stream_ptr()) == -1
    assert l.wc_gemm_q4k(dptr(x), 8, 256, dptr(x), None, 128, 1, dptr(x), stream_ptr()) == -1


def _attention_gpu(qkv16, B, L, H, lengths, bias_tab):
    out = torch.empty(B * L, H * 64, dtype=torch.float16, device="cuda")
    dl = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    db = torch.from_numpy(np.ascontiguousarray(bias_tab, np.float32)).cuda()
    check(lib().wc_attention(dptr(qkv16), B, L, H, dptr(dl), dptr(db), 32, 128, dptr(out), stream_ptr()))
    torch.cuda.synchronize()
    return out


def _attention_torch(qkv, B, L, H, lengths, bias_tab):
    """fp32 reference: softmax(QK^T + bias, key mask) V without scaling."""
    q, k, v = qkv.float().view(B, L, 3, H, 64).unbind(2)
    q, k, v = (t.permute(0, 2, 1, 3) for t in (q, k, v))
    delta = torch.arange(L)[None, :] - torch.arange(L)[:, None]
    lut = torch.tensor([O.bucket(0, d) if d >= 0 else O.bucket(-d, 0) for d in range(-(L - 1), L)])
    bucket = lut[delta + L - 1].cuda()
    bias = torch.from_numpy(bias_tab).cuda()[bucket].permute(2, 0, 1)  # H, L, L
    s = q @ k.transpose(-1, -2) + bias[None]
    mask = torch.arange(L, device="cuda")[None, :] >= torch.tensor(lengths, device="cuda")[:, None]
    s = s.masked_fill(mask[:, None, None, :], float("-inf"))
    o = torch.softmax(s, -1) @ v
    return o.permute(0, 2, 1, 3).reshape(B * L, H * 64)


@pytest.mark.parametrize("B,L,lengths", [(2, 128, [128, 128]), (4, 200, [200, 130, 64, 1]),
                                         (2, 65, [65, 33]), (1, 2048, [2048]), (3, 1, [1, 1, 1]),
                                         # L <= 64: the mma.sync kernel of short batches
                                         (4, 32, [32, 17, 1, 5]), (2, 64, [64, 40]), (3, 17, [17, 9, 16]),
                                         (2, 2, [2, 1]), (2, 33, [33, 20]), (3, 31, [0, 31, 7]),
                                         # L > 64: the tcgen05 kernel with odd tile counts, an empty
                                         # sequence and the 1024 / 1025 sizes
                                         (3, 300, [0, 300, 129]), (2, 384, [300, 384]), (1, 1024, [1024]),
                                         (5, 129, [129, 128, 127, 64, 65]), (2, 1025, [1025, 700])])
def test_attention_matches_oracle(B, L, lengths):
    H = 12
    g = torch.Generator().manual_seed(B * 1000 + L)
    qkv = torch.randn(B * L, 3 * H * 64, generator=g).to(torch.float16)
    bias_tab = (np.random.default_rng(L).standard_normal((32, H)) * 0.1).astype(np.float32)
    out = _attention_gpu(qkv.cuda(), B, L, H, lengths, bias_tab).float().cpu().numpy()
    ref = O.attention(qkv.float().numpy(), B, L, H, lengths, bias_tab)
    for b in range(B):
        if lengths[b] == 0:  # an empty sequence: every output row is zero
            assert not out[b * L:(b + 1) * L].any(), b
            continue
        rows = slice(b * L, b * L + lengths[b])
        err = np.abs(out[rows] - ref[rows]).max()
        assert err < 2e-2, (b, err)


@pytest.mark.parametrize("H", [2, 6, 3, 16])
def test_attention_head_counts(H):
    """Head counts from 2 to 16, odd and even, against the fp32 torch
    reference; rows of wholly padded query tiles are zero."""
    B, L = 3, 260
    lengths = [260, 131, 77]
    qkv = torch.randn(B * L, 3 * H * 64, generator=torch.Generator().manual_seed(H)).to(torch.float16).cuda()
    bias_tab = (np.random.default_rng(H).standard_normal((32, H)) * 0.1).astype(np.float32)
    out = _attention_gpu(qkv, B, L, H, lengths, bias_tab).float()
    ref = _attention_torch(qkv, B, L, H, lengths, bias_tab)
    for b in range(B):
        rows = slice(b * L, b * L + lengths[b])
        assert (out[rows] - ref[rows]).abs().max().item() < 2e-2, b
        assert not out[b * L + (lengths[b] + 127) // 128 * 128:(b + 1) * L].any()


def test_attention_config3_against_torch():
    """Config 3: B=64, L=512, 12 heads, lengths U[32, 512], bias N(0, 0.1)."""
    B, L, H = 64, 512, 12
    rng = np.random.default_rng(4)
    lengths = rng.integers(32, 513, B).tolist()
    qkv = torch.randn(B * L, 3 * H * 64, generator=torch.Generator().manual_seed(3)).to(torch.float16).cuda()
    bias_tab = (np.random.default_rng(3).standard_normal((32, H)) * 0.1).astype(np.float32)
    out = _attention_gpu(qkv, B, L, H, lengths, bias_tab).float()
    ref = _attention_torch(qkv, B, L, H, lengths, bias_tab)
    for b in range(B):
        rows = slice(b * L, b * L + lengths[b])
        assert (out[rows] - ref[rows]).abs().max().item() < 2e-2, b
        assert torch.all(torch.isfinite(out[b * L:(b + 1) * L]))


def test_in_kernel_wait_timeout_is_reported():
    """A wait that can never finish gives up after its limit, the kernel
    reports WC_E_TIMEOUT through the status word, and the context still works."""
    assert lib().wc_selftest_wait_timeout(20_000_000) == -5
    g = np.load(os.path.join(GOLDEN, "q4k_golden.npz"))
    assert _same_bits(dequant_gpu(g["blocks"]).cpu().numpy(), g["values"])
