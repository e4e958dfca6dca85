"""GPU: the tensor-core projection kernel (tcgen05 + TMA) of the batched path
against a float32 torch reference on the same bf16 inputs."""

from __future__ import annotations

import ctypes

import pytest
import torch

from transformer_b200 import _lib

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _gemm(W, X, epi, resid=None, ldy=None, ksplit=0):
    lib = _lib.load()
    M, K = W.shape
    N = X.shape[0]
    ldy = ldy or M
    y = torch.full((N, ldy), float("nan"), dtype=torch.float32, device=W.device) if epi != 2 else None
    ybf = torch.zeros((N, ldy), dtype=torch.bfloat16, device=W.device) if epi == 2 else None
    st = lib.b2d_test_gemm(_p(W), M, K, _p(X), N, epi | (ksplit << 8), _p(y), _p(resid), _p(ybf), ldy,
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.B2D_OK, _lib.status_str(st)
    return y if epi != 2 else ybf


@pytest.mark.parametrize("M,K,N", [(128, 64, 16), (256, 1024, 8), (1536, 1024, 64), (1024, 2816, 37),
                                   (384, 256, 130), (1024, 1024, 100), (5632, 1024, 256), (1024, 2816, 300)])
def test_gemm_f32_matches_torch(cuda, M, K, N):
    """Every tile width (16..256 batch rows) with the decode step's K split."""
    g = torch.Generator(device="cpu").manual_seed(M + K + N)
    W = (torch.randn(M, K, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    X = torch.randn(N, K, generator=g).to(torch.bfloat16).to(cuda)
    y = _gemm(W, X, 0)
    ref = X.float() @ W.float().T
    torch.testing.assert_close(y, ref, atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("ks", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_cluster_split_k(cuda, ks, epi):
    """K split over 1..8 cluster CTAs (uneven slices at ks=3, 5) for each
    epilogue; the split result equals the unsplit one up to f32 reassociation
    and is bitwise reproducible."""
    g = torch.Generator(device="cpu").manual_seed(40 + ks)
    M, K, N = 1024, 1344, 48
    W = (torch.randn(M, K, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    X = torch.randn(N, K, generator=g).to(torch.bfloat16).to(cuda)
    R = torch.randn(N, M, generator=g).to(cuda) if epi == 1 else None
    ldy = M // 2 if epi == 2 else None
    out = _gemm(W, X, epi, resid=R, ldy=ldy, ksplit=ks)
    again = _gemm(W, X, epi, resid=R, ldy=ldy, ksplit=ks)
    assert torch.equal(out, again)
    full = X.float() @ W.float().T
    if epi == 0:
        torch.testing.assert_close(out, full, atol=1e-3, rtol=1e-3)
    elif epi == 1:
        torch.testing.assert_close(out, R + full, atol=1e-3, rtol=1e-3)
    else:
        ref = torch.nn.functional.silu(full[:, 0::2]) * full[:, 1::2]
        torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("ks", [1, 3])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_96_row_tile(cuda, ks, epi):
    """Batches of 65..96 rows take 96-row tiles (a TMEM allocation of 128
    columns, 3 tiles for 256 rows): every epilogue, unsplit and split."""
    g = torch.Generator(device="cpu").manual_seed(90 + 3 * ks + epi)
    M, K, N = 512, 1024, 90
    W = (torch.randn(M, K, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    X = torch.randn(N, K, generator=g).to(torch.bfloat16).to(cuda)
    R = torch.randn(N, M, generator=g).to(cuda) if epi == 1 else None
    ldy = M // 2 if epi == 2 else None
    out = _gemm(W, X, epi, resid=R, ldy=ldy, ksplit=ks)
    full = X.float() @ W.float().T
    if epi == 0:
        torch.testing.assert_close(out, full, atol=1e-3, rtol=1e-3)
    elif epi == 1:
        torch.testing.assert_close(out, R + full, atol=1e-3, rtol=1e-3)
    else:
        ref = torch.nn.functional.silu(full[:, 0::2]) * full[:, 1::2]
        torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)


def test_gemm_residual_epilogue(cuda):
    g = torch.Generator(device="cpu").manual_seed(3)
    W = (torch.randn(1024, 1024, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    X = torch.randn(64, 1024, generator=g).to(torch.bfloat16).to(cuda)
    R = torch.randn(64, 1024, generator=g).to(cuda)
    y = _gemm(W, X, 1, resid=R)
    torch.testing.assert_close(y, R + X.float() @ W.float().T, atol=1e-3, rtol=1e-3)


def test_gemm_swiglu_epilogue(cuda):
    """Rows 2j / 2j+1 are gate / up of hidden unit j: out[:, j] = bf16(silu(g) * u)."""
    g = torch.Generator(device="cpu").manual_seed(4)
    M, K, N = 512, 1024, 48
    W = (torch.randn(M, K, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    X = torch.randn(N, K, generator=g).to(torch.bfloat16).to(cuda)
    out = _gemm(W, X, 2, ldy=M // 2)
    full = X.float() @ W.float().T
    ref = (torch.nn.functional.silu(full[:, 0::2]) * full[:, 1::2])
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)
