"""tcgen05 3xTF32 GEMM (vcb_tc_gemm) against float64 products: error within
the 3xTF32 bound (~2^-22 of sum |a||b| per element) and inside the fp32
parity tolerance of torch's fp32 matmul."""
import numpy as np
import pytest
import torch

from vibecheck_nn_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None
P = _lib.ptr


def split(x):
    hi = torch.empty_like(x)
    lo = torch.empty_like(x)
    _lib.check(_lib.lib().vcb_tf32_split(x.numel(), P(x), P(hi), P(lo),
                                         _lib.stream_of(x.device)))
    return hi, lo


def padded(x):
    """Copy into a buffer whose leading dimension is a multiple of 4."""
    r, c = x.shape
    out = torch.zeros((r, (c + 3) // 4 * 4), device=x.device)
    out[:, :c] = x
    return out


def tc_gemm(A, B, bias=None):
    M, K = A.shape
    N = B.shape[0]
    Ah, Al = split(padded(A))
    Bh, Bl = split(padded(B))
    C = torch.full((M, N), float('nan'), device=A.device)
    err = torch.zeros(1, dtype=torch.int32, device=A.device)
    _lib.check(_lib.lib().vcb_tc_gemm(M, N, K, P(Ah), P(Al), Ah.stride(0), P(Bh), P(Bl),
                                      Bh.stride(0), P(bias), P(C), N, P(err),
                                      _lib.stream_of(A.device)))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return C


def test_split_is_exact():
    x = torch.randn(10007, device=DEV) * torch.logspace(-20, 20, 10007, device=DEV)
    hi, lo = split(x)
    assert torch.equal(hi + lo, x)
    assert torch.all((hi.view(torch.int32) & 0x1FFF) == 0)
    assert torch.all(lo.abs() <= hi.abs() * 2.0 ** -11)


@pytest.mark.parametrize('M,N,K', [(128, 128, 32), (1, 1, 1), (300, 200, 100),
                                   (129, 257, 33), (1024, 512, 1000), (640, 384, 4096)])
def test_tc_gemm_matches_fp64(M, N, K):
    g = torch.Generator(device='cpu').manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, (K + 3) // 4 * 4, generator=g)[:, :K].to(DEV)
    B = torch.randn(N, (K + 3) // 4 * 4, generator=g)[:, :K].to(DEV)
    bias = torch.randn(N, generator=g).to(DEV)
    C = tc_gemm(A, B, bias)
    ref = A.double() @ B.double().T + bias.double()
    scale = A.double().abs() @ B.double().abs().T + bias.double().abs()
    rel = ((C.double() - ref).abs() / scale).max().item()
    fp32 = (A @ B.T + bias).double()
    rel32 = ((fp32 - ref).abs() / scale).max().item()
    print(f'M={M} N={N} K={K}: 3xtf32 {rel:.3e}  cuBLAS fp32 {rel32:.3e} of sum|a||b|')
    # 3xTF32 drops lo_a lo_b (~2^-22 |ab|); chunk partials are summed in fp32
    assert rel < max(4e-7, 2.0 * rel32), (rel, rel32)


def test_tc_gemm_throughput_vs_cublas_fp32():
    """Timing of the 3xTF32 GEMM against cuBLAS fp32 (CUDA events, 3 warm-up
    + 10 launches); the tensor-core path must beat cuBLAS fp32 on a large
    shape."""
    M = N = K = 4096
    A = torch.randn(M, K, device=DEV)
    B = torch.randn(N, K, device=DEV)
    Ah, Al = split(A)
    Bh, Bl = split(B)
    C = torch.empty(M, N, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)

    def tc():
        _lib.check(_lib.lib().vcb_tc_gemm(M, N, K, P(Ah), P(Al), K, P(Bh), P(Bl), K, None, P(C),
                                          N, P(err), _lib.stream_of(DEV)))

    def timed(fn):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 10

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        t_tc = timed(tc)
        t_32 = timed(lambda: A @ B.T)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    fl = 2.0 * M * N * K
    print(f'{M}x{N}x{K}: tcgen05 3xTF32 {t_tc:.3f} ms = {fl / t_tc / 1e9:.1f} TFLOP/s; '
          f'cuBLAS fp32 {t_32:.3f} ms = {fl / t_32 / 1e9:.1f} TFLOP/s')
    assert int(err.item()) == 0
    assert t_tc < t_32
