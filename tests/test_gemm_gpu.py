"""GPU numerics of the tensor-core GEMM that carries every projection of the
decode step (mb_gemm_bf16: the reference's GEMV, kernels-decode.ts:127-142,
y = b + x W, for many rows at once), through the C ABI, against a plain
PyTorch fp32 reference of the same op on the same bf16 inputs.

Tolerance: the products of bf16 inputs are exact in fp32 and only the order of
the fp32 sums differs, so outputs agree within 1e-4 relative to the row's
magnitude (|x| |W| summed over K); the GELU epilogue stores bf16, so it is
checked within one bf16 rounding (2^-8 relative) plus that."""
import ctypes

import pytest
import torch

from mockbird_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def _run(m, n, k, epi, bn=0, splits=0, bias=True, seed=0):
    lib = _lib.load()
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    x = torch.randn(m, k, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(k, n, generator=g, device=DEV) * 0.05).to(torch.bfloat16)  # W [K][N]
    wt = w.t().contiguous()                                                    # the layout the GEMM reads
    b = torch.randn(n, generator=g, device=DEV) if bias else None
    y0 = torch.randn(m, n, generator=g, device=DEV)
    y = y0.clone() if epi != 2 else torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream(DEV)
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    outs = []
    for _ in range(2):  # twice: the same plan gives the same bits
        if epi == 1:
            y.copy_(y0)
        rc = lib.mb_gemm_bf16(m, n, k, P(x), P(wt), P(b), P(y), epi, bn, splits, P(status),
                              ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0
        torch.cuda.synchronize(DEV)
        assert int(status.item()) == 0
        outs.append(y.clone())
    assert torch.equal(outs[0], outs[1])
    ref = x.float() @ w.float() + (b if bias else 0.0)
    scale = (x.float().abs() @ w.float().abs()) + 1.0
    if epi == 0:
        err = ((y - ref).abs() / scale).max().item()
        assert err < 1e-4, err
    elif epi == 1:
        err = ((y - (y0 + ref)).abs() / (scale + y0.abs())).max().item()
        assert err < 1e-4, err
    else:
        want = _gelu_tanh(ref)
        err = ((y.float() - want).abs() / (want.abs() * 2 ** -8 + scale * 1e-3)).max().item()
        assert err < 1.0, err


# the decoder step's four shapes at config 4's 256 streams, and the audio head (the library's plans)
@pytest.mark.parametrize("n,k,epi", [(2304, 768, 0), (768, 768, 1), (3072, 768, 2), (768, 3072, 1), (1024, 768, 0)])
def test_decoder_shapes(n, k, epi):
    _run(256, n, k, epi)


# row counts around the 128-row tile, one row, and more than two tiles
@pytest.mark.parametrize("m", [1, 2, 127, 128, 129, 300])
def test_row_edges(m):
    _run(m, 768, 768, 1)
    _run(m, 192, 64, 0, bias=False)


# every tile width, K split over clusters of 1..8 CTAs, including splits that do
# not divide the K blocks evenly
@pytest.mark.parametrize("bn", [32, 64, 128])
@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8])
def test_tiles_and_splits(bn, splits):
    _run(200, 768, 768, 0, bn=bn, splits=splits)
    _run(130, 256, 3072, 1, bn=bn, splits=splits)
    _run(256, 384, 512, 2, bn=bn, splits=splits)


def test_rejects_bad_shapes():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.mb_gemm_bf16(4, 48, 64, p, p, None, p, 0, 0, 0, p, None) == 1    # n % 32
    assert lib.mb_gemm_bf16(4, 64, 100, p, p, None, p, 0, 0, 0, p, None) == 1   # k % 64
    assert lib.mb_gemm_bf16(4, 64, 64, p, p, None, p, 0, 64, 2, p, None) == 1   # splits > k / 64
    assert lib.mb_gemm_bf16(4, 96, 64, p, p, None, p, 0, 64, 1, p, None) == 1   # bn does not divide n
    assert lib.mb_gemm_bf16(4, 64, 640, p, p, None, p, 0, 64, 9, p, None) == 1  # more than 8 splits
    assert lib.mb_gemm_bf16(4, 64, 64, p, p, None, p, 0, 64, 0, p, None) == 1   # bn without splits


# CTA pairs (splits = -1): one tcgen05 MMA over two CTAs, each loading half the
# rows of x and of W^T; every tile width, rows around the 128-row tile and the
# 64-row half, and the three epilogues
@pytest.mark.parametrize("bn", [32, 64, 128])
def test_cta_pairs(bn):
    _run(256, 768, 768, 0, bn=bn, splits=-1)
    _run(256, 384, 3072, 1, bn=bn, splits=-1)
    _run(256, 1024, 768, 2, bn=bn, splits=-1)


@pytest.mark.parametrize("m", [1, 63, 64, 65, 127, 129, 300])
def test_cta_pair_row_edges(m):
    _run(m, 256, 512, 1, bn=64, splits=-1)
