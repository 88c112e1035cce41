"""GPU checks of the tcgen05 3xTF32 projection (``fx_linear_3xtf32_f32``) and its
operand split (``fx_tf32_split_f32``), through the C ABI.

The projection keeps the contract of ``fx_linear_f32`` (the reference's FP32
projection, csrc/cublaslt_linear/cublaslt_linear_cuda.h:20-33): its error
against an FP64 product must stay within a small multiple of a plain FP32
GEMM's error on the same operands (TF32 alone would be ~1000x worse)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from flux_b200 import _native
    return _native, _native.load()


def split(x):
    native, lib = _lib()
    hi, lo = torch.empty_like(x), torch.empty_like(x)
    native.check(lib.fx_tf32_split_f32(x.data_ptr(), hi.data_ptr(), lo.data_ptr(), x.numel(),
                                       torch.cuda.current_stream().cuda_stream))
    return hi, lo


def linear(x, w, residual=None):
    native, lib = _lib()
    hi, lo = split(w)
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty(m, n, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    native.check(lib.fx_linear_3xtf32_f32(x.data_ptr(), hi.data_ptr(), lo.data_ptr(),
                                          residual.data_ptr() if residual is not None else None, out.data_ptr(),
                                          m, k, n, err.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def test_split_is_exact_tf32_pair():
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(4096, generator=g) * torch.logspace(-20, 20, 4096)).cuda()
    hi, lo = split(x)
    bits = lambda t: t.view(torch.int32) & 0x1FFF  # noqa: E731
    assert int(bits(hi).abs().sum()) == 0 and int(bits(lo).abs().sum()) == 0
    # hi + lo carries x to 2^-21 relative
    rel = ((hi.double() + lo.double() - x.double()).abs() / x.double().abs()).max().item()
    assert rel < 2.0 ** -21


@pytest.mark.parametrize("m,k,n", [(1, 576, 960), (64, 576, 576), (5, 1536, 576), (37, 576, 3072),
                                   (64, 576, 49152), (300, 576, 960), (1000, 1536, 576), (4096, 576, 3072),
                                   # CTA pairs (N a multiple of 192) at the prefill's size, one weight block,
                                   # and the persistent single-CTA form (N not a multiple of 192)
                                   (8192, 576, 576), (1000, 576, 192), (300, 576, 1000)])
def test_linear_3xtf32_matches_fp32(m, k, n):
    g = torch.Generator().manual_seed(m * 7 + n)
    x = torch.randn(m, k, generator=g).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).cuda()
    out = linear(x, w)
    ref = x.double() @ w.double().T
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        fp32 = x @ w.T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    err = (out.double() - ref).abs().max().item()
    err32 = (fp32.double() - ref).abs().max().item()
    assert err <= 4 * err32 + 1e-7, (err, err32)


def test_linear_3xtf32_residual_and_ragged_edges():
    g = torch.Generator().manual_seed(9)
    m, k, n = 130, 1536, 200  # neither M nor N a tile multiple
    x = torch.randn(m, k, generator=g).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).cuda()
    r = torch.randn(m, n, generator=g).cuda()
    out = linear(x, w, r)
    ref = x.double() @ w.double().T + r.double()
    assert (out.double() - ref).abs().max().item() < 2e-5


def test_linear_3xtf32_rows_are_independent():
    """A row's result does not depend on the other rows of its tile (the
    batched runtime's per-sequence bitwise property)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(64, 576, generator=g).cuda()
    w = (torch.randn(960, 576, generator=g) * 0.02).cuda()
    full = linear(x, w)
    alone = linear(x[17:18].contiguous(), w)
    assert torch.equal(full[17:18], alone)
