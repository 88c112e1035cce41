"""GPU parity of the compact-cache decode attention (the TMA-staged fast path of
``fx_gqa_decode_attention_f32``) on the isolated-attention shapes of the
benchmark configs: Q, K, V ~ N(0, 1) seeded, B in {1, 16, 64, 256}, L in
{128, 1024, 8192}, scale 1/8, causal over the valid length (the reference's
op is batch-1 only, so B > 1 is checked against the oracle restatement of
``flux/ops/gqa_decode_attention.py:37-83``)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import smollm2 as o

pytestmark = pytest.mark.gpu

TOL = dict(rtol=2e-5, atol=2e-6)


def attention(q, k, v, length, fused=False):
    """``fx_gqa_decode_attention_f32`` through the C ABI (any batch; the torch
    op keeps the reference's batch-1 contract).  `fused`: a workspace with
    zeroed merge counters after the partials (the merge runs in the chunk
    kernel)."""
    from flux_b200 import _native
    lib = _native.load()
    batch, capacity = q.shape[0], k.shape[2]
    out = torch.empty(batch, 9, 1, 64, device="cuda")
    floats = lib.fx_gqa_decode_attention_workspace_floats(batch, 9, capacity, 64) + (batch * 3 if fused else 0)
    ws = torch.zeros(floats, device="cuda") if fused else torch.empty(floats, device="cuda")
    ln = torch.tensor(length, device="cuda")
    _native.check(lib.fx_gqa_decode_attention_f32(
        q.data_ptr(), _native.int64_array(q.stride()), k.data_ptr(), _native.int64_array(k.stride()),
        v.data_ptr(), _native.int64_array(v.stride()), None, None, None, ln.data_ptr(), out.data_ptr(),
        ws.data_ptr(), floats, 0.125, batch, 9, 3, capacity, 64, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return out


def _inputs(batch, length, capacity, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, 9, 1, 64, generator=g)
    k = torch.randn(batch, 3, capacity, 64, generator=g)
    v = torch.randn(batch, 3, capacity, 64, generator=g)
    return q, k, v


@pytest.mark.parametrize("batch,length", [(1, 128), (1, 1024), (1, 8192), (16, 128), (16, 1024), (16, 8192),
                                          (64, 128), (64, 1024), (256, 128), (256, 1024)])
def test_compact_attention_vs_oracle(batch, length):
    q, k, v = _inputs(batch, length, length, seed=batch * 100003 + length)
    out = attention(q.cuda(), k.cuda(), v.cuda(), length)
    expected = o.gqa_decode_attention(q.numpy(), k.numpy(), v.numpy(), None, 0.125, length)
    np.testing.assert_allclose(out.cpu().numpy(), expected, **TOL)


@pytest.mark.parametrize("capacity,length", [(130, 1), (130, 129), (1000, 777), (4097, 4097)])
def test_compact_attention_matches_generic_path(capacity, length):
    """The fast path (contiguous caches) against the generic kernel on the same
    values (a strided view of a padded buffer forces the generic kernel)."""
    q, k, v = _inputs(3, length, capacity, seed=capacity + length)
    fast = attention(q.cuda(), k.cuda(), v.cuda(), length)
    kp = torch.zeros(3, 3, capacity, 65)
    vp = torch.zeros(3, 3, capacity, 65)
    kp[..., :64] = k
    vp[..., :64] = v
    generic = attention(q.cuda(), kp.cuda()[..., :64], vp.cuda()[..., :64], length)
    np.testing.assert_allclose(fast.cpu().numpy(), generic.cpu().numpy(), **TOL)
    expected = o.gqa_decode_attention(q.numpy(), k.numpy(), v.numpy(), None, 0.125, length)
    np.testing.assert_allclose(fast.cpu().numpy(), expected, **TOL)


def test_compact_attention_large_batch_long_context_properties():
    """B = 64 / 256 at L = 8192 (too slow for the numpy oracle in full): every
    output is a convex combination of V rows, so with V = const it equals the
    constant, and with Q = 0 it equals the mean of V (the reference's
    known-answer case, csrc/benchmarks/cuda_microbenchmarks.cu:395-405)."""
    for batch in (64, 256):
        length = 8192
        g = torch.Generator().manual_seed(batch)
        k = torch.randn(batch, 3, length, 64, generator=g).cuda()
        v = torch.randn(batch, 3, length, 64, generator=g).cuda()
        q = torch.zeros(batch, 9, 1, 64, device="cuda")
        out = attention(q, k, v, length)
        mean = v.mean(dim=2).repeat_interleave(3, dim=1).unsqueeze(2)
        torch.testing.assert_close(out, mean, rtol=1e-4, atol=1e-5)
        q = torch.randn(batch, 9, 1, 64, generator=g).cuda()
        v = torch.full_like(k, 0.75)
        out = attention(q, k, v, length)
        torch.testing.assert_close(out, torch.full_like(out, 0.75), rtol=1e-5, atol=1e-6)
        # one sequence against the oracle
        qs, ks = q[7:8].cpu().numpy(), k[7:8].cpu().numpy()
        vs = torch.randn(1, 3, length, 64, generator=torch.Generator().manual_seed(batch + 1))
        out = attention(q[7:8].contiguous(), k[7:8].contiguous(), vs.cuda(), length)
        expected = o.gqa_decode_attention(qs, ks, vs.numpy(), None, 0.125, length)
        np.testing.assert_allclose(out.cpu().numpy(), expected, **TOL)


@pytest.mark.parametrize("batch,length,capacity", [(1, 1, 130), (1, 128, 128), (3, 777, 1000), (16, 1024, 1024),
                                                   (64, 4097, 4097), (2, 8192, 8192)])
def test_in_kernel_merge_matches_merge_kernel(batch, length, capacity):
    """The last-CTA merge (workspace with counters) is bitwise the merge
    kernel's result; repeated calls on one workspace (the counters rearm)
    and a CUDA-graph replay give the same bits."""
    from flux_b200 import _native
    lib = _native.load()
    q, k, v = (t.cuda() for t in _inputs(batch, length, capacity, seed=batch * 31 + length))
    two_launch = attention(q, k, v, length)
    one_launch = attention(q, k, v, length, fused=True)
    assert torch.equal(one_launch, two_launch)
    out = torch.empty(batch, 9, 1, 64, device="cuda")
    floats = lib.fx_gqa_decode_attention_workspace_floats(batch, 9, capacity, 64) + batch * 3
    ws = torch.zeros(floats, device="cuda")
    ln = torch.tensor(length, device="cuda")
    stream = torch.cuda.Stream()

    def call():
        _native.check(lib.fx_gqa_decode_attention_f32(
            q.data_ptr(), _native.int64_array(q.stride()), k.data_ptr(), _native.int64_array(k.stride()),
            v.data_ptr(), _native.int64_array(v.stride()), None, None, None, ln.data_ptr(), out.data_ptr(),
            ws.data_ptr(), floats, 0.125, batch, 9, 3, capacity, 64, stream.cuda_stream))

    with torch.cuda.stream(stream):
        for _ in range(3):
            call()
        stream.synchronize()
        assert torch.equal(out, two_launch)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            call()
        for _ in range(3):
            out.zero_()
            graph.replay()
        stream.synchronize()
    assert torch.equal(out, two_launch)
    counters = ws[-batch * 3:].view(torch.int32)
    assert int(counters.abs().sum()) == 0

