"""Out-of-bounds write checks without compute-sanitizer: every output of the
operator surface and of the tensor-core C-ABI entries is a view in the middle
of a larger buffer whose guard bands hold a NaN sentinel bit pattern; after
the call the guard bands must be bit-for-bit unchanged (and, for the caches,
every row except the written one).  Ragged sizes (widths that are not a
multiple of a warp or tile) are used where the contract allows them."""

from __future__ import annotations

import math

import pytest
import torch

from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu

SENTINEL = 0x7FC0DEAD  # a quiet-NaN bit pattern no kernel produces
GUARD = 4096           # floats on each side (16 KB, keeps 16-byte alignment)


class Guarded:
    """A contiguous float32 view of `shape` between two sentinel guard bands."""

    def __init__(self, shape, fill=None):
        self.n = math.prod(shape)
        self.buf = torch.full((GUARD + self.n + GUARD,), SENTINEL, dtype=torch.int32, device="cuda")
        self.view = self.buf[GUARD:GUARD + self.n].view(torch.float32).view(shape)
        if fill is not None:
            self.view.copy_(fill)

    def intact(self) -> bool:
        torch.cuda.synchronize()
        return bool((self.buf[:GUARD] == SENTINEL).all()) and bool((self.buf[GUARD + self.n:] == SENTINEL).all())


def cuda(t):
    return t.to("cuda")


@pytest.mark.parametrize("width", [1, 63, 577, 2048])
def test_norm_outputs_stay_in_bounds(width):
    from flux_b200 import operators as ops
    x, r = cuda(gi.wave((3, width))), cuda(gi.wave((3, width)) * 0.5)
    w = torch.linspace(0.5, 1.5, width, device="cuda")
    out = Guarded((3, width))
    ops.rms_norm_native_out(x, w, gi.EPSILON, out.view)
    assert out.intact()
    norm, res = Guarded((3, width)), Guarded((3, width))
    ops.residual_rmsnorm_native_out(x, r, w, gi.EPSILON, norm.view, res.view)
    assert norm.intact() and res.intact()
    assert torch.equal(res.view, x + r)


def test_swiglu_and_gate_up_outputs_stay_in_bounds():
    from flux_b200 import operators as ops
    packed = cuda(gi.wave((2, 3, 2 * 1536)))
    out = Guarded((2, 3, 1536))
    ops.packed_swiglu_native_out(packed, out.view)
    assert out.intact()
    x, w = (cuda(t) for t in gi.gate_up_inputs())
    out = Guarded((1, 1, 1536))
    ops.packed_gate_up_swiglu_native_out(x, w, out.view)
    assert out.intact()


def test_qkv_rope_cache_writes_only_its_row():
    from flux_b200 import operators as ops
    packed, cos, sin, keys, values, length = (cuda(t) for t in gi.qkv_inputs())
    k, v = Guarded(tuple(keys.shape), keys), Guarded(tuple(values.shape), values)
    query = Guarded((1, 9, 1, 64))
    pos = int(length.item())
    ops.packed_qkv_rope_cache_native_out(packed, cos, sin, k.view, v.view, length, query.view)
    assert k.intact() and v.intact() and query.intact()
    others = [i for i in range(keys.shape[2]) if i != pos]
    assert torch.equal(k.view[:, :, others], keys[:, :, others])
    assert torch.equal(v.view[:, :, others], values[:, :, others])


# (the _out form needs capacity > 512)
@pytest.mark.parametrize("capacity,length", [(513, 300), (1024, 777), (4097, 4097)])
def test_gqa_attention_output_and_workspace_stay_in_bounds(capacity, length):
    from flux_b200 import operators as ops
    q, k, v, m = (cuda(t) for t in gi.gqa_inputs(capacity))
    out = Guarded((1, 9, 1, 64))
    ws = Guarded((1, 9, (capacity + 127) // 128, 66))
    ops.gqa_decode_attention_native_out(q, k, v, m, 0.125, torch.tensor(length, device="cuda"), out.view, ws.view)
    assert out.intact() and ws.intact()
    # the unmasked fast path (TMA-staged compact kernel) as well
    out2 = Guarded((1, 9, 1, 64))
    ops.gqa_decode_attention_native_out(q, k, v, None, 0.125, torch.tensor(length, device="cuda"), out2.view, ws.view)
    assert out2.intact() and ws.intact()


@pytest.mark.parametrize("m,k,n", [(1, 576, 960), (5, 1536, 200), (130, 576, 3072), (257, 576, 49152 // 64)])
def test_linear_outputs_stay_in_bounds(m, k, n):
    """The tcgen05 3xTF32 projection (ragged M and N against its 128 x 64 /
    128 x 128 tiles) and the SIMT projection."""
    from flux_b200 import _native
    lib = _native.load()
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(m + n)
    x = cuda(torch.randn(m, k, generator=g))
    w = cuda(torch.randn(n, k, generator=g) * 0.02)
    hi, lo = Guarded((n, k)), Guarded((n, k))
    _native.check(lib.fx_tf32_split_f32(w.data_ptr(), hi.view.data_ptr(), lo.view.data_ptr(), w.numel(), stream))
    assert hi.intact() and lo.intact()
    out = Guarded((m, n))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _native.check(lib.fx_linear_3xtf32_f32(x.data_ptr(), hi.view.data_ptr(), lo.view.data_ptr(), None,
                                           out.view.data_ptr(), m, k, n, err.data_ptr(), stream))
    assert out.intact() and int(err.item()) == 0
    out2 = Guarded((m, n))
    _native.check(lib.fx_linear_f32(x.data_ptr(), w.data_ptr(), out2.view.data_ptr(), m, k, n, stream))
    assert out2.intact()
    torch.testing.assert_close(out.view, out2.view, rtol=1e-4, atol=1e-5)
