"""The allocation-free GQA decode attention entry point.

Callers that cannot allocate device memory -- a host that owns the whole device
budget through its own pool, or a plugin host that passes tensors but no
allocator -- call ``fx_gqa_decode_attention_static_scratch_f32``, which keeps
its split-K partials in a static device array instead of a caller workspace.
This file checks, through the C ABI, that two calls in a row give the same
output as the allocating entry point ``fx_gqa_decode_attention_f32`` within the
tolerance the other attention tests use, and that a problem too large for the
static array is refused.  It is named so that pytest collects it last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu


def _call(lib, native, q, k, v, mask, length, out, *, workspace=None):
    if mask is None:
        mask_args = (None, None, None)
    else:
        mask_args = (mask.data_ptr(), native.int64_array(mask.shape), native.int64_array(mask.stride()))
    args = (q.data_ptr(), native.int64_array(q.stride()), k.data_ptr(), native.int64_array(k.stride()),
            v.data_ptr(), native.int64_array(v.stride()), *mask_args, length.data_ptr(), out.data_ptr())
    sizes = (0.125, q.shape[0], q.shape[1], k.shape[1], k.shape[2], q.shape[3],
             torch.cuda.current_stream().cuda_stream)
    if workspace is None:
        return lib.fx_gqa_decode_attention_static_scratch_f32(*args, *sizes)
    return lib.fx_gqa_decode_attention_f32(*args, workspace.data_ptr(), workspace.numel(), *sizes)


@pytest.mark.parametrize("masked", [True, False], ids=["masked", "compact"])
def test_static_scratch_entry_matches_the_allocating_entry(masked, ops_golden):
    """Masked calls take the generic partial + merge kernels; unmasked calls
    over contiguous SmolLM2-shaped caches take the TMA-staged compact chunk
    kernel, here with the static array as its partials (the allocating entry
    gets a workspace of exactly the partials, so both run the chunk kernel
    plus the separate merge kernel)."""
    from flux_b200 import _native
    lib = _native.load()
    q, k, v, mask = (t.cuda() for t in gi.gqa_inputs(1024))
    if not masked:
        mask = None
    for length_value in (777, 1024):  # two calls in a row, different valid lengths
        length = torch.tensor(length_value, device="cuda")
        floats = lib.fx_gqa_decode_attention_workspace_floats(1, 9, 1024, 64)
        workspace = torch.empty(floats, device="cuda")
        expected = torch.empty_like(q)
        _native.check(_call(lib, _native, q, k, v, mask, length, expected, workspace=workspace))
        actual = torch.full_like(q, float("nan"))
        _native.check(_call(lib, _native, q, k, v, mask, length, actual))
        torch.cuda.synchronize()
        np.testing.assert_allclose(actual.cpu().numpy(), expected.cpu().numpy(), rtol=2e-5, atol=1e-6)
        if masked and length_value == 777:
            # the reference's own operator oracle on the same seeded inputs
            np.testing.assert_allclose(actual.cpu().numpy(), ops_golden["gqa1024_len777"], rtol=2e-5, atol=1e-6)


def test_static_scratch_entry_rejects_sizes_beyond_its_array():
    from flux_b200 import _native
    lib = _native.load()
    limit = lib.fx_gqa_decode_attention_static_scratch_floats()
    assert limit == 262144
    # 9 heads x ceil(cap / 128) chunks x 66 floats just above the limit.
    capacity = 128 * (limit // (9 * 66) + 1)
    q = torch.zeros((1, 9, 1, 64), device="cuda")
    k = torch.zeros((1, 3, capacity, 64), device="cuda")
    mask = torch.zeros((1, 1, 1, capacity), device="cuda")
    length = torch.tensor(capacity, device="cuda")
    out = torch.empty_like(q)
    status = _call(lib, _native, q, k, k, mask, length, out)
    assert status == _native.FX_ERR_INVALID
    assert b"static array" in lib.fx_last_error()
