"""GPU parity of the torch.ops.flux.* kernels against the reference goldens
and the numpy oracle (behaviour spec: the reference's ``tests/test_ops.py``
and ``csrc/tests/test_decode_ops.cu``)."""

from __future__ import annotations

import ctypes
import hashlib

import numpy as np
import pytest
import torch
import torch.nn.functional as F
from torch._subclasses.fake_tensor import FakeTensor, FakeTensorMode

from oracle import smollm2 as o
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu

EPS = gi.EPSILON


@pytest.fixture(scope="module", autouse=True)
def _native():
    import flux_b200
    assert flux_b200.is_available(), "libfluxb200.so must be built and loadable on a GPU box"
    yield


def cuda(t):
    return t.to("cuda")


def np32(t):
    return t.detach().cpu().numpy().astype(np.float32)


def test_rmsnorm_residual_rmsnorm(ops_golden):
    from flux_b200 import operators as ops
    x = cuda(gi.wave((2, 7, 576)))
    w = torch.linspace(0.25, 1.75, 576, device="cuda")
    out = ops.rms_norm_native(x, w, EPS)
    np.testing.assert_allclose(np32(out), ops_golden["rmsnorm_out"], rtol=1e-5, atol=2e-6)
    # non-contiguous input and weight (tests/test_ops.py:104-112)
    xt = cuda(gi.wave((2, 576, 7))).transpose(1, 2)
    wt = torch.linspace(0.25, 1.75, 1152, device="cuda")[::2]
    np.testing.assert_allclose(np32(ops.rms_norm_native(xt, wt, EPS)), o.rms_norm(np32(xt), np32(wt), EPS),
                               rtol=1e-5, atol=2e-6)
    hidden, residual = cuda(gi.wave((2, 7, 576))), cuda(gi.wave((2, 7, 576)) * 0.25)
    before = hidden.clone()
    norm, res = ops.residual_rmsnorm_native(hidden, residual, w, EPS)
    assert torch.equal(hidden, before)
    np.testing.assert_array_equal(np32(res), ops_golden["residual_rmsnorm_residual"])
    np.testing.assert_allclose(np32(norm), ops_golden["residual_rmsnorm_norm"], rtol=1e-5, atol=2e-6)
    norm_out, res_out = torch.full_like(hidden, 41.0), torch.full_like(hidden, -41.0)
    returned = ops.residual_rmsnorm_native_out(hidden, residual, w, EPS, norm_out, res_out)
    assert returned[0] is norm_out and returned[1] is res_out
    np.testing.assert_array_equal(np32(res_out), ops_golden["residual_rmsnorm_residual"])
    output = torch.full_like(x, 73.0)
    assert ops.rms_norm_native_out(x, w, EPS, output) is output
    with pytest.raises(RuntimeError, match="must not alias"):
        ops.rms_norm_native_out(x, w, EPS, x)


@pytest.mark.parametrize("hidden_size", [1, 7, 63, 575, 577, 2048])
def test_residual_rmsnorm_arbitrary_widths(hidden_size):
    from flux_b200 import operators as ops
    torch.manual_seed(hidden_size)
    h, r = torch.randn(2, 3, hidden_size), torch.randn(2, 3, hidden_size)
    w = torch.linspace(0.25, 1.75, hidden_size)
    norm, res = ops.residual_rmsnorm_native(cuda(h), cuda(r), cuda(w), EPS)
    en, er = o.residual_rmsnorm(h.numpy(), r.numpy(), w.numpy(), EPS)
    np.testing.assert_array_equal(np32(res), er)
    np.testing.assert_allclose(np32(norm), en, rtol=1e-5, atol=1e-6)


def test_swiglu_softmax_attention_softmax(ops_golden):
    from flux_b200 import operators as ops
    packed = cuda(gi.wave((1, 7, 3072)))
    np.testing.assert_allclose(np32(ops.packed_swiglu_native(packed)), ops_golden["packed_swiglu_out"],
                               rtol=2e-6, atol=2e-6)
    out = torch.full((1, 7, 1536), 59.0, device="cuda")
    assert ops.packed_swiglu_native_out(packed, out) is out
    np.testing.assert_allclose(np32(ops.softmax_native(cuda(3.0 * gi.wave((5, 129))))), ops_golden["softmax_out"],
                               rtol=1e-5, atol=5e-7)
    scores, mask = cuda(3.0 * gi.wave((2, 3, 5, 17))), cuda(gi.wave((2, 1, 5, 17)) * 0.25)
    np.testing.assert_allclose(np32(ops.attention_score_softmax_native(scores, mask, 17 ** -0.5)),
                               ops_golden["attention_score_softmax_out"], rtol=1e-5, atol=5e-7)


def test_rope_bit_exact_against_transformers(ops_golden):
    from flux_b200 import operators as ops
    for b, s, off in gi.ROPE_CASES:
        q, k, cos, sin = (cuda(t) for t in gi.rope_inputs(b, s, off))
        rq, rk = ops.rope_native(q, k, cos, sin)
        assert rq.is_contiguous() and rk.is_contiguous()
        sha = [hashlib.sha256(np32(t).tobytes()).hexdigest() for t in (rq, rk)]
        assert sha == list(ops_golden[f"rope_{b}_{s}_{off}_sha"]), (b, s, off)


def test_packed_qkv_rope_cache_exact(ops_golden):
    from flux_b200 import operators as ops
    packed, cos, sin, keys, values, length = (cuda(t) for t in gi.qkv_inputs())
    keys_before, values_before = keys.clone(), values.clone()
    query = ops.packed_qkv_rope_cache_native(packed, cos, sin, keys, values, length)
    assert query.shape == (1, 9, 1, 64) and query.is_contiguous()
    assert int(length.item()) == 12
    np.testing.assert_array_equal(np32(query), ops_golden["qkv_query"])
    np.testing.assert_array_equal(np32(keys[:, :, 11:12]), ops_golden["qkv_key_row"])
    np.testing.assert_array_equal(np32(values[:, :, 11:12]), ops_golden["qkv_value_row"])
    others = [i for i in range(17) if i != 11]
    assert torch.equal(keys[:, :, others], keys_before[:, :, others])
    assert torch.equal(values[:, :, others], values_before[:, :, others])
    # out variant leaves the length alone? No: both forms advance it (same kernel contract).
    packed, cos, sin, keys, values, length = (cuda(t) for t in gi.qkv_inputs())
    output = torch.full((1, 9, 1, 64), 83.0, device="cuda")
    assert ops.packed_qkv_rope_cache_native_out(packed, cos, sin, keys, values, length, output) is output
    np.testing.assert_array_equal(np32(output), ops_golden["qkv_query"])
    with pytest.raises(RuntimeError, match=r"\[1, 1, 960\]"):
        ops.packed_qkv_rope_cache_native(packed[..., :-1], cos, sin, keys, values, length)
    with pytest.raises(RuntimeError, match="float32"):
        ops.packed_qkv_rope_cache_native(packed.double(), cos, sin, keys, values, length)


def test_gqa_decode_attention_goldens(ops_golden):
    from flux_b200 import operators as ops
    q, k, v, m = (cuda(t) for t in gi.gqa_inputs(73))
    length = torch.tensor(41, device="cuda")
    out = ops.gqa_decode_attention_native(q, k, v, m, 0.125, length)
    assert out.shape == q.shape and out.is_contiguous()
    np.testing.assert_allclose(np32(out), ops_golden["gqa73_masked"], rtol=2e-5, atol=1e-6)
    np.testing.assert_allclose(np32(ops.gqa_decode_attention_native(q, k, v, None, 0.125, length)),
                               ops_golden["gqa73_unmasked"], rtol=2e-5, atol=1e-6)
    q, k, v, m = (cuda(t) for t in gi.gqa_inputs(1024))
    output = torch.full_like(q, 67.0)
    workspace = torch.empty((1, 9, 8, 66), device="cuda")
    assert ops.gqa_decode_attention_native_out(q, k, v, m, 0.125, torch.tensor(777, device="cuda"), output,
                                               workspace) is output
    np.testing.assert_allclose(np32(output), ops_golden["gqa1024_len777"], rtol=2e-5, atol=1e-6)
    for (b, hq, hkv, d), (cap, n) in gi.GQA_PIN_CASES:
        if b != 1:
            continue
        q, k, v, m = (cuda(t) for t in gi.gqa_pin_inputs(b, hq, hkv, d, cap))
        out = ops.gqa_decode_attention_native(q, k, v, m, d ** -0.5, torch.tensor(n, device="cuda"))
        np.testing.assert_allclose(np32(out), ops_golden[f"gqa_pin_{b}_{hq}_{hkv}_{d}_{cap}_{n}"], rtol=1e-5,
                                   atol=5e-7)


def test_gqa_c_abi_batched_and_small_heads(ops_golden):
    """The C-ABI kernel itself serves any batch / head grouping; the op keeps the
    reference's batch-1 contract, so batched pins go through the C ABI."""
    from flux_b200 import _native
    lib = _native.load()
    for (b, hq, hkv, d), (cap, n) in gi.GQA_PIN_CASES:
        q, k, v, m = (cuda(t) for t in gi.gqa_pin_inputs(b, hq, hkv, d, cap))
        length = torch.tensor(n, device="cuda")
        out = torch.empty_like(q)
        floats = lib.fx_gqa_decode_attention_workspace_floats(b, hq, cap, d)
        ws = torch.empty(floats, device="cuda")
        _native.check(lib.fx_gqa_decode_attention_f32(
            q.data_ptr(), _native.int64_array(q.stride()), k.data_ptr(), _native.int64_array(k.stride()),
            v.data_ptr(), _native.int64_array(v.stride()), m.data_ptr(), _native.int64_array(m.shape),
            _native.int64_array(m.stride()), length.data_ptr(), out.data_ptr(), ws.data_ptr(), floats,
            d ** -0.5, b, hq, hkv, cap, d, torch.cuda.current_stream().cuda_stream))
        np.testing.assert_allclose(np32(out), ops_golden[f"gqa_pin_{b}_{hq}_{hkv}_{d}_{cap}_{n}"], rtol=1e-5,
                                   atol=5e-7)


@pytest.mark.parametrize("cap,length", [(8192, 8192), (8320, 8300), (257, 193)])
def test_gqa_long_context_vs_oracle(cap, length):
    """``csrc/tests/test_decode_ops.cu:158-243`` sizes (+ the lifted 8320 cap)."""
    from flux_b200 import operators as ops
    g = torch.Generator().manual_seed(cap)
    q = torch.randn((1, 9, 1, 64), generator=g)
    k = torch.randn((1, 3, cap, 64), generator=g)
    v = torch.randn((1, 3, cap, 64), generator=g)
    out = ops.gqa_decode_attention_native(cuda(q), cuda(k), cuda(v), None, 0.125, torch.tensor(length, device="cuda"))
    expected = o.gqa_decode_attention(q.numpy(), k.numpy(), v.numpy(), None, 0.125, length)
    np.testing.assert_allclose(np32(out), expected, rtol=3e-4, atol=3e-5)


def test_gqa_zero_query_gives_mean_value():
    from flux_b200 import operators as ops
    v = torch.randn((1, 3, 1000, 64), generator=torch.Generator().manual_seed(9))
    out = ops.gqa_decode_attention_native(torch.zeros((1, 9, 1, 64), device="cuda"), cuda(v), cuda(v), None, 0.125)
    expected = np.repeat(v[0].mean(dim=1).numpy(), 3, axis=0)
    np.testing.assert_allclose(np32(out)[0, :, 0], expected, rtol=1e-5, atol=1e-6)


def test_gqa_error_contract():
    from flux_b200 import operators as ops
    q, k, v, m = (cuda(t) for t in gi.gqa_inputs(17))
    cases = (
        ((q.expand(2, -1, -1, -1), k.expand(2, -1, -1, -1), v.expand(2, -1, -1, -1), m.expand(2, -1, -1, -1),
          0.125, None), "batch size must be one"),
        ((q.half(), k, v, m, 0.125, None), "float32"),
        ((q, k, v, m[..., :-1], 0.125, None), "broadcastable"),
    )
    for args, message in cases:
        with pytest.raises(RuntimeError, match=message):
            ops.gqa_decode_attention_native(*args)
    with pytest.raises(RuntimeError, match="inference-only"):
        ops.gqa_decode_attention_native(q.clone().requires_grad_(), k, v, m, 0.125)
    with FakeTensorMode():
        fq = torch.empty((1, 9, 1, 64))
        fk = torch.empty((1, 3, 129, 64))
        out = ops.gqa_decode_attention_native(fq, fk, torch.empty_like(fk), torch.empty((1, 1, 1, 129)), 0.125,
                                              torch.empty((), dtype=torch.int64))
    assert isinstance(out, FakeTensor) and out.shape == fq.shape


def test_gate_up_swiglu(ops_golden):
    from flux_b200 import operators as ops
    x, w = (cuda(t) for t in gi.gate_up_inputs())
    out = torch.full((1, 1, 1536), float("nan"), device="cuda")
    assert ops.packed_gate_up_swiglu_native_out(x, w, out) is out
    np.testing.assert_allclose(np32(out), ops_golden["gate_up_out"], rtol=1e-4, atol=1e-3)
    for args, message in (((x[..., :-1], w, out), r"\[1, 1, 576\]"), ((x, w[:-1], out), r"\[3072, 576\]"),
                          ((x.double(), w, out), "float32"), ((x, w, out[..., :-1]), "output shape")):
        with pytest.raises(RuntimeError, match=message):
            ops.packed_gate_up_swiglu_native_out(*args)


def test_projection_linear():
    from flux_b200 import operators as ops
    g = torch.Generator().manual_seed(1536)
    x = torch.randn((1, 1, 576), generator=g)
    w = torch.randn((960, 576), generator=g)
    out = torch.full((1, 1, 960), float("nan"), device="cuda")
    ws = torch.empty(0, dtype=torch.uint8, device="cuda")
    algorithm = ops.cublaslt_algorithms(cuda(x), cuda(w), max_workspace_bytes=0)[0]
    assert ops.cublaslt_linear_config_out(cuda(x), cuda(w), out, ws, algorithm) is out
    np.testing.assert_allclose(np32(out), o.linear(x.numpy(), w.numpy()), rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("m,n,k", [(1, 49152, 576), (17, 960, 576), (130, 3072, 576), (257, 576, 1536), (9, 100, 7)])
def test_linear_c_abi_shapes(m, n, k):
    from flux_b200 import _native
    g = torch.Generator().manual_seed(m * 7 + n)
    x, w = torch.randn((m, k), generator=g), torch.randn((n, k), generator=g)
    xd, wd = cuda(x), cuda(w)  # keep the device copies alive until the kernel has run
    out = torch.empty((m, n), device="cuda")
    _native.check(_native.load().fx_linear_f32(xd.data_ptr(), wd.data_ptr(), out.data_ptr(), m, k, n,
                                               torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    np.testing.assert_allclose(np32(out), o.linear(x.numpy(), w.numpy()), rtol=1e-4, atol=2e-4)


def _argmax(logits: np.ndarray) -> int:
    from flux_b200 import _native
    lib = _native.load()
    dev = torch.from_numpy(logits).cuda()
    token = torch.full((1,), -7, dtype=torch.int64, device="cuda")
    _native.check(lib.fx_greedy_argmax_f32(dev.data_ptr(), dev.numel(), token.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream))
    return int(token.item())


def test_greedy_known_answers():
    """``csrc/tests/test_greedy_generation.cu:46-68`` plus NaN-as-max."""
    vocab = 49152
    logits = gi.lcg_values(vocab, 2000.0)
    assert _argmax(logits) == int(np.argmax(logits))
    logits = np.full(vocab, -5000.0, np.float32)
    logits[177] = logits[321] = -3.0
    assert _argmax(logits) == 177
    fmax = np.finfo(np.float32).max
    logits = np.full(vocab, -fmax, np.float32)
    logits[0] = fmax
    assert _argmax(logits) == 0
    logits[0], logits[-1] = -fmax, fmax
    assert _argmax(logits) == vocab - 1
    assert _argmax(np.full(vocab, -np.inf, np.float32)) == 0
    logits = np.zeros(vocab, np.float32)
    logits[[9000, 5]] = np.nan
    assert _argmax(logits) == 5


def test_greedy_state_update():
    """``csrc/tests/test_greedy_generation.cu:70-104``."""
    from flux_b200 import _native
    lib = _native.load()
    logits = torch.full((49152,), -10.0, device="cuda")
    logits[19] = logits[27] = 4.0
    token = torch.zeros(1, dtype=torch.int64, device="cuda")
    generated = torch.tensor([3, 7, -1, -1], dtype=torch.int64, device="cuda")
    step = torch.tensor([2], dtype=torch.int64, device="cuda")
    position = torch.tensor([8], dtype=torch.int64, device="cuda")
    length = torch.tensor([9], dtype=torch.int64, device="cuda")
    _native.check(lib.fx_greedy_argmax_update_f32(logits.data_ptr(), 49152, token.data_ptr(), generated.data_ptr(), 4,
                                                  step.data_ptr(), position.data_ptr(), length.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream))
    assert int(token.item()) == 19
    assert generated.tolist() == [3, 7, 19, -1]
    assert int(step.item()) == 3 and int(position.item()) == 9


def test_opcheck_schema_and_fake():
    from flux_b200 import operators as ops  # noqa: F401
    x = cuda(gi.wave((2, 7, 576)))
    w = torch.linspace(0.25, 1.75, 576, device="cuda")
    result = torch.library.opcheck(torch.ops.flux.rmsnorm.default, (x, w, EPS), rtol=1e-5, atol=2e-6)
    assert all(v == "SUCCESS" for v in result.values()), result
    out = torch.empty_like(x)
    result = torch.library.opcheck(torch.ops.flux.rmsnorm_out.default, (x, w, EPS, out),
                                   test_utils=("test_schema", "test_faketensor"))
    assert all(v == "SUCCESS" for v in result.values()), result
    q, k, v, m = (cuda(t) for t in gi.gqa_inputs(17))
    with torch.inference_mode():
        result = torch.library.opcheck(torch.ops.flux.gqa_decode_attention.default,
                                       (q, k, v, m, 0.125, torch.tensor(11, device="cuda")), rtol=2e-5, atol=1e-6)
    assert all(v == "SUCCESS" for v in result.values()), result


def test_c_abi_rejects_bad_arguments():
    from flux_b200 import _native
    lib = _native.load()
    status = lib.fx_rmsnorm_f32(None, None, None, 1, 576, 1e-5, None)
    assert status == _native.FX_ERR_INVALID
    assert b"null pointer" in lib.fx_last_error()
    x = torch.ones(576, device="cuda")
    status = lib.fx_rmsnorm_f32(x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 576, float("nan"), None)
    assert status == _native.FX_ERR_INVALID
