"""CPU-only checks of the host side: the C ABI library loads and exports every
declared entry point, the operator schemas and their argument contracts, and
the ``enable_flux_ops`` model transformation (with exact Python formulas in
place of the native kernels, as the reference's own ``python_flux_ops``
fixture does, ``tests/test_system.py:57-133``)."""

from __future__ import annotations

import copy
import re
from pathlib import Path

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensor, FakeTensorMode
from transformers import LlamaConfig, LlamaForCausalLM

from oracle import smollm2 as o

ROOT = Path(__file__).resolve().parents[1]
RTOL, ATOL = 2e-4, 2e-5
EPS = 1e-5


def declared_symbols() -> list[str]:
    text = (ROOT / "include" / "flux_b200.h").read_text()
    return sorted(set(re.findall(r"^FX_API[^(]*?\b(fx_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from flux_b200 import _native
    lib = _native.load()
    names = declared_symbols()
    assert len(names) >= 30
    for name in names:
        assert hasattr(lib, name), name
        assert name in _native.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.fx_version().startswith(b"flux_b200")


def test_registered_operator_schemas():
    import flux_b200  # noqa: F401
    for name in ("attention_score_softmax", "cublaslt_linear_config_out", "cublaslt_linear_out",
                 "gqa_decode_attention", "gqa_decode_attention_out", "packed_gate_up_swiglu_out",
                 "packed_qkv_rope_cache", "packed_qkv_rope_cache_out", "packed_swiglu", "packed_swiglu_out",
                 "residual_rmsnorm", "residual_rmsnorm_out", "rmsnorm", "rmsnorm_out", "rope", "softmax"):
        assert hasattr(torch.ops.flux, name), name


# The native-side names `flux/ops/__init__.py` exports (its plain-PyTorch
# functions stay with Flux); each must import from flux_b200.operators.
FLUX_OPS_NATIVE_NAMES = (
    "CublasLtAlgorithm", "attention_score_softmax_native", "cublaslt_algorithms", "cublaslt_linear_config_out",
    "cublaslt_linear_out", "gqa_decode_attention_native", "gqa_decode_attention_native_out",
    "native_attention_score_softmax_is_available", "native_cublaslt_linear_is_available",
    "native_gqa_decode_attention_is_available", "native_packed_gate_up_gemv_is_available",
    "native_packed_qkv_rope_cache_is_available", "native_packed_qkv_rope_cache_load_error",
    "native_packed_swiglu_is_available", "native_residual_rmsnorm_is_available", "native_rmsnorm_is_available",
    "native_rmsnorm_load_error", "native_rope_is_available", "native_rope_load_error",
    "native_softmax_is_available", "native_softmax_load_error", "packed_gate_up_swiglu_native_out",
    "packed_qkv_rope_cache_native", "packed_qkv_rope_cache_native_out", "packed_swiglu_native",
    "packed_swiglu_native_out", "residual_rmsnorm_native", "residual_rmsnorm_native_out", "rms_norm_native",
    "rms_norm_native_out", "rope_native", "softmax_native",
)


def test_python_entry_points_cover_flux_ops():
    from flux_b200 import operators
    missing = [name for name in FLUX_OPS_NATIVE_NAMES if not hasattr(operators, name)]
    assert not missing
    for name in FLUX_OPS_NATIVE_NAMES:
        if name.endswith("_is_available"):
            assert getattr(operators, name)() is True, name  # the library is built in-tree


def test_operator_error_contracts_on_cpu():
    """``tests/test_ops.py`` error cases; valid CPU inputs are rejected loudly."""
    from flux_b200 import operators as ops
    for args, message in (((torch.tensor(1.0), torch.ones(1), EPS), "at least one dimension"),
                          ((torch.ones(2, 3), torch.ones(2), EPS), "weight length"),
                          ((torch.ones(2, 3), torch.ones(3, dtype=torch.float64), EPS),
                           "weight must have dtype torch.float32"),
                          ((torch.ones(2, 3), torch.ones(3), 0.0), "epsilon must be a positive")):
        with pytest.raises(RuntimeError, match=message):
            ops.rms_norm_native(*args)
    with pytest.raises(RuntimeError, match="inference-only"):
        ops.rms_norm_native(torch.ones(2, 3, requires_grad=True), torch.ones(3), EPS)
    with pytest.raises(RuntimeError, match="no CPU implementation"):
        ops.rms_norm_native(torch.ones(2, 3), torch.ones(3), EPS)
    for args, message in (((torch.ones(2, 3), torch.ones(1, 3), torch.ones(3), EPS), "same shape"),
                          ((torch.ones(2, 3), torch.ones(2, 3), torch.ones(2), EPS), "weight length"),
                          ((torch.ones(2, 3, dtype=torch.float64), torch.ones(2, 3), torch.ones(3), EPS),
                           "hidden must have dtype torch.float32"),
                          ((torch.ones(2, 3), torch.ones(2, 3), torch.ones(3), float("inf")), "finite")):
        with pytest.raises(RuntimeError, match=message):
            ops.residual_rmsnorm_native(*args)
    for packed, message in ((torch.tensor(1.0), "at least one dimension"), (torch.ones(2, 3), "must be even"),
                            (torch.ones(2, 4, dtype=torch.float64), "dtype torch.float32")):
        with pytest.raises(RuntimeError, match=message):
            ops.packed_swiglu_native(packed)
    for x, message in ((torch.tensor(1.0), "at least one dimension"), (torch.empty(2, 0), "non-empty final dimension"),
                       (torch.ones(2, 3, dtype=torch.float16), "dtype torch.float32")):
        with pytest.raises(RuntimeError, match=message):
            ops.softmax_native(x)
    scores, mask = torch.ones((1, 2, 3, 4)), torch.zeros((1, 1, 3, 4))
    for s, m, scale, message in ((scores.reshape(2, 3, 4), mask, 0.5, "rank four"),
                                 (scores, torch.zeros((1, 1, 2, 4)), 0.5, "broadcastable"),
                                 (scores.half(), mask, 0.5, "scores must have dtype torch.float32"),
                                 (scores, mask, float("inf"), "finite FP32")):
        with pytest.raises(RuntimeError, match=message):
            ops.attention_score_softmax_native(s, m, scale)
    q = torch.randn(1, 9, 1, 64)
    k = torch.randn(1, 3, 17, 64)
    m = torch.zeros(1, 1, 1, 17)
    for args, message in (((q.expand(2, -1, -1, -1), k.expand(2, -1, -1, -1), k.expand(2, -1, -1, -1),
                            m.expand(2, -1, -1, -1), 0.125, None), "batch size must be one"),
                          ((q.half(), k, k, m, 0.125, None), "float32"),
                          ((q, k, k, m[..., :-1], 0.125, None), "broadcastable"),
                          ((q, k, k, m, 0.125, torch.tensor(18)), "within cache capacity")):
        with pytest.raises(RuntimeError, match=message):
            ops.gqa_decode_attention_native(*args)


def test_fake_tensor_contracts():
    from flux_b200 import operators as ops
    with FakeTensorMode():
        hidden = torch.empty((2, 7, 576))
        norm, residual = ops.residual_rmsnorm_native(hidden, torch.empty_like(hidden), torch.empty(576), EPS)
        swiglu = ops.packed_swiglu_native(torch.empty((2, 32, 3072)))
        soft = ops.attention_score_softmax_native(torch.empty((2, 9, 7, 129)), torch.empty((2, 1, 7, 129)), 0.125)
    assert isinstance(norm, FakeTensor) and norm is not residual and norm.shape == hidden.shape
    assert swiglu.shape == (2, 32, 1536)
    assert soft.shape == (2, 9, 7, 129)


# --------------------------------------------------- enable_flux_ops (host)


def _config(layers: int = 2) -> LlamaConfig:
    config = LlamaConfig(hidden_size=32, intermediate_size=64, num_hidden_layers=layers, num_attention_heads=4,
                         num_key_value_heads=2, head_dim=8, vocab_size=128, max_position_embeddings=64,
                         rms_norm_eps=1e-5, attention_bias=False, attention_dropout=0.0, mlp_bias=False)
    config._attn_implementation = "eager"
    return config


def _model(layers: int = 2) -> LlamaForCausalLM:
    torch.manual_seed(1234)
    return LlamaForCausalLM(_config(layers)).float().eval()


@pytest.fixture
def python_flux_ops(monkeypatch):
    """Exact Python formulas (numpy oracle) in place of the native kernels."""
    from flux_b200 import integration
    counts = dict(rmsnorm=0, residual_rmsnorm=0, attention_score_softmax=0, rope=0, gqa_decode_attention=0)
    for name in ("native_rmsnorm_is_available", "native_residual_rmsnorm_is_available",
                 "native_softmax_is_available", "native_rope_is_available", "native_packed_swiglu_is_available",
                 "native_packed_gate_up_gemv_is_available", "native_attention_score_softmax_is_available",
                 "native_gqa_decode_attention_is_available"):
        monkeypatch.setattr(integration, name, lambda: True)

    def t(a):
        return torch.from_numpy(a)

    def rmsnorm(x, w, eps):
        counts["rmsnorm"] += 1
        return t(o.rms_norm(x.numpy(), w.detach().numpy(), eps))

    def residual_rmsnorm(h, r, w, eps):
        counts["residual_rmsnorm"] += 1
        n, res = o.residual_rmsnorm(h.numpy(), r.numpy(), w.detach().numpy(), eps)
        return t(n), t(res)

    def attention_softmax(scores, mask, scale):
        counts["attention_score_softmax"] += 1
        return t(o.softmax(scores.numpy() * o.F32(scale) + mask.numpy()))

    def rope(q, k, cos, sin):
        counts["rope"] += 1
        c, s = cos.numpy()[:, None], sin.numpy()[:, None]
        return t(o.rope(q.numpy(), c, s)), t(o.rope(k.numpy(), c, s))

    def gqa(q, k, v, mask, scale, length):
        counts["gqa_decode_attention"] += 1
        n = None if length is None else int(length)
        return t(o.gqa_decode_attention(q.numpy(), k.numpy(), v.numpy(), None if mask is None else mask.numpy(),
                                        scale, n))

    monkeypatch.setattr(integration, "rms_norm_native", rmsnorm)
    monkeypatch.setattr(integration, "residual_rmsnorm_native", residual_rmsnorm)
    monkeypatch.setattr(integration, "attention_score_softmax_native", attention_softmax)
    monkeypatch.setattr(integration, "rope_native", rope)
    monkeypatch.setattr(integration, "gqa_decode_attention_native", gqa)
    monkeypatch.setattr(integration, "packed_swiglu_native", lambda p: t(o.packed_swiglu(p.numpy())))
    monkeypatch.setattr(integration, "softmax_native", lambda x: t(o.softmax(x.numpy())))
    return counts


def test_final_configuration_is_the_complete_set():
    from flux_b200 import integration
    assert integration.FINAL_FLUX_OPERATOR_CATEGORIES == {
        "rmsnorm", "residual_rmsnorm", "rope", "softmax", "mlp", "packed_swiglu", "qkv", "gqa_decode_attention",
        "packed_qkv_rope_cache", "cublaslt_projection", "fused_gate_up_swiglu"}


def test_packed_weights_keep_the_checkpoint_interface(tmp_path):
    from flux_b200 import integration
    reference = _model(2)
    expected = copy.deepcopy(reference.state_dict())
    packed = copy.deepcopy(reference)
    integration.enable_flux_ops(packed, operators=("qkv", "mlp"))
    assert not hasattr(packed.model.layers[0].self_attn, "q_proj")
    assert not hasattr(packed.model.layers[0].mlp, "gate_proj")
    assert set(packed.state_dict()) == set(expected)
    for name, value in expected.items():
        torch.testing.assert_close(packed.state_dict()[name], value, rtol=0, atol=0)
    packed.load_state_dict(expected, strict=True)
    packed.save_pretrained(tmp_path, safe_serialization=True)
    restored = LlamaForCausalLM.from_pretrained(tmp_path, local_files_only=True)
    for name, value in expected.items():
        torch.testing.assert_close(restored.state_dict()[name], value, rtol=0, atol=0)


def test_packed_projection_views_and_outputs():
    from flux_b200 import integration
    source = _model(1)
    attention_reference = copy.deepcopy(source.model.layers[0].self_attn)
    attention = integration.FluxLlamaAttention(source.model.layers[0].self_attn, use_rope=False, use_softmax=False,
                                               use_packed_qkv=True)
    hidden = torch.randn(1, 7, 32)
    with torch.inference_mode():
        q, k, v = attention.project_qkv(hidden)
        eq = attention_reference.q_proj(hidden).view(1, 7, 4, 8).transpose(1, 2)
    assert tuple(attention.packed_qkv.weight.shape) == (64, 32)
    torch.testing.assert_close(attention.packed_qkv.weight[:32], attention_reference.q_proj.weight)
    assert k.untyped_storage().data_ptr() == q.untyped_storage().data_ptr() == v.untyped_storage().data_ptr()
    torch.testing.assert_close(q, eq, rtol=2e-5, atol=2e-5)


def test_model_transformation_and_eager_equivalence(python_flux_ops):
    from flux_b200 import integration
    reference = _model(2)
    flux = copy.deepcopy(reference)
    original = flux.model.layers[0].input_layernorm.weight
    selected = integration.FLUX_OPERATOR_CATEGORIES | {"qkv", "mlp", "packed_swiglu"}
    returned = integration.enable_flux_ops(flux, operators=selected)
    ids = torch.tensor([[1, 17, 42, 9, 3]])
    with torch.inference_mode():
        expected = reference(input_ids=ids, use_cache=True)
        actual = flux(input_ids=ids, use_cache=True)
    assert returned is flux
    assert flux.model.layers[0].input_layernorm.weight is original
    assert flux._flux_operator_categories == tuple(sorted(selected))
    counts = integration.flux_operator_counts(flux)
    assert counts["decoder_layers"] == 2 and counts["packed_qkv_modules"] == counts["packed_mlp_modules"] == 2
    assert python_flux_ops["rmsnorm"] == 3
    assert python_flux_ops["residual_rmsnorm"] == 2
    assert python_flux_ops["attention_score_softmax"] == 2
    assert python_flux_ops["rope"] == 2
    torch.testing.assert_close(actual.logits, expected.logits, rtol=RTOL, atol=ATOL)
    for a, e in zip(actual.past_key_values.layers, expected.past_key_values.layers, strict=True):
        torch.testing.assert_close(a.keys, e.keys, rtol=RTOL, atol=ATOL)
        torch.testing.assert_close(a.values, e.values, rtol=RTOL, atol=ATOL)


def test_gqa_category_is_decode_only(python_flux_ops):
    from flux_b200 import integration
    reference = _model(2)
    flux = copy.deepcopy(reference)
    integration.enable_flux_ops(flux, operators=integration.FLUX_OPERATOR_CATEGORIES | {"gqa_decode_attention"})
    prompt, token = torch.tensor([[1, 17, 42, 9, 3]]), torch.tensor([[11]])
    with torch.inference_mode():
        expected_prefill = reference(prompt, use_cache=True)
        actual_prefill = flux(prompt, use_cache=True)
        assert python_flux_ops["gqa_decode_attention"] == 0
        expected = reference(token, past_key_values=expected_prefill.past_key_values, use_cache=True)
        actual = flux(token, past_key_values=actual_prefill.past_key_values, use_cache=True)
    assert flux._flux_gqa_decode_attention_enabled
    assert python_flux_ops["gqa_decode_attention"] == 2
    torch.testing.assert_close(actual_prefill.logits, expected_prefill.logits, rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(actual.logits, expected.logits, rtol=RTOL, atol=ATOL)


def test_enable_flux_ops_error_contract(python_flux_ops):
    from flux_b200 import integration
    with pytest.raises(ValueError, match="inference-only"):
        integration.enable_flux_ops(_model(1).train())
    with pytest.raises(TypeError, match="torch.float32"):
        integration.enable_flux_ops(_model(1).half())
    for operators in ((), ("unknown",)):
        with pytest.raises(ValueError, match="operator categor"):
            integration.enable_flux_ops(_model(1), operators=operators)
    for operators, message in ((("packed_swiglu",), "requires.*mlp"),
                               (("packed_qkv_rope_cache",), 'requires the "rope", "qkv", and'),
                               (("cublaslt_projection",), 'requires the "packed_qkv_rope_cache"'),
                               (("fused_gate_up_swiglu",), "requires.*mlp.*packed_swiglu")):
        with pytest.raises(ValueError, match=message):
            integration.enable_flux_ops(_model(1), operators=operators)
    model = _model(1)
    integration.enable_flux_ops(model)
    with pytest.raises(ValueError, match="already enabled"):
        integration.enable_flux_ops(model)


def test_missing_native_library_fails_loudly(monkeypatch, tmp_path):
    """Without the library the product raises instead of computing on the CPU."""
    from flux_b200 import _native
    monkeypatch.setattr(_native, "_LIB", None)
    with pytest.raises(_native.NativeLibraryUnavailable):
        _native.load(tmp_path / "missing.so")
