"""Source compatibility: every name the reference's own tests and benchmarks
import from ``flux.*`` (collected from ``tests/*.py`` and ``benchmarks/*.py``
of the reference) imports from the same path here and is the flux_b200
implementation."""

from __future__ import annotations

import importlib

import pytest

REFERENCE_IMPORTS = {
    "flux.model": ["smollm2", "smollm2_flux"],
    "flux.model.smollm2": ["MODEL_ID", "MODEL_REVISION", "load_model"],
    "flux.model.smollm2_flux": ["FINAL_FLUX_OPERATOR_CATEGORIES", "enable_flux_ops", "flux_operator_counts"],
    "flux.ops": [
        "attention_score_softmax_native", "cublaslt_algorithms", "cublaslt_linear_out", "gqa_decode_attention",
        "gqa_decode_attention_native", "gqa_decode_attention_native_out",
        "native_attention_score_softmax_is_available", "native_cublaslt_linear_is_available",
        "native_gqa_decode_attention_is_available", "native_packed_gate_up_gemv_is_available",
        "native_packed_qkv_rope_cache_is_available", "native_packed_swiglu_is_available",
        "native_residual_rmsnorm_is_available", "native_rmsnorm_is_available", "native_rmsnorm_load_error",
        "native_rope_is_available", "native_softmax_is_available", "packed_gate_up_swiglu_native_out",
        "packed_qkv_rope_cache_native", "packed_qkv_rope_cache_native_out", "packed_swiglu_native",
        "packed_swiglu_native_out", "residual_rmsnorm", "residual_rmsnorm_native", "residual_rmsnorm_native_out",
        "rms_norm", "rms_norm_native", "rms_norm_native_out", "rope", "rope_native", "softmax", "softmax_native",
        "CublasLtAlgorithm", "cublaslt_linear_config_out", "packed_swiglu", "attention_score_softmax"],
    "flux.ops.attention_score_softmax": ["attention_score_softmax"],
    "flux.ops.gqa_decode_attention": ["gqa_decode_attention"],
    "flux.ops.packed_swiglu": ["packed_swiglu"],
    "flux.ops.residual_rmsnorm": ["residual_rmsnorm"],
    "flux.ops.rmsnorm": ["rms_norm"],
    "flux.ops.rope": ["rope"],
    "flux.ops.softmax": ["softmax"],
    "flux.ops.native_rmsnorm": ["_operator_is_registered", "_try_load_native_library", "rms_norm_native",
                                "native_rmsnorm_is_available", "residual_rmsnorm_native_out"],
    "flux.ops.native_rope": ["rope_native", "native_rope_is_available", "native_rope_load_error"],
    "flux.ops.native_softmax": ["softmax_native", "native_softmax_is_available", "native_softmax_load_error"],
    "flux.ops.native_attention_score_softmax": ["attention_score_softmax_native",
                                                "native_attention_score_softmax_is_available"],
    "flux.ops.native_cublaslt_linear": ["CublasLtAlgorithm", "cublaslt_algorithms", "cublaslt_linear_config_out",
                                        "cublaslt_linear_out", "native_cublaslt_linear_is_available"],
    "flux.ops.native_gqa_decode_attention": ["gqa_decode_attention_native", "gqa_decode_attention_native_out",
                                             "native_gqa_decode_attention_is_available"],
    "flux.ops.native_packed_gate_up_gemv": ["packed_gate_up_swiglu_native_out",
                                            "native_packed_gate_up_gemv_is_available"],
    "flux.ops.native_packed_qkv_rope_cache": ["packed_qkv_rope_cache_native", "packed_qkv_rope_cache_native_out",
                                              "native_packed_qkv_rope_cache_is_available"],
    "flux.ops.native_packed_swiglu": ["packed_swiglu_native", "packed_swiglu_native_out",
                                      "native_packed_swiglu_is_available"],
    "flux.runtime": ["NativeSmolLM2Decode", "NativeSmolLM2Prefill", "native_smollm2_greedy_generate",
                     "native_smollm2_prefill_is_available", "native_smollm2_runtime_is_available",
                     "NativeDecodeRuntimeMemory", "NativePrefillRuntimeMemory"],
    "flux.runtime.native_smollm2": ["NativeSmolLM2Decode", "NativeSmolLM2Prefill", "native_smollm2_greedy_generate"],
}


@pytest.mark.parametrize("module", sorted(REFERENCE_IMPORTS))
def test_reference_import_paths_resolve(module):
    imported = importlib.import_module(module)
    for name in REFERENCE_IMPORTS[module]:
        assert hasattr(imported, name), f"{module}.{name}"


def test_reference_paths_are_the_flux_b200_implementations():
    from flux.model.smollm2_flux import enable_flux_ops
    from flux.ops import gqa_decode_attention, rms_norm
    from flux.ops.native_rmsnorm import _operator_is_registered, _try_load_native_library
    from flux.runtime import NativeSmolLM2Prefill

    from flux_b200 import integration, operators, runtime
    assert enable_flux_ops is integration.enable_flux_ops
    assert NativeSmolLM2Prefill is runtime.NativeSmolLM2Prefill
    assert rms_norm is operators.rms_norm_native
    assert gqa_decode_attention is operators.gqa_decode_attention_native
    assert _try_load_native_library() is True  # the in-tree library loads (no GPU call)
    assert _operator_is_registered("gqa_decode_attention")


def test_plain_operators_refuse_cpu_tensors():
    """The reference's plain operators are PyTorch formulas that run anywhere;
    here they are the native kernels, which refuse CPU tensors instead of
    computing on the host."""
    import torch

    from flux.ops import rms_norm
    with pytest.raises(RuntimeError):
        rms_norm(torch.ones(1, 1, 576), torch.ones(576), 1e-5)
