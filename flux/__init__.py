"""Source-compatible ``flux`` import paths over flux_b200.

Code written against the reference package imports from ``flux.ops``,
``flux.ops.native_*``, ``flux.model.smollm2_flux``, ``flux.model.smollm2`` and
``flux.runtime``; every one of those module paths is registered here as an
alias of the flux_b200 module that implements it (``_ALIASES``), so an
unmodified caller runs on the B200 library.

``torch.classes.flux.NativeSmolLM2Decode`` and ``NativeSmolLM2Prefill`` are
registered (``libfluxb200_torch.so``) with the reference's constructor
argument lists and methods, for code that builds the runtime objects directly.

Differences a caller can see:
* the plain operator functions the reference ships as PyTorch formulas
  (``flux.ops.rms_norm``, ``residual_rmsnorm``, ``rope``, ``softmax``,
  ``packed_swiglu``, ``attention_score_softmax``, ``gqa_decode_attention``)
  keep their signatures but run the native kernels, so they take CUDA tensors
  (CPU tensors are refused, as every flux_b200 operator refuses them);
* ``flux.model.smollm2.load_model`` / ``load_tokenizer`` load the pinned Hub
  checkpoint through transformers, which needs it in the local cache or
  network access.
"""

from __future__ import annotations

import sys
import types

from flux_b200 import _native
from flux_b200 import integration as _integration
from flux_b200 import operators as _operators
from flux_b200 import runtime as _runtime

# torch.classes.flux.NativeSmolLM2Decode / NativeSmolLM2Prefill, the custom
# classes the reference's runtime module constructs (registered when the
# library is built; the probes in flux.runtime load it as well).
_native.load_torch_classes()

# The reference's plain (PyTorch-formula) operators, same signatures, on the
# native kernels (flux/ops/{rmsnorm,residual_rmsnorm,rope,softmax,
# packed_swiglu,attention_score_softmax,gqa_decode_attention}.py).
_PLAIN_OPERATORS = {
    "rmsnorm": ("rms_norm", _operators.rms_norm_native),
    "residual_rmsnorm": ("residual_rmsnorm", _operators.residual_rmsnorm_native),
    "rope": ("rope", _operators.rope_native),
    "softmax": ("softmax", _operators.softmax_native),
    "packed_swiglu": ("packed_swiglu", _operators.packed_swiglu_native),
    "attention_score_softmax": ("attention_score_softmax", _operators.attention_score_softmax_native),
    "gqa_decode_attention": ("gqa_decode_attention", _operators.gqa_decode_attention_native),
}

# flux.ops.native_<name> modules and the names each exports
# (flux/ops/native_*.py in the reference).
_NATIVE_MODULES = {
    "native_rmsnorm": ("native_rmsnorm_is_available", "native_residual_rmsnorm_is_available",
                       "native_rmsnorm_load_error", "rms_norm_native", "rms_norm_native_out",
                       "residual_rmsnorm_native", "residual_rmsnorm_native_out"),
    "native_softmax": ("native_softmax_is_available", "native_softmax_load_error", "softmax_native"),
    "native_attention_score_softmax": ("native_attention_score_softmax_is_available",
                                       "attention_score_softmax_native"),
    "native_rope": ("native_rope_is_available", "native_rope_load_error", "rope_native"),
    "native_packed_swiglu": ("native_packed_swiglu_is_available", "packed_swiglu_native",
                             "packed_swiglu_native_out"),
    "native_packed_gate_up_gemv": ("native_packed_gate_up_gemv_is_available", "packed_gate_up_swiglu_native_out"),
    "native_packed_qkv_rope_cache": ("native_packed_qkv_rope_cache_is_available",
                                     "native_packed_qkv_rope_cache_load_error", "packed_qkv_rope_cache_native",
                                     "packed_qkv_rope_cache_native_out"),
    "native_gqa_decode_attention": ("native_gqa_decode_attention_is_available", "gqa_decode_attention_native",
                                    "gqa_decode_attention_native_out"),
    "native_cublaslt_linear": ("native_cublaslt_linear_is_available", "CublasLtAlgorithm", "cublaslt_algorithms",
                               "cublaslt_linear_config_out", "cublaslt_linear_out"),
}


def _try_load_native_library() -> bool:
    """Load ``libfluxb200.so`` if it is not loaded yet; True when it is."""
    return _operators._available()


def _operator_is_registered(name: str) -> bool:
    """Whether ``torch.ops.flux.<name>`` exists (the schemas register on import)."""
    import torch
    return hasattr(torch.ops.flux, name)


def _module(name: str, doc: str, names: dict) -> types.ModuleType:
    module = types.ModuleType(name, doc)
    module.__dict__.update(names)
    module.__all__ = sorted(k for k in names if not k.startswith("_"))
    sys.modules[name] = module
    return module


def _install() -> None:
    ops_names = {}
    for submodule, (public, function) in _PLAIN_OPERATORS.items():
        _module(f"flux.ops.{submodule}", f"flux.ops.{submodule} on flux_b200", {public: function})
        ops_names[public] = function
    for submodule, names in _NATIVE_MODULES.items():
        exported = {n: getattr(_operators, n) for n in names}
        if submodule == "native_rmsnorm":
            exported.update(_try_load_native_library=_try_load_native_library,
                            _operator_is_registered=_operator_is_registered)
        _module(f"flux.ops.{submodule}", f"flux.ops.{submodule} on flux_b200", exported)
        ops_names.update({n: v for n, v in exported.items() if not n.startswith("_")})
    ops = _module("flux.ops", "Flux operator interfaces on flux_b200.", ops_names)
    ops.__path__ = []  # a package, so ``import flux.ops.native_rope`` resolves through sys.modules

    smollm2_flux = sys.modules.setdefault("flux.model.smollm2_flux", _integration)
    smollm2 = _module("flux.model.smollm2", "SmolLM2 Hub checkpoint helpers (pinned revision).", {
        "MODEL_ID": "HuggingFaceTB/SmolLM2-135M",
        "MODEL_REVISION": "93efa2f097d58c2a74874c7e644dbc9b0cee75a2",
        "load_model": _load_model, "load_tokenizer": _load_tokenizer})
    model = _module("flux.model", "SmolLM2 model utilities on flux_b200.", {
        name: getattr(_integration, name) for name in (
            "FINAL_FLUX_OPERATOR_CATEGORIES", "FLUX_PACKED_MLP_CATEGORY", "FLUX_PACKED_QKV_CATEGORY",
            "FLUX_PACKED_SWIGLU_CATEGORY", "FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY", "FluxPackedLlamaMLP",
            "enable_flux_ops", "flux_operator_counts")})
    model.__path__ = []
    model.smollm2_flux, model.smollm2 = smollm2_flux, smollm2
    sys.modules.setdefault("flux.runtime.native_smollm2", _runtime)
    runtime = _module("flux.runtime", "Native SmolLM2 runtimes on flux_b200.", {
        name: getattr(_runtime, name) for name in (
            "NativeDecodeRuntimeMemory", "NativePrefillRuntimeMemory", "NativeSmolLM2Decode", "NativeSmolLM2Prefill",
            "native_smollm2_greedy_generate", "native_smollm2_prefill_is_available",
            "native_smollm2_runtime_is_available")})
    runtime.__path__ = []
    runtime.native_smollm2 = sys.modules["flux.runtime.native_smollm2"]
    this = sys.modules[__name__]
    this.ops, this.model, this.runtime = ops, model, runtime
    for submodule in (*_PLAIN_OPERATORS, *_NATIVE_MODULES):
        # as in the reference package, a function named like its module wins
        # (``flux.ops.rope`` is the function, ``flux.ops.rmsnorm`` the module)
        if submodule not in ops_names:
            setattr(ops, submodule, sys.modules[f"flux.ops.{submodule}"])


def _load_model(device="cpu"):
    """The FP32 SmolLM2-135M checkpoint at the pinned revision, eager attention, eval mode."""
    import torch
    from transformers import AutoModelForCausalLM
    model = AutoModelForCausalLM.from_pretrained("HuggingFaceTB/SmolLM2-135M",
                                                 revision="93efa2f097d58c2a74874c7e644dbc9b0cee75a2",
                                                 torch_dtype=torch.float32, attn_implementation="eager")
    return model.to(device).eval()


def _load_tokenizer():
    from transformers import AutoTokenizer
    return AutoTokenizer.from_pretrained("HuggingFaceTB/SmolLM2-135M",
                                         revision="93efa2f097d58c2a74874c7e644dbc9b0cee75a2")


_install()
