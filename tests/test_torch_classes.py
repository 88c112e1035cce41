"""``torch.classes.flux`` runtime classes (``flux_b200/csrc/torch_classes.cpp``):
registered with the constructor argument lists and method names of the
reference's custom classes (``csrc/native_decode_runtime/native_decode_runtime_torch.cpp:38-79``,
``csrc/native_prefill_runtime/native_prefill_runtime_torch.cpp:5-45``), and
refusing CPU tensors before touching a device."""

from __future__ import annotations

import pytest
import torch

from flux_b200 import _native

# Method names of the reference's classes, in registration order.
DECODE_METHODS = [
    "replay", "generate_greedy", "reset", "logits", "current_token", "generated_tokens", "device_generation_step",
    "key_cache", "value_cache", "device_position", "device_cache_length", "workspace", "addresses", "position",
    "cache_length", "capacity", "replay_count", "generation_step", "workspace_bytes", "stable_buffer_bytes",
    "vocabulary_size", "layer_count",
]
PREFILL_METHODS = [
    "prefill", "replay", "generate_greedy", "logits", "current_token", "generated_tokens", "device_generation_step",
    "final_hidden", "key_cache", "value_cache", "device_position", "device_cache_length", "addresses", "position",
    "cache_length", "prompt_length", "capacity", "replay_count", "generation_step", "workspace_bytes",
    "cache_bytes", "stable_buffer_bytes",
]
# Constructor argument types (after self).
DECODE_INIT = (["Tensor", "Tensor"] + ["List[Tensor]"] * 6 + ["Tensor"] * 4 + ["List[Tensor]"] * 2
               + ["int", "int", "List[float]", "List[float]"])
PREFILL_INIT = ["Tensor", "Tensor"] + ["List[Tensor]"] * 6 + ["Tensor"] * 4 + ["int", "List[float]", "List[float]"]

pytestmark = pytest.mark.skipif(not _native.TORCH_CLASSES_PATH.exists(),
                                reason="libfluxb200_torch.so is not built (python -m flux_b200.build)")


def _schemas(cls: str) -> dict[str, list]:
    out: dict[str, list] = {}
    for schema in torch._C._jit_get_custom_class_schemas():
        args = schema.arguments
        if args and str(args[0].type) == f"__torch__.torch.classes.flux.{cls}":
            out.setdefault(schema.name, []).append([str(a.type) for a in args[1:]])
    return out


def test_classes_registered_with_reference_surface():
    assert _native.load_torch_classes()
    for cls, methods, init in (("NativeSmolLM2Decode", DECODE_METHODS, DECODE_INIT),
                               ("NativeSmolLM2Prefill", PREFILL_METHODS, PREFILL_INIT)):
        schemas = _schemas(cls)
        assert set(methods) | {"__init__"} == set(schemas), cls
        assert schemas["__init__"] == [init], cls
        getattr(torch.classes.flux, cls)  # resolvable the way the reference resolves it


def test_reference_optional_token_and_reset_signatures():
    assert _native.load_torch_classes()
    decode = _schemas("NativeSmolLM2Decode")
    assert decode["replay"] == [["Optional[Tensor]"]]
    assert decode["reset"] == [["Tensor", "List[Tensor]", "List[Tensor]", "int"]]
    assert decode["generate_greedy"] == [["int"]]
    assert _schemas("NativeSmolLM2Prefill")["prefill"] == [["Tensor"]]


def test_cpu_tensors_refused_before_any_device_work():
    assert _native.load_torch_classes()
    f = torch.zeros
    layers = 30
    args = [f(1, 1, dtype=torch.long), f(8, 576), [f(576)] * layers, [f(960, 576)] * layers, [f(576, 576)] * layers,
            [f(576)] * layers, [f(3072, 576)] * layers, [f(576, 1536)] * layers, f(576), f(8, 576), f(16, 64),
            f(16, 64), [], [], 16, 0, [1e-5] * layers, [0.125] * layers]
    with pytest.raises(RuntimeError, match="flux native full decode: embedding weight must be a CUDA tensor"):
        torch.classes.flux.NativeSmolLM2Decode(*args)
    prefill_args = [f(1, 4, dtype=torch.long)] + args[1:12] + [16, [1e-5] * layers, [0.125] * layers]
    with pytest.raises(RuntimeError, match="flux native prefill: embedding weight must be a CUDA tensor"):
        torch.classes.flux.NativeSmolLM2Prefill(*prefill_args)


def test_flux_package_registers_the_classes():
    import flux  # noqa: F401  (registers at import)
    assert _schemas("NativeSmolLM2Decode") and _schemas("NativeSmolLM2Prefill")
