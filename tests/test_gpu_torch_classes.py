"""GPU: ``torch.classes.flux.NativeSmolLM2Decode`` / ``NativeSmolLM2Prefill``
built with the reference's argument lists (``flux/runtime/native_smollm2.py:145-160,
362-381``) run the same native runtime as ``flux_b200.runtime``: bitwise the
same logits and tokens, views that outlive their object, reset."""

from __future__ import annotations

import copy
import gc

import pytest
import torch

from oracle import hf_reference as hf
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(smollm2_model):
    from flux_b200 import _native
    from flux_b200.integration import FINAL_FLUX_OPERATOR_CATEGORIES, enable_flux_ops
    assert _native.load_torch_classes(), "libfluxb200_torch.so must be built and load"
    return enable_flux_ops(copy.deepcopy(smollm2_model).to("cuda"), operators=FINAL_FLUX_OPERATOR_CATEGORIES)


def _weights(model):
    layers = list(model.model.layers)
    return ([layer.input_layernorm.weight for layer in layers], [layer.self_attn.packed_qkv.weight for layer in layers],
            [layer.self_attn.o_proj.weight for layer in layers],
            [layer.post_attention_layernorm.weight for layer in layers],
            [layer.mlp.gate_up_proj.weight for layer in layers], [layer.mlp.down_proj.weight for layer in layers])


def _scalars(model):
    layers = list(model.model.layers)
    return ([float(layer.input_layernorm.variance_epsilon) for layer in layers],
            [float(layer.self_attn.scaling) for layer in layers])


def test_decode_class_matches_runtime(model):
    from flux_b200.runtime import NativeSmolLM2Decode, _rope_tables
    position, capacity = 300, 312
    keys, values = hf.synthetic_cache(hf.smollm2_config(), position, seed=41, std=0.5)
    keys, values = [k.cuda() for k in keys], [v.cuda() for v in values]
    token = torch.tensor([[1234]], device="cuda")
    cos, sin = _rope_tables(model, capacity, token.device)
    eps, scales = _scalars(model)
    native = torch.classes.flux.NativeSmolLM2Decode(
        token, model.model.embed_tokens.weight, *_weights(model), model.model.norm.weight, model.lm_head.weight, cos,
        sin, keys, values, capacity, position, eps, scales)
    runtime = NativeSmolLM2Decode.capture_from_state(model, token, keys, values, cache_position=position,
                                                     cache_capacity=capacity)
    assert native.capacity() == capacity and native.layer_count() == 30 and native.vocabulary_size() == 49152
    assert len(native.addresses()) == 13 and native.position() == position
    first = None
    for t in gi.uniform_prompt(4, seed=41)[0].tolist():
        a = native.replay(torch.tensor([[t]], device="cuda")).clone()
        b = runtime.replay(torch.tensor([[t]], device="cuda")).clone()
        assert torch.equal(a, b)
        first = a if first is None else first
    assert native.position() == position + 4 and native.replay_count() == 4
    assert torch.equal(native.key_cache(), runtime.key_cache)
    native.reset(token, keys, values, position)
    assert native.position() == position
    again = native.replay(torch.tensor([[gi.uniform_prompt(4, seed=41)[0, 0].item()]], device="cuda"))
    assert torch.equal(again, first)
    logits = native.logits()
    del native
    gc.collect()
    torch.cuda.synchronize()
    assert torch.equal(logits, again)  # the view keeps the runtime's memory alive


def test_prefill_class_matches_runtime(model):
    from flux_b200.runtime import NativeSmolLM2Prefill, _rope_tables
    prompt = gi.uniform_prompt(77, seed=5).cuda()
    new_tokens = 6
    capacity = 77 + new_tokens
    cos, sin = _rope_tables(model, capacity, prompt.device)
    eps, scales = _scalars(model)
    native = torch.classes.flux.NativeSmolLM2Prefill(
        prompt, model.model.embed_tokens.weight, *_weights(model), model.model.norm.weight, model.lm_head.weight, cos,
        sin, capacity, eps, scales)
    runtime = NativeSmolLM2Prefill.capture(model, prompt, max_decode_steps=new_tokens)
    assert torch.equal(native.logits(), runtime.logits)
    assert native.prompt_length() == 77 and native.capacity() == capacity
    assert torch.equal(native.generate_greedy(new_tokens), runtime.generate_greedy(new_tokens))
    assert torch.equal(native.key_cache()[:, :, :, :77], runtime.key_cache[:, :, :, :77])
    # a second prefill of the same prompt restarts the generation
    native.prefill(prompt)
    assert torch.equal(native.logits(), runtime.logits)
    assert native.cache_bytes() == 2 * 30 * 3 * capacity * 64 * 4
