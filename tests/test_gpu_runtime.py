"""GPU parity of the native decode / prefill runtimes against the reference's
FP32 path (goldens) and the numpy oracle (behaviour spec: the reference's
``tests/test_system.py:318-497`` and ``csrc/tests/test_native_runtimes.cu``)."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from oracle import hf_reference as hf
from oracle import smollm2 as o
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-4, 2e-5  # tests/test_system.py:30-31
LOGIT_TOL = 1e-4         # the 1e-4 abs / rel logits bar for the benchmark geometry


def np32(t):
    return t.detach().reshape(-1).cpu().numpy().astype(np.float32)


def flux_model(cpu_model):
    from flux_b200.integration import FINAL_FLUX_OPERATOR_CATEGORIES, enable_flux_ops
    model = copy.deepcopy(cpu_model).to("cuda")
    return enable_flux_ops(model, operators=FINAL_FLUX_OPERATOR_CATEGORIES)


@pytest.fixture(scope="module")
def tiny_flux(tiny30_model):
    return flux_model(tiny30_model)


@pytest.fixture(scope="module")
def smollm2_flux(smollm2_model):
    return flux_model(smollm2_model)


def test_prefill_decode_matches_reference_and_caches(tiny_flux, tiny30_golden):
    from flux_b200.runtime import NativeSmolLM2Prefill
    g = tiny30_golden
    ids = gi.tiny30_ids(17).cuda()
    with torch.inference_mode():
        native = NativeSmolLM2Prefill.capture(tiny_flux, ids, max_decode_steps=3)
    np.testing.assert_allclose(np32(native.logits), g["prefill17_logits"], rtol=RTOL, atol=ATOL)
    assert native.prompt_length == native.cache_position == native.cache_length == 17
    assert native.key_cache.shape == native.value_cache.shape == (30, 1, 3, 20, 64)
    token = int(torch.argmax(native.logits))
    assert token == g["steps3_tokens"][0]
    for step in range(3):
        logits = native.replay(torch.tensor([[token]], device="cuda"))
        np.testing.assert_allclose(np32(logits), g["steps3_logits"][step], rtol=RTOL, atol=ATOL)
        token = int(torch.argmax(logits))
        assert token == g["steps3_tokens"][step + 1]
        assert native.cache_position == native.cache_length == 18 + step
    keys = native.key_cache[:, 0].double()
    values = native.value_cache[:, 0].double()
    np.testing.assert_allclose(keys.sum(dim=(1, 2, 3)).cpu().numpy(), g["cache20_key_sums"], rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(values.sum(dim=(1, 2, 3)).cpu().numpy(), g["cache20_value_sums"], rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(native.key_cache[0, 0].cpu().numpy(), g["cache20_key_l0"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(native.value_cache[29, 0].cpu().numpy(), g["cache20_value_l29"], rtol=RTOL, atol=ATOL)
    with pytest.raises(RuntimeError, match="exhausted"):
        native.replay(torch.tensor([[token]], device="cuda"))


def test_greedy_generation_matches_reference_exactly(tiny_flux, tiny30_golden):
    from flux_b200.runtime import NativeSmolLM2Prefill, native_smollm2_greedy_generate
    expected = torch.from_numpy(tiny30_golden["generate7_8"]).view(1, -1)
    ids = gi.tiny30_ids(7).cuda()
    with torch.inference_mode():
        native = NativeSmolLM2Prefill.capture(tiny_flux, ids, max_decode_steps=7)
        addresses = native.stable_addresses()
        generated = native.generate_greedy(8)
        actual = torch.cat((ids, generated), dim=-1).cpu()
    assert actual.shape == (1, 15)
    assert torch.equal(actual, expected)
    assert torch.equal(generated[:, :1].cpu(), torch.argmax(native.prefill_logits, dim=-1).cpu())
    assert native.cache_position == native.cache_length == 7 + 7
    assert native.generation_step == 8
    assert native.stable_addresses() == addresses
    with pytest.raises(RuntimeError, match="prefill or reset"):
        native.generate_greedy(1)
    with torch.inference_mode():
        native.prefill(ids)
        repeated = native.generate_greedy(8).clone().cpu()
    assert torch.equal(repeated, expected[:, 7:])
    assert native.stable_addresses() == addresses
    with torch.inference_mode():
        full = native_smollm2_greedy_generate(tiny_flux, ids, max_new_tokens=8).cpu()
    assert torch.equal(full, expected)


@pytest.mark.parametrize("mode", ["persistent", "kernels"])
def test_greedy_generation_stops_on_eos(tiny_flux, tiny30_golden, monkeypatch, mode):
    """EOS-aware generation (the reference generates a fixed length; its README
    lists on-device EOS termination as the next step): the device loop stops
    after the step that samples the EOS token -- returned tokens, generation
    step and cache position all end there -- for an EOS inside the sequence,
    one equal to the prefill's own token, and one never sampled."""
    from flux_b200.runtime import NativeSmolLM2Prefill, native_smollm2_greedy_generate
    if mode == "kernels":
        monkeypatch.setenv("FLUX_B200_DECODE_STEP", "kernels")
    tokens = tiny30_golden["generate7_8"].reshape(-1)[7:].tolist()  # the reference's 8 greedy tokens
    k = next((i for i in range(1, len(tokens)) if tokens[i] not in tokens[:i]), None)
    ids = gi.tiny30_ids(7).cuda()
    with torch.inference_mode():
        native = NativeSmolLM2Prefill.capture(tiny_flux, ids, max_decode_steps=7)
        if k is not None:
            out = native.generate_greedy(8, eos_token_id=tokens[k]).cpu()
            assert out.view(-1).tolist() == tokens[:k + 1]
            assert native.generation_step == k + 1
            assert native.cache_position == 7 + k
            native.prefill(ids)
        out = native.generate_greedy(8, eos_token_id=tokens[0]).cpu()
        assert out.view(-1).tolist() == tokens[:1]
        assert native.cache_position == 7
        native.prefill(ids)
        never = next(t for t in range(128) if t not in tokens)
        out = native.generate_greedy(8, eos_token_id=never).cpu()
        assert out.view(-1).tolist() == tokens
        assert native.cache_position == 7 + 7
        native.prefill(ids)
        assert native.generate_greedy(8).cpu().view(-1).tolist() == tokens  # no EOS: fixed length
        if k is not None:
            full = native_smollm2_greedy_generate(tiny_flux, ids, max_new_tokens=8, eos_token_id=tokens[k]).cpu()
            assert full.view(-1).tolist() == ids.view(-1).cpu().tolist() + tokens[:k + 1]


def test_eager_flux_path_and_decode_capture(tiny30_model, tiny_flux, tiny30_golden):
    """Eager Flux ops (HF forward with torch.ops.flux.*) then the native decode
    captured from that eager prefill (``NativeSmolLM2Decode.capture``)."""
    from flux_b200.runtime import NativeSmolLM2Decode
    g = tiny30_golden
    ids = gi.tiny30_ids(17).cuda()
    with torch.inference_mode():
        out = tiny_flux(input_ids=ids, use_cache=True, logits_to_keep=1)
    np.testing.assert_allclose(np32(out.logits), g["prefill17_logits"], rtol=RTOL, atol=ATOL)
    with torch.inference_mode():
        decode = NativeSmolLM2Decode.capture(tiny_flux, ids, max_decode_steps=3)
    np.testing.assert_allclose(np32(decode.prefill_logits), g["prefill17_logits"], rtol=RTOL, atol=ATOL)
    token = torch.argmax(decode.prefill_logits, dim=-1).view(1, 1)
    for step in range(3):
        logits = decode.replay(token)
        np.testing.assert_allclose(np32(logits), g["steps3_logits"][step], rtol=RTOL, atol=ATOL)
        token = torch.argmax(logits, dim=-1).view(1, 1)
    token = torch.argmax(decode.prefill_logits, dim=-1).view(1, 1)
    decode.reset(token, decode._source_key_caches, decode._source_value_caches, cache_position=17)
    assert decode.cache_position == decode.cache_length == 17
    np.testing.assert_allclose(np32(decode.replay(token)), g["steps3_logits"][0], rtol=RTOL, atol=ATOL)
    with pytest.raises(RuntimeError, match="one K/V tensor per layer"):
        decode.reset(token, decode._source_key_caches[:-1], decode._source_value_caches, cache_position=17)


def test_prefill_reuse_and_input_errors(tiny_flux):
    from flux_b200.runtime import NativeSmolLM2Prefill
    first = gi.tiny30_ids(9).cuda()
    second = (first + 7) % 128
    native = NativeSmolLM2Prefill.capture(tiny_flux, first, max_decode_steps=1)
    with torch.inference_mode():
        actual = native.prefill(second).clone()
        expected = tiny_flux(input_ids=second, use_cache=True, logits_to_keep=1)
    np.testing.assert_allclose(np32(actual), np32(expected.logits), rtol=RTOL, atol=ATOL)
    for layer, cache in enumerate(expected.past_key_values.layers):
        np.testing.assert_allclose(native.key_cache[layer, ..., :9, :].cpu().numpy(), cache.keys.cpu().numpy(),
                                   rtol=RTOL, atol=ATOL)
    ids = gi.tiny30_ids(5).cuda()
    with pytest.raises(ValueError, match="non-negative"):
        NativeSmolLM2Prefill.capture(tiny_flux, ids, max_decode_steps=-1)
    with pytest.raises(ValueError, match="batch of one"):
        NativeSmolLM2Prefill.capture(tiny_flux, ids.expand(2, -1))
    with pytest.raises(ValueError, match="vocabulary"):
        NativeSmolLM2Prefill.capture(tiny_flux, torch.full_like(ids, 128))
    native = NativeSmolLM2Prefill.capture(tiny_flux, ids)
    with pytest.raises(ValueError, match="prompt shape"):
        native.prefill(ids[:, :-1])


def test_benchmark_geometry_teacher_forced(smollm2_flux, smollm2_golden):
    """Vocab 49152, tied head: logits within 1e-4 abs/rel of the reference FP32
    path for the prefill and four teacher-forced steps."""
    from flux_b200.runtime import NativeSmolLM2Prefill
    g = smollm2_golden
    prompt = gi.uniform_prompt(128).cuda()
    native = NativeSmolLM2Prefill.capture(smollm2_flux, prompt, max_decode_steps=4)
    np.testing.assert_allclose(np32(native.logits), g["prompt128_forced4_logits"][0], rtol=LOGIT_TOL, atol=LOGIT_TOL)
    for step, token in enumerate(g["forced4_tokens"]):
        logits = native.replay(torch.tensor([[int(token)]], device="cuda"))
        np.testing.assert_allclose(np32(logits), g["prompt128_forced4_logits"][step + 1], rtol=LOGIT_TOL,
                                   atol=LOGIT_TOL)


def test_synthetic_cache_decode_matches_reference(smollm2_model, smollm2_flux, smollm2_golden):
    from flux_b200.runtime import NativeSmolLM2Decode
    config = hf.smollm2_config()
    keys, values = hf.synthetic_cache(config, 1000, seed=5)
    token = torch.tensor([[17]], device="cuda")
    decode = NativeSmolLM2Decode.capture_from_state(smollm2_flux, token, [k.cuda() for k in keys],
                                                    [v.cuda() for v in values], cache_position=1000,
                                                    cache_capacity=1002)
    for step in range(2):
        logits = decode.replay(token)
        np.testing.assert_allclose(np32(logits), smollm2_golden["synth1000_logits"][step], rtol=LOGIT_TOL,
                                   atol=LOGIT_TOL)
        token = torch.argmax(logits, dim=-1).view(1, 1)


@pytest.mark.parametrize("mode", ["persistent", "kernels"])
@pytest.mark.parametrize("context", [1, 2, 10, 129, 2048, 8192])
def test_long_context_decode_vs_oracle(smollm2_model, smollm2_flux, context, mode, monkeypatch):
    """Decode over ``context`` synthetic rows (split-K chunking at every size up
    to the benchmark's 8192 -> 8194) against the numpy oracle, teacher-forced,
    for both step implementations: the single persistent launch (default) and
    the 151-kernel graph."""
    from flux_b200.runtime import NativeSmolLM2Decode
    monkeypatch.setenv("FLUX_B200_DECODE_STEP", mode)
    config = hf.smollm2_config()
    keys, values = hf.synthetic_cache(config, context, seed=context, std=0.5)
    capacity = context + 3
    tokens = gi.uniform_prompt(3, seed=context)[0].tolist()
    decode = NativeSmolLM2Decode.capture_from_state(
        smollm2_flux, torch.tensor([[tokens[0]]], device="cuda"), [k.cuda() for k in keys],
        [v.cuda() for v in values], cache_position=context, cache_capacity=capacity)
    cos, sin = hf.rope_tables(smollm2_model, capacity)
    oracle = o.Decoder(hf.oracle_weights(smollm2_model), capacity, cos.numpy(), sin.numpy())
    oracle.load_cache([k.numpy()[0] for k in keys], [v.numpy()[0] for v in values], context)
    for token in tokens:
        logits = np32(decode.replay(torch.tensor([[token]], device="cuda")))
        expected = oracle.step(token)
        np.testing.assert_allclose(logits, expected, rtol=LOGIT_TOL, atol=LOGIT_TOL)
        assert int(np.argmax(logits)) == o.greedy_argmax(expected)
    assert decode.cache_position == capacity
    # the three new cache rows match the oracle's
    np.testing.assert_allclose(decode.key_cache[:, 0, :, context:capacity].cpu().numpy(),
                               oracle.key_cache[:, :, context:capacity], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(decode.value_cache[:, 0, :, context:capacity].cpu().numpy(),
                               oracle.value_cache[:, :, context:capacity], rtol=1e-4, atol=1e-5)


def test_replay_on_non_default_stream_and_memory(tiny_flux):
    """Replays enqueue on the caller's current stream (``test_native_runtimes.cu``
    non-default stream case) and the memory report adds up."""
    from flux_b200.runtime import NativeSmolLM2Prefill
    ids = gi.tiny30_ids(5).cuda()
    native = NativeSmolLM2Prefill.capture(tiny_flux, ids, max_decode_steps=4)
    reference = NativeSmolLM2Prefill.capture(tiny_flux, ids, max_decode_steps=4)
    stream = torch.cuda.Stream()
    token = torch.argmax(native.logits, dim=-1).view(1, 1)
    stream.wait_stream(torch.cuda.current_stream())  # the token comes from the default stream
    with torch.cuda.stream(stream):
        a = native.replay(token).clone()
    stream.synchronize()
    b = reference.replay(token)
    # The step is deterministic (exact integer split-K tallies, fixed-order
    # merges): two runtimes agree bit for bit.
    assert torch.equal(a, b)
    memory = native.memory
    assert memory.cache_bytes == 2 * 30 * 3 * 9 * 64 * 4
    assert memory.owned_tensor_bytes > memory.cache_bytes


def test_replay_host_matches_tensor_replay(tiny_flux):
    """The host-buffer step (``fx_decode_replay_host``): teacher-forced host
    tokens in, the sampled token back as an int; bitwise the same logits and
    tokens as the tensor replay path, and None keeps the device token."""
    from flux_b200.runtime import NativeSmolLM2Prefill
    ids = gi.tiny30_ids(5).cuda()
    host = NativeSmolLM2Prefill.capture(tiny_flux, ids, max_decode_steps=6)
    dev = NativeSmolLM2Prefill.capture(tiny_flux, ids, max_decode_steps=6)
    host_logits = host.native_object()._decode.logits()  # the decode step's (not the prefill's) logits
    for i, token in enumerate([7, 123, 49151, None, 5]):
        nxt = host.replay_host(token)
        if token is None:
            expected = dev.replay().clone()
        else:
            expected = dev.replay(torch.tensor([[token]], dtype=torch.int64, device="cuda")).clone()
        torch.cuda.synchronize()
        assert torch.equal(host_logits, expected), i
        assert nxt == int(dev.current_token.item()) == int(host.current_token.item())
    with pytest.raises(RuntimeError, match="exhausted"):
        for _ in range(8):
            host.replay_host(1)


@pytest.mark.parametrize("prompt_length", [1, 64, 65, 200, 777])
def test_prefill_long_prompt_vs_oracle(smollm2_model, smollm2_flux, prompt_length):
    """The native prefill (tensor-core causal attention over 128-query blocks
    and 64-row key tiles: one row, partial last tile, causal diagonal)
    against the oracle: prefill logits, every cache row, and the first decode
    step after it."""
    from flux_b200.runtime import NativeSmolLM2Prefill
    ids = gi.uniform_prompt(prompt_length, seed=prompt_length).cuda()
    with torch.inference_mode():
        native = NativeSmolLM2Prefill.capture(smollm2_flux, ids, max_decode_steps=2)
    capacity = prompt_length + 2
    cos, sin = hf.rope_tables(smollm2_model, capacity)
    oracle = o.Decoder(hf.oracle_weights(smollm2_model), capacity, cos.numpy(), sin.numpy())
    expected = oracle.prefill(ids[0].cpu().numpy())
    np.testing.assert_allclose(np32(native.logits), expected, rtol=LOGIT_TOL, atol=LOGIT_TOL)
    np.testing.assert_allclose(native.key_cache[:, 0, :, :prompt_length].cpu().numpy(),
                               oracle.key_cache[:, :, :prompt_length], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(native.value_cache[:, 0, :, :prompt_length].cpu().numpy(),
                               oracle.value_cache[:, :, :prompt_length], rtol=1e-4, atol=1e-5)
    token = int(np.argmax(expected))
    logits = native.replay(torch.tensor([[token]], device="cuda"))
    np.testing.assert_allclose(np32(logits), oracle.step(token), rtol=LOGIT_TOL, atol=LOGIT_TOL)


def test_prefill_tensor_core_attention_matches_simt(smollm2_flux, monkeypatch):
    """A 2500-token prompt (neither a multiple of the 128-query blocks nor of
    the 64-key tiles) through the tcgen05 3xTF32 attention and through the
    FP32 SIMT flash kernel (FLUX_B200_PREFILL_ATTENTION=simt): prefill logits
    and every layer's cache rows agree to FP32 rounding."""
    from flux_b200.runtime import NativeSmolLM2Prefill
    ids = gi.uniform_prompt(2500, seed=25).cuda()
    with torch.inference_mode():
        tc = NativeSmolLM2Prefill.capture(smollm2_flux, ids, max_decode_steps=1)
        tc_logits, tc_keys = tc.logits.clone(), tc.key_cache[:, 0, :, :2500].clone()
        tc_values = tc.value_cache[:, 0, :, :2500].clone()
        del tc
        monkeypatch.setenv("FLUX_B200_PREFILL_ATTENTION", "simt")
        simt = NativeSmolLM2Prefill.capture(smollm2_flux, ids, max_decode_steps=1)
    torch.testing.assert_close(tc_logits, simt.logits, rtol=LOGIT_TOL, atol=LOGIT_TOL)
    torch.testing.assert_close(tc_keys, simt.key_cache[:, 0, :, :2500], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(tc_values, simt.value_cache[:, 0, :, :2500], rtol=1e-4, atol=1e-5)



def _decode_from_cache(model, length=300, capacity=320, token=77):
    from flux_b200.runtime import NativeSmolLM2Decode
    keys, values = hf.synthetic_cache(hf.smollm2_config(), length, seed=9, std=0.5)
    keys, values = [k.cuda() for k in keys], [v.cuda() for v in values]
    tok = torch.tensor([[token]], device="cuda")
    rt = NativeSmolLM2Decode.capture_from_state(model, tok, keys, values, cache_position=length,
                                                cache_capacity=capacity)
    return rt, tok, keys, values


def test_step_failure_is_reported_and_recoverable(smollm2_flux):
    """Failure detection without a GPU fault: CTA 0 of the persistent step
    reports a failure at layer 7 (fx_decode_inject_failure, as if one of its
    bounded waits had expired).  The other CTAs find the error word in their
    polls within ~1 ms and drain, so the step ends promptly (well inside the
    2 s wait bound), the host reads FX_ERR_DEVICE, the context stays usable,
    and after a reset the runtime reproduces a fresh runtime's logits."""
    import time
    from flux_b200 import _native
    fresh, tok, keys, values = _decode_from_cache(smollm2_flux)
    expected = fresh.replay().clone()
    rt, _, _, _ = _decode_from_cache(smollm2_flux)
    handle = rt.native_object()._handle
    _native.check(_native.load().fx_decode_inject_failure(handle, 7))
    start = time.perf_counter()
    rt.replay()
    torch.cuda.synchronize()
    assert time.perf_counter() - start < 1.0
    with pytest.raises(RuntimeError, match="bounded wait"):
        rt.cache_position  # noqa: B018  (reads the state and the error word)
    _native.check(_native.load().fx_decode_inject_failure(handle, -1))
    rt.reset(tok, keys, values, cache_position=300)
    logits = rt.replay()
    torch.cuda.synchronize()
    assert rt.cache_position == 301
    torch.testing.assert_close(logits, expected, rtol=1e-6, atol=1e-6)


def test_capture_failure_is_reported_and_cleaned_up(smollm2_flux, monkeypatch):
    """Host-side injection: a launch that fails while the step graph is being
    captured ends the capture, frees the half-built runtime and reports the
    error; the next runtime builds and runs normally."""
    monkeypatch.setenv("FLUX_B200_INJECT_CAPTURE_FAILURE", "1")
    with pytest.raises(RuntimeError, match="injected failure during CUDA graph capture"):
        _decode_from_cache(smollm2_flux)
    monkeypatch.delenv("FLUX_B200_INJECT_CAPTURE_FAILURE")
    rt, _, _, _ = _decode_from_cache(smollm2_flux)
    rt.replay()
    torch.cuda.synchronize()
    assert rt.cache_position == 301
