"""GPU parity of the batched greedy decode runtime (``fx_batch_*``, no reference
counterpart: the reference is batch 1 only) against the numpy oracle of the
reference's FP32 path, per sequence, and against the batch-1 runtime."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from oracle import hf_reference as hf
from oracle import smollm2 as o

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4


@pytest.fixture(scope="module")
def model_gpu(smollm2_model):
    from flux_b200.integration import FINAL_FLUX_OPERATOR_CATEGORIES, enable_flux_ops
    return enable_flux_ops(copy.deepcopy(smollm2_model).to("cuda"), operators=FINAL_FLUX_OPERATOR_CATEGORIES)


def _load(runtime, index, length, seed, token):
    config = hf.smollm2_config()
    if length == 0:
        runtime.load(index, token, [], [], 0)
        return None, None
    keys, values = hf.synthetic_cache(config, length, seed=seed, std=0.5)
    runtime.load(index, token, [k.cuda() for k in keys], [v.cuda() for v in values], length)
    return keys, values


@pytest.mark.parametrize("step", ["kernels", "layers"])
def test_batched_greedy_steps_match_oracle(model_gpu, smollm2_model, monkeypatch, step):
    """Both batched steps: the launch chain (default) and the cooperative
    layer kernel (FLUX_B200_BATCH_STEP=layers)."""
    from flux_b200.runtime import NativeSmolLM2BatchedDecode
    monkeypatch.setenv("FLUX_B200_BATCH_STEP", step)
    lengths = [0, 5, 130, 300]
    capacity = 304
    runtime = NativeSmolLM2BatchedDecode(model_gpu, len(lengths), capacity)
    cos, sin = hf.rope_tables(smollm2_model, capacity)
    weights = hf.oracle_weights(smollm2_model)
    oracles, tokens = [], []
    for i, length in enumerate(lengths):
        token = (7919 * (i + 1)) % 49152
        keys, values = _load(runtime, i, length, seed=100 + i, token=token)
        dec = o.Decoder(weights, capacity, cos.numpy(), sin.numpy())
        if length:
            dec.load_cache([k.numpy()[0] for k in keys], [v.numpy()[0] for v in values], length)
        oracles.append(dec)
        tokens.append(token)
    for step in range(3):
        logits = runtime.step(1).cpu().numpy()
        runtime.check()
        for i, dec in enumerate(oracles):
            expected = dec.step(tokens[i])
            np.testing.assert_allclose(logits[i], expected, rtol=LOGIT_TOL, atol=LOGIT_TOL)
            tokens[i] = o.greedy_argmax(expected)
        assert runtime.tokens().cpu().tolist() == tokens
        assert runtime.positions().cpu().tolist() == [n + step + 1 for n in lengths]
    generated = runtime.generated_tokens()[:, :3].cpu()
    assert int(runtime.device_generation_step().item()) == 3
    assert generated[:, 2].tolist() == tokens


def test_batched_matches_batch_one_runtime(model_gpu):
    """One sequence through the batched runtime and through the batch-1 graph."""
    from flux_b200.runtime import NativeSmolLM2BatchedDecode, NativeSmolLM2Decode
    config = hf.smollm2_config()
    length, capacity = 777, 784
    keys, values = hf.synthetic_cache(config, length, seed=3, std=0.5)
    keys, values = [k.cuda() for k in keys], [v.cuda() for v in values]
    single = NativeSmolLM2Decode.capture_from_state(model_gpu, torch.tensor([[123]], device="cuda"), keys, values,
                                                    cache_position=length, cache_capacity=capacity)
    batched = NativeSmolLM2BatchedDecode(model_gpu, 2, capacity)
    batched.load(0, 123, keys, values, length)
    batched.load(1, 5, keys, values, 300)
    for _ in range(4):
        a = single.replay().cpu().numpy().reshape(-1)
        b = batched.step(1)[0].cpu().numpy()
        np.testing.assert_allclose(b, a, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(batched.key_cache()[:, 0, :, length:length + 4].cpu().numpy(),
                               single.key_cache[:, 0, :, length:length + 4].cpu().numpy(), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("step", ["kernels", "layers"])
def test_batch_of_64_equals_each_sequence_alone(model_gpu, monkeypatch, step):
    """Rows never interact: a sequence's logits in a batch of 64 ragged
    contexts are bitwise those of the same sequence run alone."""
    from flux_b200.runtime import NativeSmolLM2BatchedDecode
    monkeypatch.setenv("FLUX_B200_BATCH_STEP", step)
    rng = np.random.default_rng(11)
    lengths = [int(x) for x in rng.integers(1, 600, size=64)]
    capacity = 608
    full = NativeSmolLM2BatchedDecode(model_gpu, 64, capacity)
    config = hf.smollm2_config()
    caches = {}
    for i, n in enumerate(lengths):
        keys, values = hf.synthetic_cache(config, n, seed=1000 + i, std=0.5)
        caches[i] = ([k.cuda() for k in keys], [v.cuda() for v in values])
        full.load(i, (31 * i + 7) % 49152, *caches[i], n)
    full.step(2)
    full.check()
    for i in (0, 17, 63):
        alone = NativeSmolLM2BatchedDecode(model_gpu, 1, capacity)
        alone.load(0, (31 * i + 7) % 49152, *caches[i], lengths[i])
        alone.step(2)
        assert torch.equal(alone.logits()[0], full.logits()[i])
        assert torch.equal(alone.generated_tokens()[0, :2], full.generated_tokens()[i, :2])


def test_batched_capacity_exhausted(model_gpu):
    from flux_b200.runtime import NativeSmolLM2BatchedDecode
    runtime = NativeSmolLM2BatchedDecode(model_gpu, 2, 8)
    runtime.load(0, 1, [], [], 0)
    runtime.step(8)
    runtime.check()
    with pytest.raises(RuntimeError, match="exhausted"):
        runtime.step(1)


def test_two_lanes_match_one_lane(model_gpu, monkeypatch):
    """The batch split into two lanes on two streams (the default) against
    the whole batch as one chain (FLUX_B200_BATCH_LANES=1): the split-K plans
    differ, so the logits agree to rounding; each run's tokens are the argmax
    of its own logits."""
    from flux_b200.runtime import NativeSmolLM2BatchedDecode
    monkeypatch.setenv("FLUX_B200_BATCH_STEP", "kernels")  # lanes belong to the launch-chain step
    rng = np.random.default_rng(5)
    lengths = [int(x) for x in rng.integers(1, 500, size=7)]
    capacity = 512
    config = hf.smollm2_config()
    caches = [hf.synthetic_cache(config, n, seed=2000 + i, std=0.5) for i, n in enumerate(lengths)]
    runs = []
    for lanes in ("1", "2"):
        monkeypatch.setenv("FLUX_B200_BATCH_LANES", lanes)
        runtime = NativeSmolLM2BatchedDecode(model_gpu, len(lengths), capacity)
        for i, n in enumerate(lengths):
            keys, values = caches[i]
            runtime.load(i, (101 * i + 3) % 49152, [k.cuda() for k in keys], [v.cuda() for v in values], n)
        logits = [runtime.step(1).clone() for _ in range(3)]
        runtime.check()
        runs.append((logits, runtime.generated_tokens()[:, :3].clone(), runtime.kernels_per_step))
    (one, gen_one, k_one), (two, gen_two, k_two) = runs
    for a, b in zip(one, two):
        torch.testing.assert_close(b, a, rtol=2e-5, atol=2e-5)
    for logits, gen in ((one, gen_one), (two, gen_two)):
        for step, row in enumerate(logits):
            assert torch.equal(gen[:, step], row.argmax(dim=-1).to(gen.dtype))
    assert k_two == k_one + 1 + 30 * 10


def test_layer_kernel_matches_launch_chain(model_gpu, monkeypatch):
    """The cooperative layer-kernel step (FLUX_B200_BATCH_STEP=layers: the
    attention merge, projections, norms, SwiGLU and RoPE between attention
    launches in one launch, SIMT FP32) against the default launch chain
    (tensor-core 3xTF32 split-K projections and separate reduction kernels):
    the same math in other summation orders, so the logits agree to rounding;
    2 launches per layer instead of 10."""
    from flux_b200.runtime import NativeSmolLM2BatchedDecode
    rng = np.random.default_rng(8)
    lengths = [int(x) for x in rng.integers(1, 700, size=9)]
    capacity = 712
    config = hf.smollm2_config()
    caches = [hf.synthetic_cache(config, n, seed=3000 + i, std=0.5) for i, n in enumerate(lengths)]
    runs = {}
    for mode in ("kernels", "layers"):
        monkeypatch.setenv("FLUX_B200_BATCH_STEP", mode)
        monkeypatch.setenv("FLUX_B200_BATCH_LANES", "1")
        runtime = NativeSmolLM2BatchedDecode(model_gpu, len(lengths), capacity)
        for i, n in enumerate(lengths):
            keys, values = caches[i]
            runtime.load(i, (211 * i + 5) % 49152, [k.cuda() for k in keys], [v.cuda() for v in values], n)
        logits = [runtime.step(1).clone() for _ in range(3)]
        runtime.check()
        runs[mode] = (logits, runtime.key_cache().clone(), runtime.kernels_per_step)
    (chain, chain_k, k_chain), (layers, layers_k, k_layers) = runs["kernels"], runs["layers"]
    for a, b in zip(chain, layers):
        torch.testing.assert_close(b, a, rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(layers_k, chain_k, rtol=1e-5, atol=1e-5)
    assert k_chain == k_layers + 30 * 8
