"""GPU parity on the configurations the benchmark times, against the oracle and
the reference's own FP32 path, at the benchmark's sizes.

* the batch-1 step at every sweep context (128 ... 8192), 32
  consecutive teacher-forced steps each (128 at 8192), logits checked against
  the numpy oracle at every step;
* the native prefill of the benchmark's seeded 8192-token prompt
  against goldens of transformers' eager FP32 path on the same prompt
  (``tests/golden/make_prefill_golden.py``): last-position logits, per-layer
  cache sums and sampled cache rows;
* checkpoints with outlier dimensions: split-K partials far beyond the
  fixed-point tally range stay finite and match the oracle;
* sequences of a 64-sequence batch at the benchmark's ragged
  contexts (seeded U[512, 4096]) against the oracle over several steps;
* B = 64 / 256 at L = 8192, sampled sequences against the oracle.

The bar (north_star): logits within 1e-4 abs / 1e-4 rel; greedy tokens equal
except where the oracle's top-2 logit margin is below that tolerance.
"""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from oracle import hf_reference as hf
from oracle import smollm2 as o
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4


def np32(t):
    return t.detach().reshape(-1).cpu().numpy().astype(np.float32)


def flux_model(cpu_model):
    from flux_b200.integration import FINAL_FLUX_OPERATOR_CATEGORIES, enable_flux_ops
    return enable_flux_ops(copy.deepcopy(cpu_model).to("cuda"), operators=FINAL_FLUX_OPERATOR_CATEGORIES)


@pytest.fixture(scope="module")
def smollm2_flux(smollm2_model):
    return flux_model(smollm2_model)


@pytest.fixture(scope="module")
def oracle_weights(smollm2_model):
    return hf.oracle_weights(smollm2_model)


def assert_greedy_matches(logits: np.ndarray, expected: np.ndarray) -> None:
    """Equal greedy tokens unless the oracle's top two logits are within the
    logits tolerance of each other (then either token is acceptable)."""
    token = int(np.argmax(logits))
    want = o.greedy_argmax(expected)
    if token != want:
        top2 = np.sort(expected)[-2:]
        assert top2[1] - top2[0] < LOGIT_TOL * max(1.0, abs(float(top2[1]))), (token, want, top2)
        assert expected[token] >= top2[0] - LOGIT_TOL


@pytest.mark.parametrize("context,steps", [(128, 32), (512, 32), (1024, 32), (2048, 32), (4096, 32), (8192, 128)])
def test_context_sweep_steps_vs_oracle(smollm2_model, smollm2_flux, oracle_weights, context, steps):
    """the persistent step over ``context`` seeded cache rows (the
    step does not depend on how the rows were produced; prefill parity has its
    own tests), ``steps`` consecutive teacher-forced seeded tokens -- the
    double-buffered exchange words and tallies cycle through every parity and
    epoch -- with the logits compared at every step and the new cache rows at
    the end."""
    from flux_b200.runtime import NativeSmolLM2Decode
    config = hf.smollm2_config()
    keys, values = hf.synthetic_cache(config, context, seed=context + 1, std=0.5)
    capacity = context + steps
    tokens = gi.uniform_prompt(steps, seed=context + 2)[0].tolist()
    decode = NativeSmolLM2Decode.capture_from_state(
        smollm2_flux, torch.tensor([[tokens[0]]], device="cuda"), [k.cuda() for k in keys],
        [v.cuda() for v in values], cache_position=context, cache_capacity=capacity)
    cos, sin = hf.rope_tables(smollm2_model, capacity)
    oracle = o.Decoder(oracle_weights, capacity, cos.numpy(), sin.numpy())
    oracle.load_cache([k.numpy()[0] for k in keys], [v.numpy()[0] for v in values], context)
    for step, token in enumerate(tokens):
        logits = np32(decode.replay(torch.tensor([[token]], device="cuda")))
        expected = oracle.step(token)
        np.testing.assert_allclose(logits, expected, rtol=LOGIT_TOL, atol=LOGIT_TOL, err_msg=f"step {step}")
        assert_greedy_matches(logits, expected)
    assert decode.cache_position == capacity
    np.testing.assert_allclose(decode.key_cache[:, 0, :, context:capacity].cpu().numpy(),
                               oracle.key_cache[:, :, context:capacity], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(decode.value_cache[:, 0, :, context:capacity].cpu().numpy(),
                               oracle.value_cache[:, :, context:capacity], rtol=1e-4, atol=1e-5)


def test_benchmark_prefill_8192_vs_reference_golden(smollm2_flux):
    """configs[1]'s cache: the native prefill of the seed-0 8192-token prompt
    against transformers' eager FP32 prefill of the same prompt."""
    from flux_b200.runtime import NativeSmolLM2Prefill
    golden = dict(np.load(gi.GOLDEN_DIR / "prefill8192.npz"))
    prompt = gi.uniform_prompt(8192, seed=0).cuda()
    with torch.inference_mode():
        native = NativeSmolLM2Prefill.capture(smollm2_flux, prompt, max_decode_steps=1)
    logits = np32(native.logits)
    np.testing.assert_allclose(logits, golden["logits"], rtol=LOGIT_TOL, atol=LOGIT_TOL)
    assert_greedy_matches(logits, golden["logits"])
    rows = golden["rows"].tolist()
    for name, cache in (("key", native.key_cache), ("value", native.value_cache)):
        layers = cache[:, 0, :, :8192].double()
        sums = torch.stack([layers.sum(dim=(2, 3)), (layers * layers).sum(dim=(2, 3))], dim=-1).cpu().numpy()
        # each sum adds 524,288 cached values: the 1e-4 relative bar of the rows
        np.testing.assert_allclose(sums, golden[f"{name}_sums"], rtol=1e-4, atol=5e-2)
        np.testing.assert_allclose(cache[:, 0, :, rows].cpu().numpy(), golden[f"{name}_rows"], rtol=1e-4,
                                   atol=1e-5)


def test_large_split_k_partials_vs_oracle(smollm2_model):
    """Checkpoints with outlier dimensions ("massive activations"): o_proj of
    layer 7 and down of layers 3 and 20 scaled so the persistent step's
    split-K partials reach ~1e4-1e6, beyond the fixed-point tally range
    (|y| < 2^13); they go through the FP64 overflow words and the logits stay
    finite and within the bar."""
    from flux_b200.runtime import NativeSmolLM2Decode
    model = copy.deepcopy(smollm2_model)
    with torch.no_grad():
        model.model.layers[3].mlp.down_proj.weight.mul_(1e7)
        model.model.layers[20].mlp.down_proj.weight.mul_(3e5)
        model.model.layers[7].self_attn.o_proj.weight.mul_(1e7)
    flux = flux_model(model)
    context = 300
    keys, values = hf.synthetic_cache(hf.smollm2_config(), context, seed=31, std=0.5)
    tokens = gi.uniform_prompt(4, seed=31)[0].tolist()
    capacity = context + len(tokens)
    decode = NativeSmolLM2Decode.capture_from_state(
        flux, torch.tensor([[tokens[0]]], device="cuda"), [k.cuda() for k in keys], [v.cuda() for v in values],
        cache_position=context, cache_capacity=capacity)
    cos, sin = hf.rope_tables(model, capacity)
    oracle = o.Decoder(hf.oracle_weights(model), capacity, cos.numpy(), sin.numpy())
    oracle.load_cache([k.numpy()[0] for k in keys], [v.numpy()[0] for v in values], context)
    for token in tokens:
        logits = np32(decode.replay(torch.tensor([[token]], device="cuda")))
        expected = oracle.step(token)
        assert np.isfinite(logits).all()
        np.testing.assert_allclose(logits, expected, rtol=LOGIT_TOL, atol=LOGIT_TOL)
        assert_greedy_matches(logits, expected)
    # the residual stream really left the fixed-point range
    assert float(np.abs(oracle.final_hidden).max()) > 8192.0


def test_batched_benchmark_contexts_vs_oracle(smollm2_model, smollm2_flux, oracle_weights):
    """64 sequences at the benchmark's seeded ragged contexts in
    [512, 4096] (cache rows drawn on the GPU as the benchmark does); four of
    them, spread over the batch, against the oracle for four greedy steps."""
    from flux_b200 import sharding
    from flux_b200.runtime import NativeSmolLM2BatchedDecode
    batch, steps = 64, 4
    lengths, tokens = sharding.shard_contexts(0, sharding.sequence_shard(batch, 1, 0), 512, 4096)
    capacity = max(lengths) + steps
    runtime = NativeSmolLM2BatchedDecode(smollm2_flux, batch, capacity)
    checked = (0, 21, 42, 63)
    cos, sin = hf.rope_tables(smollm2_model, capacity)
    oracles = {}
    gen = torch.Generator(device="cuda")
    for i, n in enumerate(lengths):
        gen.manual_seed(1_000_003 + 29 + i)
        keys = torch.randn(30, 3, n, 64, device="cuda", generator=gen) * 0.5
        values = torch.randn(30, 3, n, 64, device="cuda", generator=gen) * 0.5
        runtime.load(i, tokens[i], list(keys), list(values), n)
        if i in checked:
            dec = o.Decoder(oracle_weights, capacity, cos.numpy(), sin.numpy())
            dec.load_cache(list(keys.cpu().numpy()), list(values.cpu().numpy()), n)
            oracles[i] = dec
        del keys, values
    runtime.check()
    current = {i: tokens[i] for i in checked}
    for _ in range(steps):
        logits = runtime.step(1).cpu().numpy()
        runtime.check()
        sampled = runtime.tokens().cpu().tolist()
        for i, dec in oracles.items():
            expected = dec.step(current[i])
            np.testing.assert_allclose(logits[i], expected, rtol=LOGIT_TOL, atol=LOGIT_TOL, err_msg=f"seq {i}")
            assert_greedy_matches(logits[i], expected)
            current[i] = sampled[i]  # follow the runtime's own greedy choice


@pytest.mark.parametrize("batch", [64, 256])
def test_large_batch_attention_sampled_vs_oracle(batch):
    """configs[4] at L = 8192: inputs drawn on the GPU (Q, K, V ~ N(0, 1)),
    the whole batch through the compact kernel, 12 sequences spread over the
    batch against the oracle."""
    from tests.test_gpu_attention import TOL, attention
    length = 8192
    g = torch.Generator(device="cuda").manual_seed(batch * 7 + 1)
    q = torch.randn(batch, 9, 1, 64, device="cuda", generator=g)
    k = torch.randn(batch, 3, length, 64, device="cuda", generator=g)
    v = torch.randn(batch, 3, length, 64, device="cuda", generator=g)
    out = attention(q, k, v, length).cpu().numpy()
    for b in np.linspace(0, batch - 1, 12).astype(int):
        expected = o.gqa_decode_attention(q[b:b + 1].cpu().numpy(), k[b:b + 1].cpu().numpy(),
                                          v[b:b + 1].cpu().numpy(), None, 0.125, length)
        np.testing.assert_allclose(out[b:b + 1], expected, **TOL, err_msg=f"sequence {b}")
