"""Pin the numpy oracle to the reference's own outputs (CPU only).

The goldens were produced by ``tests/golden/make_golden.py`` from the
reference's Python operator oracles and its transformers FP32 path.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from oracle import hf_reference as hf
from oracle import smollm2 as o
from tests.golden import inputs as gi

RTOL, ATOL = 2e-4, 2e-5  # tests/test_system.py:30-31


def close(a, b, rtol=1e-5, atol=1e-6):
    np.testing.assert_allclose(np.asarray(a, np.float32), np.asarray(b, np.float32), rtol=rtol, atol=atol)


def test_rmsnorm_and_residual_rmsnorm(ops_golden):
    x = gi.wave((2, 7, 576)).numpy()
    w = np.linspace(0.25, 1.75, 576, dtype=np.float32)
    close(o.rms_norm(x, w, gi.EPSILON), ops_golden["rmsnorm_out"], 1e-5, 2e-6)
    hidden, residual = gi.wave((2, 7, 576)).numpy(), (gi.wave((2, 7, 576)) * 0.25).numpy()
    norm, res = o.residual_rmsnorm(hidden, residual, w, gi.EPSILON)
    np.testing.assert_array_equal(res, ops_golden["residual_rmsnorm_residual"])
    close(norm, ops_golden["residual_rmsnorm_norm"], 1e-5, 2e-6)


def test_swiglu_softmax_attention_softmax(ops_golden):
    close(o.packed_swiglu(gi.wave((1, 7, 3072)).numpy()), ops_golden["packed_swiglu_out"], 2e-6, 2e-6)
    close(o.softmax(3.0 * gi.wave((5, 129)).numpy()), ops_golden["softmax_out"], 1e-5, 5e-7)
    scores, mask = 3.0 * gi.wave((2, 3, 5, 17)).numpy(), gi.wave((2, 1, 5, 17)).numpy() * 0.25
    scale = np.float32(17 ** -0.5)
    close(o.softmax(scores * scale + mask), ops_golden["attention_score_softmax_out"], 1e-5, 5e-7)


def test_gqa_decode_attention(ops_golden):
    q, k, v, m = (t.numpy() for t in gi.gqa_inputs(73))
    close(o.gqa_decode_attention(q, k, v, m, 0.125, 41), ops_golden["gqa73_masked"], 2e-5, 1e-6)
    close(o.gqa_decode_attention(q, k, v, None, 0.125, 41), ops_golden["gqa73_unmasked"], 2e-5, 1e-6)
    q, k, v, m = (t.numpy() for t in gi.gqa_inputs(1024))
    close(o.gqa_decode_attention(q, k, v, m, 0.125, 777), ops_golden["gqa1024_len777"], 2e-5, 1e-6)
    for (b, hq, hkv, d), (cap, n) in gi.GQA_PIN_CASES:
        q, k, v, m = (t.numpy() for t in gi.gqa_pin_inputs(b, hq, hkv, d, cap))
        close(o.gqa_decode_attention(q, k, v, m, d ** -0.5, n), ops_golden[f"gqa_pin_{b}_{hq}_{hkv}_{d}_{cap}_{n}"],
              1e-5, 5e-7)


def test_gqa_known_answers():
    """Q = 0 gives mean(V) (``csrc/benchmarks/cuda_microbenchmarks.cu:395-405``); a
    -FLT_MAX mask keeps only position 0 (``tests/test_references.py:292-299``)."""
    rng = np.random.default_rng(3)
    v = rng.standard_normal((1, 3, 50, 64)).astype(np.float32)
    out = o.gqa_decode_attention(np.zeros((1, 9, 1, 64), np.float32), v, v, None, 0.125, 50)
    close(out[0, :, 0], np.repeat(v[0].mean(axis=1), 3, axis=0), 1e-5, 1e-6)
    q = np.ones((1, 2, 1, 2), np.float32)
    key = np.zeros((1, 1, 3, 2), np.float32)
    value = np.array([[[[1.0, 2.0], [10.0, 20.0], [100.0, 200.0]]]], np.float32)
    fmin = np.finfo(np.float32).min
    mask = np.array([[[[0.0, fmin, fmin]]]], np.float32)
    close(o.gqa_decode_attention(q, key, value, mask, 1.0), np.broadcast_to(value[:, :, :1], (1, 2, 1, 2)))


def test_rope_bit_exact_against_transformers(ops_golden):
    for b, s, off in gi.ROPE_CASES:
        q, k, cos, sin = (t.numpy() for t in gi.rope_inputs(b, s, off))
        rq = o.rope(q, cos[:, None], sin[:, None])
        rk = o.rope(k, cos[:, None], sin[:, None])
        sha = [hashlib.sha256(np.ascontiguousarray(t, np.float32).tobytes()).hexdigest() for t in (rq, rk)]
        assert sha == list(ops_golden[f"rope_{b}_{s}_{off}_sha"]), (b, s, off)


def test_packed_qkv_rope_cache_pin(ops_golden):
    packed, cos, sin, _, _, _ = (t.numpy() for t in gi.qkv_inputs())
    q = packed[0, 0, :576].reshape(9, 1, 64)
    k = packed[0, 0, 576:768].reshape(3, 1, 64)
    np.testing.assert_array_equal(o.rope(q, cos[0], sin[0])[None], ops_golden["qkv_query"])
    np.testing.assert_array_equal(o.rope(k, cos[0], sin[0])[None], ops_golden["qkv_key_row"])
    np.testing.assert_array_equal(packed[0, 0, 768:].reshape(1, 3, 1, 64), ops_golden["qkv_value_row"])


def test_gate_up_pin(ops_golden):
    x, w = (t.numpy() for t in gi.gate_up_inputs())
    close(o.packed_swiglu(o.linear(x, w)), ops_golden["gate_up_out"], 1e-4, 1e-3)


def test_greedy_known_answers():
    """``csrc/tests/test_greedy_generation.cu:46-68``."""
    vocab = 49152
    logits = gi.lcg_values(vocab, 2000.0)
    assert o.greedy_argmax(logits) == int(np.argmax(logits))
    logits = np.full(vocab, -5000.0, np.float32)
    logits[177] = logits[321] = -3.0
    assert o.greedy_argmax(logits) == 177
    fmax = np.finfo(np.float32).max
    logits = np.full(vocab, -fmax, np.float32)
    logits[0] = fmax
    assert o.greedy_argmax(logits) == 0
    logits[0], logits[-1] = -fmax, fmax
    assert o.greedy_argmax(logits) == vocab - 1
    assert o.greedy_argmax(np.full(vocab, -np.inf, np.float32)) == 0
    logits = np.zeros(vocab, np.float32)
    logits[[9, 5000]] = np.nan
    assert o.greedy_argmax(logits) == 9


def test_tiny30_prefill_decode_and_cache(tiny30_model, tiny30_golden):
    g = tiny30_golden
    weights = hf.oracle_weights(tiny30_model)
    cos, sin = hf.rope_tables(tiny30_model, 20)
    dec = o.Decoder(weights, 20, cos.numpy(), sin.numpy())
    close(dec.prefill(gi.tiny30_ids(17).numpy()), g["prefill17_logits"], RTOL, ATOL)
    token = o.greedy_argmax(g["prefill17_logits"])
    assert token == g["steps3_tokens"][0]
    for step in range(3):
        logits = dec.step(token)
        close(logits, g["steps3_logits"][step], RTOL, ATOL)
        token = o.greedy_argmax(logits)
        assert token == g["steps3_tokens"][step + 1]
    np.testing.assert_allclose(dec.key_cache.astype(np.float64).sum(axis=(1, 2, 3)), g["cache20_key_sums"], rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(dec.value_cache.astype(np.float64).sum(axis=(1, 2, 3)), g["cache20_value_sums"], rtol=1e-4, atol=1e-3)
    close(dec.key_cache[0], g["cache20_key_l0"], RTOL, ATOL)
    close(dec.value_cache[29], g["cache20_value_l29"], RTOL, ATOL)


def test_tiny30_greedy_generation(tiny30_model, tiny30_golden):
    weights = hf.oracle_weights(tiny30_model)
    cos, sin = hf.rope_tables(tiny30_model, 15)
    dec = o.Decoder(weights, 15, cos.numpy(), sin.numpy())
    ids = gi.tiny30_ids(7).numpy()[0]
    token = o.greedy_argmax(dec.prefill(ids))
    out = list(ids) + [token]
    for _ in range(7):
        token = o.greedy_argmax(dec.step(token))
        out.append(token)
    np.testing.assert_array_equal(out, tiny30_golden["generate7_8"])


def test_smollm2_geometry_teacher_forced(smollm2_model, smollm2_golden):
    g = smollm2_golden
    weights = hf.oracle_weights(smollm2_model)
    assert weights.vocab == 49152 and weights.lm_head is weights.embed or np.shares_memory(weights.lm_head, weights.embed) or np.array_equal(weights.lm_head, weights.embed)
    cos, sin = hf.rope_tables(smollm2_model, 132)
    dec = o.Decoder(weights, 132, cos.numpy(), sin.numpy())
    close(dec.prefill(gi.uniform_prompt(128).numpy()), g["prompt128_forced4_logits"][0], 1e-4, 1e-4)
    for step, token in enumerate(g["forced4_tokens"]):
        close(dec.step(int(token)), g["prompt128_forced4_logits"][step + 1], 1e-4, 1e-4)


def test_smollm2_synthetic_cache_decode(smollm2_model, smollm2_golden):
    config = hf.smollm2_config()
    weights = hf.oracle_weights(smollm2_model)
    keys, values = hf.synthetic_cache(config, 1000, seed=5)
    cos, sin = hf.rope_tables(smollm2_model, 1002)
    dec = o.Decoder(weights, 1002, cos.numpy(), sin.numpy())
    dec.load_cache([k.numpy()[0] for k in keys], [v.numpy()[0] for v in values], 1000)
    token = 17
    for step in range(2):
        logits = dec.step(token)
        close(logits, smollm2_golden["synth1000_logits"][step], 1e-4, 1e-4)
        token = o.greedy_argmax(logits)


@pytest.mark.parametrize("name", ["rmsnorm", "residual_rmsnorm", "packed_swiglu"])
def test_oracle_against_reference_cpu_kernels(name):
    """Cross-check against the reference's own C++ CPU kernels when
    ``oracle/Makefile`` has built them into ``oracle/_ref``."""
    from oracle import ref_cpu
    lib = ref_cpu.load()
    if lib is None:
        pytest.skip("oracle/_ref not built (needs the reference checkout)")
    x = gi.wave((3, 576)).numpy()
    w = np.linspace(0.25, 1.75, 576, dtype=np.float32)
    if name == "rmsnorm":
        close(ref_cpu.rmsnorm(lib, x, w, 1e-5), o.rms_norm(x, w, 1e-5), 1e-6, 1e-6)
    elif name == "residual_rmsnorm":
        r = (x * np.float32(0.25)).astype(np.float32)
        norm, res = ref_cpu.residual_rmsnorm(lib, x, r, w, 1e-5)
        np.testing.assert_array_equal(res, o.residual_rmsnorm(x, r, w, 1e-5)[1])
        close(norm, o.residual_rmsnorm(x, r, w, 1e-5)[0], 1e-6, 1e-6)
    else:
        packed = gi.wave((3, 3072)).numpy()
        close(ref_cpu.packed_swiglu(lib, packed), o.packed_swiglu(packed), 2e-6, 2e-6)
