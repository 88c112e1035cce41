"""Generate the golden vectors by running the reference itself.

Run in a container that has the reference checkout (it is read-only and not
available on the GPU box):

    FLUX_REFERENCE=<reference checkout> python tests/golden/make_golden.py

(``FLUX_REFERENCE`` defaults to a ``reference`` directory beside this
repository.  The reference's ``flux`` package is put first on ``sys.path``, so
it, not this repository's ``flux`` compatibility package, is the one run.)

Op-level goldens come from the reference's own Python operator oracles
(``flux/ops/*.py``) and transformers' ``apply_rotary_pos_emb``.  Model-level
goldens come from the reference's FP32 path: transformers ``LlamaForCausalLM``
eager on the CPU, configured and driven as the reference's tests and benchmark
do (``tests/test_system.py:318-497``, ``benchmarks/benchmark_flux.py:533-564``).
Inputs are regenerated from seeds by ``tests/golden/inputs.py``; only small
inputs are stored.  Large bit-exact outputs are stored as SHA-256 digests.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden import inputs as gi  # noqa: E402
from oracle import hf_reference as hf  # noqa: E402
from transformers.models.llama.modeling_llama import apply_rotary_pos_emb  # noqa: E402

REFERENCE = Path(os.environ.get("FLUX_REFERENCE") or HERE.parents[2] / "reference").resolve()
sys.path.insert(0, str(REFERENCE))
for _name in [m for m in sys.modules if m == "flux" or m.startswith("flux.")]:
    del sys.modules[_name]
import flux.ops as ref_ops  # noqa: E402  (the reference package)

if not Path(ref_ops.__file__).resolve().is_relative_to(REFERENCE):
    raise SystemExit(f"flux.ops resolved to {ref_ops.__file__}, not the reference checkout at {REFERENCE}")


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().numpy().astype(np.float32).tobytes()).hexdigest()


def op_goldens() -> dict:
    g: dict[str, np.ndarray] = {}
    eps = gi.EPSILON
    # RMSNorm / residual RMSNorm on the reference's wave inputs.
    x = gi.wave((2, 7, 576))
    w = torch.linspace(0.25, 1.75, 576)
    g["rmsnorm_out"] = ref_ops.rms_norm(x, w, eps).numpy()
    hidden, residual = gi.wave((2, 7, 576)), gi.wave((2, 7, 576)) * 0.25
    norm, res = ref_ops.residual_rmsnorm(hidden, residual, w, eps)
    g["residual_rmsnorm_norm"], g["residual_rmsnorm_residual"] = norm.numpy(), res.numpy()
    # Packed SwiGLU, softmax and attention-score softmax.
    g["packed_swiglu_out"] = ref_ops.packed_swiglu(gi.wave((1, 7, 3072))).numpy()
    g["softmax_out"] = ref_ops.softmax(3.0 * gi.wave((5, 129))).numpy()
    scores, mask = 3.0 * gi.wave((2, 3, 5, 17)), gi.wave((2, 1, 5, 17)) * 0.25
    g["attention_score_softmax_out"] = ref_ops.attention_score_softmax(scores, mask, 17 ** -0.5).numpy()
    # GQA decode attention (seed 1307, cap 73, len 41; mask and no mask).
    q, k, v, m = gi.gqa_inputs(73)
    length = torch.tensor(41)
    g["gqa73_masked"] = ref_ops.gqa_decode_attention(q, k, v, m, 0.125, length).numpy()
    g["gqa73_unmasked"] = ref_ops.gqa_decode_attention(q, k, v, None, 0.125, length).numpy()
    q, k, v, m = gi.gqa_inputs(1024)
    g["gqa1024_len777"] = ref_ops.gqa_decode_attention(q, k, v, m, 0.125, torch.tensor(777)).numpy()
    for (b, hq, hkv, d), (cap, n) in gi.GQA_PIN_CASES:
        q, k, v, m = gi.gqa_pin_inputs(b, hq, hkv, d, cap)
        out = ref_ops.gqa_decode_attention(q, k, v, m, d ** -0.5, torch.tensor(n))
        g[f"gqa_pin_{b}_{hq}_{hkv}_{d}_{cap}_{n}"] = out.numpy()
    # RoPE: bit-exact transformers results (digests), plus the small cases in full.
    for b, s, off in gi.ROPE_CASES:
        q, k, cos, sin = gi.rope_inputs(b, s, off)
        eq, ek = apply_rotary_pos_emb(q, k, cos, sin)
        fq, fk = ref_ops.rope(q, k, cos, sin)
        assert torch.equal(eq, fq) and torch.equal(ek, fk)
        g[f"rope_{b}_{s}_{off}_sha"] = np.array([digest(eq), digest(ek)])
        if b * s <= 8:
            g[f"rope_{b}_{s}_{off}_q"], g[f"rope_{b}_{s}_{off}_k"] = eq.numpy(), ek.numpy()
    # Packed QKV / RoPE / cache update (seed 1245, position 11): expected query
    # and the rotated key / raw value rows that land in the cache.
    packed, cos, sin, keys, values, _ = gi.qkv_inputs()
    query = packed[..., :576].view(1, 1, 9, 64).transpose(1, 2)
    key = packed[..., 576:768].view(1, 1, 3, 64).transpose(1, 2)
    value = packed[..., 768:].view(1, 1, 3, 64).transpose(1, 2)
    rq, rk = ref_ops.rope(query, key, cos, sin)
    g["qkv_query"], g["qkv_key_row"], g["qkv_value_row"] = rq.numpy(), rk.numpy(), value.numpy()
    # Gate/up GEMV + SwiGLU (seed 1234), computed in float64 for a clean golden.
    x, weight = gi.gate_up_inputs()
    packed64 = torch.nn.functional.linear(x.double(), weight.double())
    g["gate_up_out"] = (torch.nn.functional.silu(packed64[..., :1536]) * packed64[..., 1536:]).float().numpy()
    return g


def tiny30_goldens() -> dict:
    """The reference runtime tests' model (``tests/test_system.py:318-497``)."""
    g: dict[str, np.ndarray] = {}
    config = hf.reference_runtime_config()
    model = hf.build_model(config, 2701)
    ids = gi.tiny30_ids(17)
    with torch.inference_mode():
        out = model(input_ids=ids, use_cache=True, logits_to_keep=1)
        g["prefill17_logits"] = out.logits[0, -1].numpy()
        cache = out.past_key_values
        token = out.logits.argmax(dim=-1)
        tokens, step_logits = [int(token)], []
        for _ in range(3):
            out = model(input_ids=token, past_key_values=cache, use_cache=True, logits_to_keep=1)
            step_logits.append(out.logits[0, -1].numpy())
            token = out.logits.argmax(dim=-1)
            tokens.append(int(token))
        g["steps3_logits"] = np.stack(step_logits)
        g["steps3_tokens"] = np.array(tokens, np.int64)
        keys = torch.stack([layer.keys[0] for layer in cache.layers])      # [30, 3, 20, 64]
        values = torch.stack([layer.values[0] for layer in cache.layers])
        g["cache20_key_sums"] = keys.double().sum(dim=(1, 2, 3)).numpy()
        g["cache20_value_sums"] = values.double().sum(dim=(1, 2, 3)).numpy()
        g["cache20_key_l0"], g["cache20_value_l29"] = keys[0].numpy(), values[29].numpy()
        gen = model.generate(input_ids=gi.tiny30_ids(7), do_sample=False, num_beams=1, max_new_tokens=8,
                             use_cache=True, pad_token_id=0)
        g["generate7_8"] = gen[0].numpy()
    return g


def smollm2_goldens() -> dict:
    """Benchmark geometry (vocab 49152, tied, theta 1e5), seed 0."""
    g: dict[str, np.ndarray] = {}
    config = hf.smollm2_config()
    model = hf.build_model(config, 0)
    prompt = gi.uniform_prompt(128, seed=0)
    forced = gi.uniform_prompt(4, seed=1)[0]
    with torch.inference_mode():
        out = model(input_ids=prompt, use_cache=True, logits_to_keep=1)
        logits = [out.logits[0, -1].numpy()]
        cache = out.past_key_values
        for token in forced:
            out = model(input_ids=token.view(1, 1), past_key_values=cache, use_cache=True, logits_to_keep=1)
            logits.append(out.logits[0, -1].numpy())
        g["prompt128_forced4_logits"] = np.stack(logits)
        g["forced4_tokens"] = forced.numpy()
        # Decode over a synthetic 1000-row cache (seed 5), two greedy steps.
        keys, values = hf.synthetic_cache(config, 1000, seed=5)
        cache = hf.dynamic_cache(config, keys, values)
        token, synth = 17, []
        for _ in range(2):
            row = hf.decode_step(model, token, cache)
            synth.append(row.numpy())
            token = int(torch.argmax(row))
        g["synth1000_logits"] = np.stack(synth)
    return g


def main() -> None:
    torch.set_num_threads(8)
    np.savez(HERE / "ops.npz", **op_goldens())
    np.savez(HERE / "model_tiny30.npz", **tiny30_goldens())
    np.savez(HERE / "model_smollm2.npz", **smollm2_goldens())
    for name in ("ops.npz", "model_tiny30.npz", "model_smollm2.npz"):
        print(name, (HERE / name).stat().st_size)


if __name__ == "__main__":
    main()
