"""The reference's own FP32 CPU path: Hugging Face ``LlamaForCausalLM`` eager.

TEST INFRASTRUCTURE ONLY -- used by ``tests/`` to build seeded models, by
``__graft_entry__.smoke()`` and by ``bench.py``'s ``cpu_baseline`` and
``--impl reference`` legs as the timed CPU baseline.  Never imported by the
product.

Flux's FP32 reference path is the transformers eager model loaded by
``flux/model/smollm2.py:25-36`` and driven as ``benchmarks/benchmark_flux.py:
533-564`` (``model(input_ids=tok, past_key_values=cache, use_cache=True,
logits_to_keep=1)``).  The real SmolLM2 checkpoint is not available offline, so
the models here use the same architecture with seeded random init (HF default
N(0, 0.02) linear/embedding init, unit norms), tied embeddings and RoPE theta
1e5, as the benchmark configuration specifies.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch
from transformers import DynamicCache, LlamaForCausalLM

from oracle import smollm2
# The seeded workload models are defined beside the other seeded inputs (the
# GPU path and the benchmark build the same models without importing the oracle).
from tests.golden.inputs import build_model, reference_runtime_config, smollm2_config  # noqa: F401


def numpy_state(model: torch.nn.Module) -> dict[str, np.ndarray]:
    return {k: v.detach().cpu().numpy() for k, v in model.state_dict().items()}


def oracle_weights(model: torch.nn.Module) -> smollm2.ModelWeights:
    layer = model.model.layers[0]
    return smollm2.weights_from_state_dict(
        numpy_state(model), eps=float(layer.input_layernorm.variance_epsilon),
        scale=float(layer.self_attn.scaling))


def rope_tables(model: torch.nn.Module, positions: int) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin ``[positions, 64]`` from the model's own ``rotary_emb`` exactly as
    the reference runtime owner builds them (``flux/runtime/native_smollm2.py:
    131-138``), on the model's device."""
    device = model.model.embed_tokens.weight.device
    ids = torch.arange(positions, dtype=torch.long, device=device).unsqueeze(0)
    seed = model.model.embed_tokens.weight[:1].view(1, 1, -1)
    with torch.inference_mode():
        cos, sin = model.model.rotary_emb(seed, ids)
    return cos.reshape(positions, -1).contiguous(), sin.reshape(positions, -1).contiguous()


def synthetic_cache(config: LlamaConfig, length: int, seed: int, std: float = 1.0):
    """Per-layer K/V ``[1, 3, length, 64]`` drawn from N(0, std^2), seeded."""
    generator = torch.Generator().manual_seed(seed)
    keys, values = [], []
    for _ in range(config.num_hidden_layers):
        keys.append(torch.randn((1, config.num_key_value_heads, length, config.head_dim), generator=generator) * std)
        values.append(torch.randn((1, config.num_key_value_heads, length, config.head_dim), generator=generator) * std)
    return keys, values


def dynamic_cache(config: LlamaConfig, keys, values) -> DynamicCache:
    cache = DynamicCache(config=config)
    for layer, (k, v) in enumerate(zip(keys, values)):
        cache.update(k.clone(), v.clone(), layer)
    return cache


def decode_step(model, token: int, cache) -> torch.Tensor:
    """One HF eager decode step, the way the reference benchmark drives it."""
    with torch.inference_mode():
        out = model(input_ids=torch.tensor([[int(token)]], dtype=torch.long), past_key_values=cache,
                    use_cache=True, logits_to_keep=1)
    return out.logits[0, -1]


def time_cpu_decode(model, config: LlamaConfig, context: int, steps: int, seed: int = 0,
                    threads: int | None = None, budget_s: float = 20.0) -> dict:
    """Time HF eager FP32 decode on the host cores at a given context.

    The bounded sample: the cache is filled with ``context`` seeded synthetic
    K/V rows per layer (a decode step's cost does not depend on the values),
    then up to ``steps`` greedy steps are timed one by one (wall clock), stopping
    early once ``budget_s`` is spent.  Returns ms/token (median) and the sample
    description.
    """
    from oracle.host import limit_threads
    threads = limit_threads(threads)
    keys, values = synthetic_cache(config, context, seed)
    cache = dynamic_cache(config, keys, values)
    token = int(seed) % config.vocab_size
    # one untimed warm-up step
    logits = decode_step(model, token, cache)
    token = int(torch.argmax(logits))
    times = []
    start_all = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        logits = decode_step(model, token, cache)
        token = int(torch.argmax(logits))
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - start_all > budget_s:
            break
    times.sort()
    median = times[len(times) // 2]
    return {
        "ms_per_token": median * 1e3,
        "steps": len(times),
        "context": context,
        "threads": threads,
        "total_s": time.perf_counter() - start_all,
    }


def time_cpu_generation(model, prompt: torch.Tensor, new_tokens: int, threads: int | None = None) -> dict:
    """configs[0] on the host cores: HF eager FP32 prefill of ``prompt`` then
    ``new_tokens - 1`` greedy decode steps (``new_tokens`` generated tokens, the
    first from the prefill), as ``benchmarks/benchmark_flux.py:633-660`` drives
    the eager generation; wall-clock prefill and decode times and the tokens."""
    from oracle.host import limit_threads
    threads = limit_threads(threads)
    with torch.inference_mode():
        t0 = time.perf_counter()
        out = model(input_ids=prompt, use_cache=True, logits_to_keep=1)
        token = out.logits[:, -1].argmax(dim=-1, keepdim=True)
        t1 = time.perf_counter()
        cache, tokens = out.past_key_values, [int(token)]
        for _ in range(new_tokens - 1):
            out = model(input_ids=token, past_key_values=cache, use_cache=True, logits_to_keep=1)
            token = out.logits[:, -1].argmax(dim=-1, keepdim=True)
            tokens.append(int(token))
        t2 = time.perf_counter()
    return {"prefill_ms": (t1 - t0) * 1e3, "decode_ms": (t2 - t1) * 1e3, "total_ms": (t2 - t0) * 1e3,
            "tokens": tokens, "threads": threads}


__all__ = [
    "build_model", "decode_step", "dynamic_cache", "numpy_state", "oracle_weights",
    "reference_runtime_config", "rope_tables", "smollm2_config", "synthetic_cache",
    "time_cpu_decode", "time_cpu_generation",
]
