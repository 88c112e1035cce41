"""Deterministic inputs shared by the golden generator and the tests.

Every generator here restates the input recipe of one of the reference's own
tests (cited per function), using torch's CPU generator so that the same bytes
come out here and on the GPU box (same image, same torch).  Where a reference
test drew its inputs from a CUDA generator, the CPU generator is used instead
with the same seed (CUDA RNG streams cannot be reproduced on a CPU host).
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import torch

EPSILON = 1e-5
GOLDEN_DIR = Path(__file__).resolve().parent  # the committed .npz fixtures


# ------------------------------------------------------------ seeded models
# The real SmolLM2 checkpoint is not available offline; the workloads use the
# same architecture with seeded random init (transformers' default N(0, 0.02)
# linear / embedding init, unit norms), built on the CPU in FP32.

def smollm2_config(vocab_size: int = 49152, max_positions: int = 8320, layers: int = 30) -> "LlamaConfig":
    """SmolLM2-135M geometry (30 x 576, MLP 1536, 9/3 heads x 64, tied)."""
    from transformers import LlamaConfig
    config = LlamaConfig(
        hidden_size=576, intermediate_size=1536, num_hidden_layers=layers,
        num_attention_heads=9, num_key_value_heads=3, head_dim=64,
        vocab_size=vocab_size, max_position_embeddings=max_positions,
        rms_norm_eps=1e-5, rope_theta=1.0e5, tie_word_embeddings=True,
        attention_bias=False, attention_dropout=0.0, mlp_bias=False,
    )
    config._attn_implementation = "eager"
    return config


def reference_runtime_config() -> "LlamaConfig":
    """The full-geometry, vocab-128 configuration of the reference's runtime
    tests (``tests/test_system.py:318-335``): untied, default RoPE theta."""
    from transformers import LlamaConfig
    config = LlamaConfig(
        hidden_size=576, intermediate_size=1536, num_hidden_layers=30,
        num_attention_heads=9, num_key_value_heads=3, head_dim=64,
        vocab_size=128, max_position_embeddings=8192, rms_norm_eps=1e-5,
        attention_bias=False, attention_dropout=0.0, mlp_bias=False,
    )
    config._attn_implementation = "eager"
    return config


def build_model(config: "LlamaConfig", seed: int) -> "LlamaForCausalLM":
    """Seeded CPU FP32 model in eval mode (``torch.manual_seed`` then HF init)."""
    from transformers import LlamaForCausalLM
    torch.manual_seed(seed)
    return LlamaForCausalLM(config).float().eval()


def wave(shape) -> torch.Tensor:
    """``sin(0.013 i) + cos(0.007 i)`` -- ``tests/test_ops.py:71-73``."""
    values = torch.arange(math.prod(shape), dtype=torch.float32)
    return (torch.sin(values * 0.013) + torch.cos(values * 0.007)).reshape(shape)


def gqa_inputs(capacity: int = 73):
    """Seed-1307 Q/K/V/mask -- ``tests/test_ops.py:360-366`` (CPU generator)."""
    generator = torch.Generator().manual_seed(1307)
    query = torch.randn((1, 9, 1, 64), generator=generator)
    keys = torch.randn((1, 3, capacity, 64), generator=generator)
    values = torch.randn((1, 3, capacity, 64), generator=generator)
    mask = torch.randn((1, 1, 1, capacity), generator=generator) * 0.05
    return query, keys, values, mask


def gqa_pin_inputs(batch, query_heads, kv_heads, head_dim, capacity):
    """``tests/test_references.py:279-290``: seed 1000+capacity, mask x 0.1."""
    torch.manual_seed(1000 + capacity)
    query = torch.randn(batch, query_heads, 1, head_dim)
    key = torch.randn(batch, kv_heads, capacity, head_dim)
    value = torch.randn_like(key)
    mask = torch.randn(batch, 1, 1, capacity) * 0.1
    return query, key, value, mask


GQA_PIN_CASES = [
    (shape, cap_len)
    for shape in ((1, 9, 3, 64), (2, 4, 2, 8))
    for cap_len in ((1, 1), (17, 11), (129, 128))
]


def rope_inputs(batch: int, sequence: int, position_offset: int):
    """``tests/test_references.py:303-314``: seed 191, theta 1e5 tables."""
    torch.manual_seed(191)
    query = torch.randn(batch, 9, sequence, 64)
    key = torch.randn(batch, 3, sequence, 64)
    positions = torch.arange(position_offset, position_offset + sequence).float()
    inv_freq = 1.0 / 100000.0 ** (torch.arange(0, 64, 2).float() / 64)
    frequencies = torch.outer(positions, inv_freq)
    embedding = torch.cat((frequencies, frequencies), dim=-1)
    cos = embedding.cos().unsqueeze(0).expand(batch, -1, -1)
    sin = embedding.sin().unsqueeze(0).expand(batch, -1, -1)
    return query, key, cos, sin


ROPE_CASES = ((1, 1, 0), (1, 1, 4095), (1, 7, 37), (2, 128, 1024))


def qkv_inputs():
    """Seed-1245 packed QKV case -- ``tests/test_ops.py:436-444`` (CPU generator)."""
    generator = torch.Generator().manual_seed(1245)
    packed = torch.randn((1, 1, 960), generator=generator)
    frequencies = torch.randn((1, 1, 64), generator=generator)
    keys = torch.randn((1, 3, 17, 64), generator=generator)
    values = torch.randn((1, 3, 17, 64), generator=generator)
    return packed, frequencies.cos(), frequencies.sin(), keys, values, torch.tensor(11)


def gate_up_inputs():
    """Seed-1234 gate/up GEMV case -- ``tests/test_ops.py:539-543`` (CPU generator)."""
    generator = torch.Generator().manual_seed(1234)
    return (torch.randn((1, 1, 576), generator=generator),
            torch.randn((3072, 576), generator=generator))


def lcg_values(count: int, scale: float = 1.0, bias: float = 0.0, seed: int = 1729) -> np.ndarray:
    """The native tests' LCG -- ``csrc/tests/cuda_test_utils.cuh:128-140``."""
    out = np.empty(count, np.float32)
    state = seed
    for index in range(count):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        unit = np.float32(state >> 8) / np.float32(1 << 24)
        out[index] = np.float32(bias) + np.float32(scale) * (np.float32(2.0) * unit - np.float32(1.0))
    return out


def tiny30_ids(length: int, vocab: int = 128) -> torch.Tensor:
    """``(11 i + 3) % 128`` -- ``tests/test_system.py:352-353``."""
    return ((torch.arange(length).unsqueeze(0) * 11 + 3) % vocab).long()


def uniform_prompt(length: int, vocab: int = 49152, seed: int = 0) -> torch.Tensor:
    """Seeded uniform token ids (the benchmark configurations' prompts)."""
    return torch.randint(0, vocab, (1, length), generator=torch.Generator().manual_seed(seed))
