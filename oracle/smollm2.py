"""numpy FP32 restatement of the Flux SmolLM2-135M decode path (test oracle).

TEST INFRASTRUCTURE ONLY -- imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU legs as the checker; never by the product.

The reference computes its FP32 path with Hugging Face ``LlamaForCausalLM``
eager (transformers, not vendored in the reference; 5.5.0 in this image, the
reference README validated 5.16.1) driven as ``benchmarks/benchmark_flux.py:
533-564`` does, and with Flux's own operator oracles in ``flux/ops/*.py``.
Each function below restates one of those and cites the line it follows.
Parity with the real thing is pinned in ``tests/test_oracle.py`` against the
golden vectors that ``tests/golden/make_golden.py`` produced by running the
reference code itself.

Layout conventions match the reference native runtime:

* packed QKV weight ``[960, 576]`` = q rows 0..575 | k rows 576..767 | v rows
  768..959 (``flux/model/smollm2_flux.py:321-338``);
* packed gate/up weight ``[3072, 576]`` = gate rows | up rows
  (``flux/model/smollm2_flux.py:152-161``);
* compact cache per layer ``[3, capacity, 64]`` (batch dim dropped), the whole
  cache ``[30, 3, capacity, 64]`` (``native_decode_runtime_cuda.cu:1170-1173``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

F32 = np.float32

HIDDEN = 576
INTERMEDIATE = 1536
Q_HEADS = 9
KV_HEADS = 3
HEAD_DIM = 64
QKV_WIDTH = 960
LAYERS = 30


# ---------------------------------------------------------------- operators


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """RMSNorm over the last axis.

    Follows ``transformers ... LlamaRMSNorm.forward`` (x * rsqrt(mean(x^2) +
    eps), then weight *) which Flux restates in ``flux/ops/rmsnorm.py:6-24``.
    """
    x = np.asarray(x, dtype=F32)
    variance = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    inv = (F32(1.0) / np.sqrt(variance + F32(eps))).astype(F32)
    return (np.asarray(weight, F32) * (x * inv)).astype(F32)


def residual_rmsnorm(hidden, residual, weight, eps):
    """``(norm_out, residual_out)`` -- ``flux/ops/residual_rmsnorm.py:10-33``.

    ``residual_out`` is the exact FP32 sum; the reference pins it at atol 0.
    """
    residual_out = (np.asarray(hidden, F32) + np.asarray(residual, F32)).astype(F32)
    return rms_norm(residual_out, weight, eps), residual_out


def rotate_half(x: np.ndarray) -> np.ndarray:
    """``cat(-x2, x1)`` -- transformers ``rotate_half`` / ``flux/ops/rope.py:40-42``."""
    half = x.shape[-1] // 2
    return np.concatenate((-x[..., half:], x[..., :half]), axis=-1)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """``x*cos + rotate_half(x)*sin`` with both products rounded separately.

    numpy evaluates the two products and the sum as three FP32 roundings, which
    is what transformers ``apply_rotary_pos_emb`` does on the CPU and what the
    reference CUDA kernel forces with ``__fmul_rn``/``__fadd_rn``
    (``csrc/packed_qkv_rope_cache/packed_qkv_rope_cache_cuda.cu:19-49``), so the
    result is bit-exact with both.
    """
    x = np.asarray(x, F32)
    return (x * cos).astype(F32) + (rotate_half(x) * sin).astype(F32)


def rope_tables(positions: int, theta: float = 1.0e5, dim: int = HEAD_DIM):
    """cos/sin tables ``[positions, dim]`` with HF's default RoPE recipe.

    transformers ``LlamaRotaryEmbedding.compute_default_rope_parameters`` and
    ``forward``: inv_freq = 1 / theta**(arange(0, dim, 2)/dim) in FP32, freqs =
    inv_freq * position, emb = cat(freqs, freqs).  numpy's FP32 cos/sin may
    differ from torch's by an ulp; tests that need bit-exact tables feed the
    tables produced by the model's own ``rotary_emb`` instead.
    """
    exponents = (np.arange(0, dim, 2, dtype=np.int64).astype(F32) / F32(dim)).astype(F32)
    inv_freq = (F32(1.0) / np.power(F32(theta), exponents, dtype=F32)).astype(F32)
    pos = np.arange(positions, dtype=F32)[:, None]
    freqs = (pos * inv_freq[None, :]).astype(F32)
    emb = np.concatenate((freqs, freqs), axis=-1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """Max-subtracted FP32 softmax -- ``flux/ops/softmax.py:6-20``."""
    x = np.asarray(x, F32)
    shifted = x - np.max(x, axis=axis, keepdims=True)
    e = np.exp(shifted).astype(F32)
    return (e / np.sum(e, axis=axis, keepdims=True, dtype=F32)).astype(F32)


def gqa_decode_attention(query, key_cache, value_cache, mask=None, scale=0.125, length=None):
    """One-token grouped-query attention over an unexpanded cache.

    ``flux/ops/gqa_decode_attention.py:10-83``: query ``[B, Hq, 1, D]``, caches
    ``[B, Hkv, cap, D]``, q-head ``h`` reads kv-head ``h // (Hq // Hkv)``, only the
    first ``length`` positions are valid, optional additive mask broadcastable
    to ``[B, Hq, 1, cap]``.  Returns ``[B, Hq, 1, D]``.
    """
    q = np.asarray(query, F32)
    k = np.asarray(key_cache, F32)
    v = np.asarray(value_cache, F32)
    b, hq, _, d = q.shape
    _, hkv, cap, _ = k.shape
    n = cap if length is None else int(length)
    if not 1 <= n <= cap:
        raise ValueError("cache_length must be within cache capacity")
    groups = hq // hkv
    qg = q[:, :, 0, :].reshape(b, hkv, groups, d)
    scores = np.einsum("bkgd,bkld->bkgl", qg, k[:, :, :n], dtype=F32).astype(F32)
    scores = (scores * F32(scale)).reshape(b, hq, 1, n)
    if mask is not None:
        scores = scores + np.broadcast_to(np.asarray(mask, F32), (b, hq, 1, cap))[..., :n]
    p = softmax(scores).reshape(b, hkv, groups, n)
    out = np.einsum("bkgl,bkld->bkgd", p, v[:, :, :n], dtype=F32).astype(F32)
    return out.reshape(b, hq, 1, d)


def silu(x: np.ndarray) -> np.ndarray:
    """``x * sigmoid(x)`` (torch ``F.silu``; the reference CUDA kernels use
    ``g / (1 + expf(-g))``, ``packed_gate_up_gemv_cuda.cu:44``)."""
    x = np.asarray(x, F32)
    with np.errstate(over="ignore"):  # exp(-x) -> inf gives silu -> -0, as in FP32 torch
        return (x * (F32(1.0) / (F32(1.0) + np.exp(-x)))).astype(F32)


def packed_swiglu(packed: np.ndarray) -> np.ndarray:
    """``silu(gate) * up`` on ``[..., 2I]`` -- ``flux/ops/packed_swiglu.py:9-19``."""
    packed = np.asarray(packed, F32)
    half = packed.shape[-1] // 2
    return (silu(packed[..., :half]) * packed[..., half:]).astype(F32)


def linear(x: np.ndarray, weight: np.ndarray) -> np.ndarray:
    """``x @ W^T`` in FP32 (``torch.nn.functional.linear``)."""
    return np.matmul(np.asarray(x, F32), np.asarray(weight, F32).T).astype(F32)


def greedy_argmax(logits: np.ndarray) -> int:
    """Greedy token: the maximum with NaN counted as the maximum and the lowest
    index winning ties (``csrc/greedy_generation/greedy_generation_cuda.cu:19-37``
    and torch ``argmax``)."""
    logits = np.asarray(logits, F32).reshape(-1)
    nan = np.flatnonzero(np.isnan(logits))
    if nan.size:
        return int(nan[0])
    return int(np.argmax(logits))


# ------------------------------------------------------------------ the model


@dataclass
class LayerWeights:
    input_norm: np.ndarray   # [576]
    qkv: np.ndarray          # [960, 576]
    o: np.ndarray            # [576, 576]
    post_norm: np.ndarray    # [576]
    gate_up: np.ndarray      # [3072, 576]
    down: np.ndarray         # [576, 1536]


@dataclass
class ModelWeights:
    embed: np.ndarray        # [V, 576]
    lm_head: np.ndarray      # [V, 576] (the same array when tied)
    final_norm: np.ndarray   # [576]
    layers: list[LayerWeights] = field(default_factory=list)
    eps: float = 1.0e-5
    scale: float = 0.125

    @property
    def vocab(self) -> int:
        return int(self.embed.shape[0])


def weights_from_state_dict(state: dict, eps: float = 1.0e-5, scale: float = 0.125) -> ModelWeights:
    """Build oracle weights from a Hugging Face Llama state dict of numpy arrays
    (standard ``q_proj``/``k_proj``/... keys).  Packing follows
    ``flux/model/smollm2_flux.py:321-338`` (QKV) and ``:152-161`` (gate/up)."""
    def get(name):
        return np.ascontiguousarray(np.asarray(state[name], F32))

    embed = get("model.embed_tokens.weight")
    lm_head = get("lm_head.weight") if "lm_head.weight" in state else embed
    layers = []
    index = 0
    while f"model.layers.{index}.input_layernorm.weight" in state:
        p = f"model.layers.{index}."
        qkv = np.concatenate([get(p + "self_attn.q_proj.weight"),
                              get(p + "self_attn.k_proj.weight"),
                              get(p + "self_attn.v_proj.weight")], axis=0)
        gate_up = np.concatenate([get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")], axis=0)
        layers.append(LayerWeights(
            input_norm=get(p + "input_layernorm.weight"), qkv=qkv,
            o=get(p + "self_attn.o_proj.weight"),
            post_norm=get(p + "post_attention_layernorm.weight"),
            gate_up=gate_up, down=get(p + "mlp.down_proj.weight")))
        index += 1
    return ModelWeights(embed=embed, lm_head=lm_head, final_norm=get("model.norm.weight"),
                        layers=layers, eps=eps, scale=scale)


class Decoder:
    """Batch-1 decode state: the compact cache plus a position counter.

    ``step`` is one native replay (``native_decode_runtime_cuda.cu:1042-1098``):
    embedding row -> 30 x (input norm, packed QKV, RoPE, cache write at
    ``position``, GQA over ``position + 1`` rows, o_proj, residual norm, gate/up
    SwiGLU, down, residual) -> final norm -> LM head.  ``prefill`` is the causal
    multi-token path that fills rows ``[0, S)`` (``native_prefill_runtime_cuda.cu:
    553-665``).
    """

    def __init__(self, weights: ModelWeights, capacity: int, cos: np.ndarray, sin: np.ndarray):
        self.w = weights
        self.capacity = int(capacity)
        self.cos = np.asarray(cos, F32)
        self.sin = np.asarray(sin, F32)
        n_layers = len(weights.layers)
        self.key_cache = np.zeros((n_layers, KV_HEADS, self.capacity, HEAD_DIM), F32)
        self.value_cache = np.zeros_like(self.key_cache)
        self.position = 0

    def load_cache(self, keys, values, position: int) -> None:
        """Install ``position`` prefilled rows per layer (``reset`` semantics)."""
        self.key_cache[:] = 0
        self.value_cache[:] = 0
        for layer, (k, v) in enumerate(zip(keys, values)):
            self.key_cache[layer, :, :position] = np.asarray(k, F32).reshape(KV_HEADS, -1, HEAD_DIM)[:, :position]
            self.value_cache[layer, :, :position] = np.asarray(v, F32).reshape(KV_HEADS, -1, HEAD_DIM)[:, :position]
        self.position = int(position)

    def _layer(self, layer: int, h: np.ndarray, start: int) -> np.ndarray:
        """One decoder layer over rows ``h[s]`` at positions ``start + s``."""
        lw = self.w.layers[layer]
        s_len = h.shape[0]
        n = rms_norm(h, lw.input_norm, self.w.eps)
        qkv = linear(n, lw.qkv)
        q = qkv[:, :576].reshape(s_len, Q_HEADS, HEAD_DIM).transpose(1, 0, 2)
        k = qkv[:, 576:768].reshape(s_len, KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
        v = qkv[:, 768:].reshape(s_len, KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
        cos = self.cos[start:start + s_len][None]
        sin = self.sin[start:start + s_len][None]
        q = rope(q, cos, sin)
        k = rope(k, cos, sin)
        self.key_cache[layer, :, start:start + s_len] = k
        self.value_cache[layer, :, start:start + s_len] = v
        total = start + s_len
        keys = self.key_cache[layer, :, :total]
        values = self.value_cache[layer, :, :total]
        groups = Q_HEADS // KV_HEADS
        out = np.empty((Q_HEADS, s_len, HEAD_DIM), F32)
        for kv in range(KV_HEADS):
            qg = q[kv * groups:(kv + 1) * groups]                     # [g, S, D]
            scores = (np.matmul(qg, keys[kv].T) * F32(self.w.scale)).astype(F32)  # [g, S, total]
            if s_len > 1:
                rows = np.arange(s_len)[:, None] + start
                cols = np.arange(total)[None, :]
                scores = np.where(cols <= rows, scores, -np.inf).astype(F32)
            out[kv * groups:(kv + 1) * groups] = np.matmul(softmax(scores), values[kv])
        attn = out.transpose(1, 0, 2).reshape(s_len, HIDDEN)
        normed, residual = residual_rmsnorm(linear(attn, lw.o), h, lw.post_norm, self.w.eps)
        swiglu = packed_swiglu(linear(normed, lw.gate_up))
        return (residual + linear(swiglu, lw.down)).astype(F32)

    def logits_for(self, h_row: np.ndarray) -> np.ndarray:
        return linear(rms_norm(h_row, self.w.final_norm, self.w.eps), self.w.lm_head)

    def forward(self, tokens, start: int) -> np.ndarray:
        """Run ``tokens`` at positions ``start..`` and return the last row's logits."""
        tokens = np.asarray(tokens, np.int64).reshape(-1)
        if start + tokens.size > self.capacity:
            raise ValueError("fixed-capacity state is exhausted")
        h = self.w.embed[tokens].astype(F32)
        for layer in range(len(self.w.layers)):
            h = self._layer(layer, h, start)
        self.position = start + tokens.size
        self.final_hidden = h[-1]
        return self.logits_for(h[-1:])[0]

    def prefill(self, ids) -> np.ndarray:
        self.key_cache[:] = 0
        self.value_cache[:] = 0
        return self.forward(ids, 0)

    def step(self, token: int) -> np.ndarray:
        return self.forward([int(token)], self.position)


__all__ = [
    "Decoder", "LayerWeights", "ModelWeights", "gqa_decode_attention", "greedy_argmax",
    "linear", "packed_swiglu", "residual_rmsnorm", "rms_norm", "rope", "rope_tables",
    "rotate_half", "silu", "softmax", "weights_from_state_dict",
]
