"""``enable_flux_ops``: the reference's operator-category surface on flux_b200.

Interface kept from ``flux/model/smollm2_flux.py`` (names, category strings,
state-dict keys, error messages and *when* each fused branch applies); the
code is organised around three tables of this module:

* ``_CATEGORY_RULES`` -- which categories need which others, with the error a
  caller gets when one is missing;
* ``_NATIVE_PROBES`` -- which availability probe guards which category;
* ``_FUSED_DECODE_SHAPES`` -- the one-token tensor shapes the fused
  packed-QKV / RoPE / cache branch is compiled for.

A ``LayerPlan`` (the flags one decoder layer runs with) is derived once from
the selected categories and handed to every Flux module of the layer.  Packed
projections (``packed_qkv``, ``gate_up_proj``) are one helper,
``_PackedWeight``, that also keeps the standard Llama checkpoint keys in
``state_dict`` / ``load_state_dict``.

Every native call goes through a module global looked up at call time
(``rms_norm_native``, ``gqa_decode_attention_native``, ...), so a caller may
monkeypatch them, as the reference's own system tests do
(``tests/test_system.py:57-133``).  A caller that owns preallocated decode
buffers attaches them as ``module._flux_decode_scratch`` (attribute names as in
``smollm2_flux.py``); the forward paths then write into them with the ``_out``
operators.
"""

from __future__ import annotations

from collections.abc import Collection, Sequence
from dataclasses import dataclass
from typing import Any

import torch
from torch import nn
from transformers import StaticCache
from transformers.models.llama.modeling_llama import (
    LlamaAttention,
    LlamaDecoderLayer,
    LlamaForCausalLM,
    LlamaMLP,
    LlamaRMSNorm,
    apply_rotary_pos_emb,
    repeat_kv,
)

from flux_b200.operators import (  # noqa: F401  (re-exported names are patch points)
    CublasLtAlgorithm,
    attention_score_softmax_native,
    cublaslt_linear_config_out,
    gqa_decode_attention_native,
    gqa_decode_attention_native_out,
    native_attention_score_softmax_is_available,
    native_cublaslt_linear_is_available,
    native_gqa_decode_attention_is_available,
    native_packed_gate_up_gemv_is_available,
    native_packed_qkv_rope_cache_is_available,
    native_packed_swiglu_is_available,
    native_residual_rmsnorm_is_available,
    native_rmsnorm_is_available,
    native_rope_is_available,
    native_softmax_is_available,
    packed_gate_up_swiglu_native_out,
    packed_qkv_rope_cache_native,
    packed_qkv_rope_cache_native_out,
    packed_swiglu_native,
    packed_swiglu_native_out,
    residual_rmsnorm_native,
    residual_rmsnorm_native_out,
    rms_norm_native,
    rms_norm_native_out,
    rope_native,
    softmax_native,
)

# ------------------------------------------------------------------ categories
# Category strings and public constant names: smollm2_flux.py:58-80.

FLUX_OPERATOR_CATEGORIES = frozenset({"rmsnorm", "residual_rmsnorm", "rope", "softmax"})
FLUX_PACKED_MLP_CATEGORY = "mlp"
FLUX_PACKED_SWIGLU_CATEGORY = "packed_swiglu"
FLUX_PACKED_QKV_CATEGORY = "qkv"
FLUX_GQA_DECODE_ATTENTION_CATEGORY = "gqa_decode_attention"
FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY = "packed_qkv_rope_cache"
FLUX_CUBLASLT_PROJECTION_CATEGORY = "cublaslt_projection"
FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY = "fused_gate_up_swiglu"
FINAL_FLUX_OPERATOR_CATEGORIES = FLUX_OPERATOR_CATEGORIES | {
    FLUX_GQA_DECODE_ATTENTION_CATEGORY, FLUX_PACKED_MLP_CATEGORY, FLUX_PACKED_SWIGLU_CATEGORY,
    FLUX_PACKED_QKV_CATEGORY, FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY, FLUX_CUBLASLT_PROJECTION_CATEGORY,
    FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY,
}

# (category, categories it needs, message when one is missing) -- the
# reference's dependency checks (smollm2_flux.py:906-937), as data.
_CATEGORY_RULES: tuple[tuple[str, frozenset[str], str], ...] = (
    (FLUX_PACKED_SWIGLU_CATEGORY, frozenset({FLUX_PACKED_MLP_CATEGORY}),
     '"packed_swiglu" requires the "mlp" operator category'),
    (FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY,
     frozenset({"rope", FLUX_PACKED_QKV_CATEGORY, FLUX_GQA_DECODE_ATTENTION_CATEGORY}),
     '"packed_qkv_rope_cache" requires the "rope", "qkv", and "gqa_decode_attention" operator categories'),
    (FLUX_CUBLASLT_PROJECTION_CATEGORY, frozenset({FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY}),
     '"cublaslt_projection" requires the "packed_qkv_rope_cache" operator category'),
    (FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY, frozenset({FLUX_PACKED_MLP_CATEGORY, FLUX_PACKED_SWIGLU_CATEGORY}),
     '"fused_gate_up_swiglu" requires the "mlp" and "packed_swiglu" operator categories'),
)

# (category, operator name in the error, availability probe) -- the probes are
# looked up as module globals when enable_flux_ops runs (smollm2_flux.py:813-866).
_NATIVE_PROBES: tuple[tuple[str, str, str], ...] = (
    ("rmsnorm", "rmsnorm", "native_rmsnorm_is_available"),
    ("residual_rmsnorm", "residual_rmsnorm", "native_residual_rmsnorm_is_available"),
    ("softmax", "softmax", "native_softmax_is_available"),
    ("rope", "rope", "native_rope_is_available"),
    (FLUX_PACKED_SWIGLU_CATEGORY, "packed_swiglu", "native_packed_swiglu_is_available"),
    ("softmax+scores", "attention_score_softmax", "native_attention_score_softmax_is_available"),
    (FLUX_GQA_DECODE_ATTENTION_CATEGORY, "gqa_decode_attention", "native_gqa_decode_attention_is_available"),
    (FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY, "packed_qkv_rope_cache", "native_packed_qkv_rope_cache_is_available"),
    (FLUX_CUBLASLT_PROJECTION_CATEGORY, "cublaslt_projection", "native_cublaslt_linear_is_available"),
    (FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY, "gate_up_gemv", "native_packed_gate_up_gemv_is_available"),
)


@dataclass(frozen=True)
class LayerPlan:
    """The Flux paths one decoder layer runs, fixed when the model is enabled."""

    rmsnorm: bool = False
    residual_rmsnorm: bool = False
    rope: bool = False
    softmax: bool = False
    fuse_attention_scores: bool = True
    gqa_decode_attention: bool = False
    packed_qkv: bool = False
    packed_qkv_rope_cache: bool = False
    cublaslt_projection: bool = False
    packed_mlp: bool = False
    packed_swiglu: bool = False
    fused_gate_up_swiglu: bool = False

    @classmethod
    def from_categories(cls, selected: Collection[str], fuse_attention_scores: bool = True) -> "LayerPlan":
        s = frozenset(selected)
        return cls(rmsnorm="rmsnorm" in s, residual_rmsnorm="residual_rmsnorm" in s, rope="rope" in s,
                   softmax="softmax" in s, fuse_attention_scores=fuse_attention_scores,
                   gqa_decode_attention=FLUX_GQA_DECODE_ATTENTION_CATEGORY in s,
                   packed_qkv=FLUX_PACKED_QKV_CATEGORY in s,
                   packed_qkv_rope_cache=FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY in s,
                   cublaslt_projection=FLUX_CUBLASLT_PROJECTION_CATEGORY in s,
                   packed_mlp=FLUX_PACKED_MLP_CATEGORY in s, packed_swiglu=FLUX_PACKED_SWIGLU_CATEGORY in s,
                   fused_gate_up_swiglu=FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY in s)

    @property
    def replaces_attention(self) -> bool:
        return self.softmax or self.rope or self.gqa_decode_attention or self.packed_qkv


def _scratch(module: nn.Module):
    """The caller's preallocated decode buffers attached to ``module``, if any."""
    return getattr(module, "_flux_decode_scratch", None)


# ------------------------------------------------------------ packed weights


class _PackedWeight:
    """One parameter holding several source projections' weights stacked by
    rows, as ``nn.Linear`` attribute ``name`` of ``owner``; ``state_dict``
    reports (and ``load_state_dict`` accepts) the sources' own keys."""

    def __init__(self, owner: nn.Module, name: str, parts: Sequence[tuple[str, nn.Linear]],
                 errors: dict[str, str]) -> None:
        weights = [linear.weight for _, linear in parts]
        if any(linear.bias is not None for _, linear in parts):
            raise ValueError(errors["bias"])
        if len({w.requires_grad for w in weights}) != 1:
            raise ValueError(errors["requires_grad"])
        self.name = name
        self.keys = tuple(f"{key}.weight" for key, _ in parts)
        self.rows = tuple(w.shape[0] for w in weights)
        linear = nn.Linear(weights[0].shape[1], sum(self.rows), bias=False, device="meta", dtype=weights[0].dtype)
        linear.weight = nn.Parameter(torch.cat(weights, dim=0), requires_grad=weights[0].requires_grad)
        owner.add_module(name, linear)
        # (torch tags registered hooks with attributes, so they are plain functions)

        def split(_module, state_dict, prefix, _metadata) -> None:
            self.split(state_dict, prefix)

        def join(_module, state_dict, prefix, *_args) -> None:
            self.join(state_dict, prefix)

        owner.register_state_dict_post_hook(split)
        owner.register_load_state_dict_pre_hook(join)

    def split(self, state_dict: dict, prefix: str) -> None:
        """Replace the packed key by the sources' keys (row blocks of it)."""
        packed = state_dict.pop(f"{prefix}{self.name}.weight", None)
        if packed is not None:
            for key, part in zip(self.keys, packed.split(self.rows, dim=0), strict=True):
                state_dict[prefix + key] = part

    def join(self, state_dict: dict, prefix: str) -> None:
        """Replace the sources' keys by the packed key, when all are present."""
        keys = [prefix + key for key in self.keys]
        if f"{prefix}{self.name}.weight" not in state_dict and all(k in state_dict for k in keys):
            state_dict[f"{prefix}{self.name}.weight"] = torch.cat([state_dict.pop(k) for k in keys], dim=0)


# -------------------------------------------------------------- decode shapes
# The fused packed-QKV / RoPE / cache branch (smollm2_flux.py:441-489) runs on
# exactly one SmolLM2 token: every tensor must match its row here ("cap" is the
# cache capacity, required in [513, 8192]; None = any size in that dim).

_MIN_GRAPH_CAPACITY = 513   # the native graph's attention workspace needs > 512 rows
_MAX_DECODE_CAPACITY = 8192
_FUSED_DECODE_SHAPES: dict[str, tuple[Any, ...]] = {
    "hidden": (1, 1, 576),
    "cos": (1, 1, 64),
    "sin": (1, 1, 64),
    "keys": (1, 3, "cap", 64),
    "values": (1, 3, "cap", 64),
    "length": (),
}
_FUSED_DECODE_WIDTHS = {"query_width": 576, "key_width": 192, "value_width": 192, "query_heads": 9,
                        "key_value_heads": 3, "head_dim": 64}


def _shape_matches(tensor: torch.Tensor, pattern: tuple[Any, ...], cap: int) -> bool:
    if tensor.ndim != len(pattern):
        return False
    return all(size == (cap if want == "cap" else want) for size, want in zip(tensor.shape, pattern))


def _mask_broadcasts(mask: torch.Tensor, target: tuple[int, ...]) -> bool:
    return (mask.ndim == 4 and mask.dtype == torch.float32
            and all(m in (1, t) for m, t in zip(mask.shape, target, strict=True)))


def _mask_ok(mask: torch.Tensor | None, device: torch.device, target: tuple[int, ...]) -> bool:
    return mask is None or (mask.device == device and _mask_broadcasts(mask, target))


# ------------------------------------------------------------------ modules


class FluxRMSNorm(LlamaRMSNorm):
    """``LlamaRMSNorm`` on ``torch.ops.flux.rmsnorm``; shares the source
    Parameter, so parameter names and tying are unchanged
    (``smollm2_flux.py:238-263``)."""

    def __init__(self, source: LlamaRMSNorm) -> None:
        nn.Module.__init__(self)
        self.weight = source.weight
        self.variance_epsilon = source.variance_epsilon

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        buffers = _scratch(self)
        if buffers is None:
            return rms_norm_native(hidden_states, self.weight, self.variance_epsilon)
        return rms_norm_native_out(hidden_states, self.weight, self.variance_epsilon, buffers.norm_output)


class FluxPackedLlamaMLP(nn.Module):
    """MLP whose gate and up projections are one ``[gate; up]`` weight
    (``gate_up_proj``); ``state_dict`` keeps ``gate_proj`` / ``up_proj``
    (``smollm2_flux.py:119-235``)."""

    _packing_errors = {"bias": "Flux packed MLP requires bias-free gate/up projections",
                       "requires_grad": "gate/up projection weights must agree on requires_grad"}

    def __init__(self, source: LlamaMLP, *, use_packed_swiglu: bool = False,
                 fuse_gate_up_swiglu: bool = False) -> None:
        super().__init__()
        self.config = source.config
        self.hidden_size = source.hidden_size
        self.intermediate_size = source.intermediate_size
        self.act_fn = source.act_fn
        self.use_packed_swiglu = use_packed_swiglu
        self.fuse_gate_up_swiglu = fuse_gate_up_swiglu
        _PackedWeight(self, "gate_up_proj", (("gate_proj", source.gate_proj), ("up_proj", source.up_proj)),
                      self._packing_errors)
        self.down_proj = source.down_proj

    def _activation(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """silu(gate) * up of the packed projection, by the layer's plan."""
        buffers = _scratch(self)
        if self.fuse_gate_up_swiglu and buffers is not None:
            # one GEMV + SwiGLU launch straight from the hidden state
            return packed_gate_up_swiglu_native_out(hidden_states, self.gate_up_proj.weight, buffers.swiglu_output)
        packed = self.gate_up_proj(hidden_states)
        if not self.use_packed_swiglu:
            gate, up = packed.chunk(2, dim=-1)
            return self.act_fn(gate) * up
        if buffers is not None:
            return packed_swiglu_native_out(packed, buffers.swiglu_output)
        return packed_swiglu_native(packed)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return self.down_proj(self._activation(hidden_states))


# Native one-token projection GEMV for the two decode projection shapes the
# reference routes to its tuned cuBLASLt kernel (smollm2_flux.py:82-116); the
# algorithm fields are accepted for schema compatibility and ignored.
_DECODE_PROJECTION_ALGORITHM = CublasLtAlgorithm(index=-1, algorithm_id=13, tile_id=0, split_k=1,
                                                 reduction_scheme=0, cta_swizzle=0, custom_option=91, stages_id=0,
                                                 workspace_bytes=0, waves_count=0.0)
_DECODE_PROJECTION_SHAPES = frozenset({(960, 576), (576, 576)})


def _project(linear: nn.Linear, x: torch.Tensor, buffers, output_name: str, use_gemv: bool) -> torch.Tensor:
    """``linear(x)``, through the native GEMV into the caller's buffer when the
    plan asks for it, the buffers exist and the weight has a decode shape."""
    output = getattr(buffers, output_name, None) if buffers is not None else None
    workspace = getattr(buffers, "projection_workspace", None) if buffers is not None else None
    if not use_gemv or output is None or workspace is None:
        return linear(x)
    if tuple(linear.weight.shape) not in _DECODE_PROJECTION_SHAPES:
        return torch.nn.functional.linear(x, linear.weight)
    return cublaslt_linear_config_out(x, linear.weight, output, workspace, _DECODE_PROJECTION_ALGORITHM)


class FluxLlamaAttention(LlamaAttention):
    """Llama attention whose RoPE, softmax, one-token GQA attention and
    packed-QKV cache update run on Flux operators (``smollm2_flux.py:266-680``).

    A call takes one of three routes, chosen per call:
      fused  -- packed QKV GEMV, then RoPE + compact cache write in one op
                (``_fused_cache_target``), then native GQA decode attention;
      decode -- the usual projection / RoPE / cache update, then native GQA
                decode attention (``_gqa_eligible``);
      eager  -- the Llama eager attention around the Flux softmax ops.
    """

    _packing_errors = {"bias": "Flux packed QKV requires bias-free projections",
                       "requires_grad": "Q/K/V projection weights must agree on requires_grad"}

    def __init__(self, source: LlamaAttention, *, use_rope: bool = True, use_softmax: bool = True,
                 fuse_attention_scores: bool = True, use_gqa_decode_attention: bool = False,
                 use_packed_qkv: bool = False, use_packed_qkv_rope_cache: bool = False,
                 use_cublaslt_projection: bool = False) -> None:
        nn.Module.__init__(self)
        for name in ("config", "layer_idx", "head_dim", "num_key_value_groups", "scaling", "attention_dropout",
                     "is_causal"):
            setattr(self, name, getattr(source, name))
        self.use_rope = use_rope
        self.use_softmax = use_softmax
        self.fuse_attention_scores = fuse_attention_scores
        self.use_gqa_decode_attention = use_gqa_decode_attention
        self.use_packed_qkv = use_packed_qkv
        self.use_packed_qkv_rope_cache = use_packed_qkv_rope_cache
        self.use_cublaslt_projection = use_cublaslt_projection
        q, k, v = source.q_proj, source.k_proj, source.v_proj
        if use_packed_qkv:
            self._check_packable(q, k, v)
            self.query_width, self.key_width, self.value_width = q.out_features, k.out_features, v.out_features
            self.query_heads = self.query_width // self.head_dim
            self.key_value_heads = self.key_width // self.head_dim
            _PackedWeight(self, "packed_qkv", (("q_proj", q), ("k_proj", k), ("v_proj", v)), self._packing_errors)
        else:
            self.q_proj, self.k_proj, self.v_proj = q, k, v
        self.o_proj = source.o_proj

    def _check_packable(self, q: nn.Linear, k: nn.Linear, v: nn.Linear) -> None:
        projections = (q, k, v)
        if any(p.bias is not None for p in projections):
            raise ValueError(self._packing_errors["bias"])
        agree = {"input width": {p.in_features for p in projections},
                 "dtype": {p.weight.dtype for p in projections},
                 "device": {p.weight.device for p in projections}}
        messages = {"input width": "Q/K/V projections must have the same input width",
                    "dtype": "Q/K/V projection weights must have the same dtype",
                    "device": "Q/K/V projection weights must be on the same device"}
        for what, values in agree.items():
            if len(values) != 1:
                raise ValueError(messages[what])
        if len({p.weight.requires_grad for p in projections}) != 1:
            raise ValueError(self._packing_errors["requires_grad"])
        if q.out_features % self.head_dim or k.out_features % self.head_dim:
            raise ValueError("Q/K projection widths must be divisible by head_dim")
        if v.out_features != k.out_features:
            raise ValueError("K/V projection widths must match")

    # ---------------------------------------------------------------- routes

    def project_qkv(self, hidden_states: torch.Tensor):
        """Head-major Q/K/V views ``[B, heads, S, head_dim]`` of one projection
        (the packed case splits one output, no extra allocation)."""
        lead = hidden_states.shape[:-1]
        if not self.use_packed_qkv:
            return tuple(p(hidden_states).view(*lead, -1, self.head_dim).transpose(1, 2)
                         for p in (self.q_proj, self.k_proj, self.v_proj))
        parts = self.packed_qkv(hidden_states).split((self.query_width, self.key_width, self.value_width), dim=-1)
        heads = (self.query_heads, self.key_value_heads, self.key_value_heads)
        return tuple(p.view(*lead, h, self.head_dim).transpose(1, 2) for p, h in zip(parts, heads))

    def _fused_cache_target(self, hidden_states, cos, sin, attention_mask, past_key_values, kwargs):
        """``(cache layer, device length)`` when the fused packed-QKV / RoPE /
        cache branch applies to this call, else None."""
        if not self.use_packed_qkv_rope_cache or not isinstance(past_key_values, StaticCache):
            return None
        layer = past_key_values.layers[self.layer_idx]
        keys, values = getattr(layer, "keys", None), getattr(layer, "values", None)
        length = getattr(layer, "cumulative_length", None)
        if not getattr(layer, "is_initialized", False) or keys is None or values is None or length is None:
            return None
        if kwargs.get("output_attentions", False):
            return None
        if any(getattr(self, name) != want for name, want in _FUSED_DECODE_WIDTHS.items()):
            return None
        device = hidden_states.device
        capacity = keys.shape[2] if keys.ndim == 4 else -1
        if device.type != "cuda" or not _MIN_GRAPH_CAPACITY <= capacity <= _MAX_DECODE_CAPACITY:
            return None
        tensors = {"hidden": hidden_states, "cos": cos, "sin": sin, "keys": keys, "values": values,
                   "length": length}
        for name, tensor in tensors.items():
            wanted_dtype = torch.int64 if name == "length" else torch.float32
            if (tensor.dtype != wanted_dtype or tensor.device != device
                    or not _shape_matches(tensor, _FUSED_DECODE_SHAPES[name], capacity)):
                return None
        if not _mask_ok(attention_mask, device, (1, 9, 1, capacity)):
            return None
        return layer, length

    def _gqa_eligible(self, query, keys, values, attention_mask, past_key_values, cache_length, kwargs) -> bool:
        """One-token batch-1 FP32 attention over a cache of at most 8192 rows
        (at least 513 when the cache length lives on the device)."""
        if not self.use_gqa_decode_attention or past_key_values is None or kwargs.get("output_attentions", False):
            return False
        if not (query.ndim == keys.ndim == values.ndim == 4) or keys.shape != values.shape:
            return False
        if {query.dtype, keys.dtype, values.dtype} != {torch.float32}:
            return False
        batch, heads, steps, width = query.shape
        capacity = keys.shape[-2]
        if batch != 1 or steps != 1 or keys.shape[0] != batch or keys.shape[-1] != width:
            return False
        if keys.shape[1] <= 0 or heads % keys.shape[1] or capacity > _MAX_DECODE_CAPACITY:
            return False
        if cache_length is not None and capacity < _MIN_GRAPH_CAPACITY:
            return False
        return _mask_ok(attention_mask, query.device, (batch, heads, 1, capacity))

    def _eager_attention(self, query, keys, values, attention_mask):
        """Llama eager attention with the Flux softmax (``smollm2_flux.py:636-680``)."""
        keys = repeat_kv(keys, self.num_key_value_groups)
        values = repeat_kv(values, self.num_key_value_groups)
        scores = torch.matmul(query, keys.transpose(2, 3))
        if self.use_softmax and self.fuse_attention_scores and attention_mask is not None and query.shape[-2] > 1:
            weights = attention_score_softmax_native(scores, attention_mask, self.scaling)
        else:
            scores = scores * self.scaling
            if attention_mask is not None:
                scores = scores + attention_mask
            if self.use_softmax:
                weights = softmax_native(scores)
            else:
                weights = torch.nn.functional.softmax(scores, dim=-1, dtype=torch.float32).to(query.dtype)
                weights = torch.nn.functional.dropout(weights, p=self.attention_dropout, training=self.training)
        return torch.matmul(weights, values).transpose(1, 2).contiguous(), weights

    def forward(self, hidden_states: torch.Tensor, position_embeddings=None, attention_mask=None,
                past_key_values=None, **kwargs: Any):
        if position_embeddings is None:
            raise ValueError("position_embeddings must be provided")
        cos, sin = position_embeddings
        lead = hidden_states.shape[:-1]
        buffers = _scratch(self)
        fused = self._fused_cache_target(hidden_states, cos, sin, attention_mask, past_key_values, kwargs)
        if fused is not None:
            layer, cache_length = fused
            packed = _project(self.packed_qkv, hidden_states, buffers, "qkv_projection_output",
                              self.use_cublaslt_projection)
            if buffers is None:
                query = packed_qkv_rope_cache_native(packed, cos, sin, layer.keys, layer.values, cache_length)
            else:
                query = packed_qkv_rope_cache_native_out(packed, cos, sin, layer.keys, layer.values, cache_length,
                                                         buffers.query_output)
            keys, values = layer.keys, layer.values
        else:
            query, keys, values = self.project_qkv(hidden_states)
            rotate = rope_native if self.use_rope else apply_rotary_pos_emb
            query, keys = rotate(query, keys, cos, sin)
            cache_length = None
            if past_key_values is not None:
                keys, values = past_key_values.update(keys, values, self.layer_idx)
                cache_length = getattr(past_key_values.layers[self.layer_idx], "cumulative_length", None)

        if self._gqa_eligible(query, keys, values, attention_mask, past_key_values, cache_length, kwargs):
            if buffers is None:
                attended = gqa_decode_attention_native(query, keys, values, attention_mask, self.scaling,
                                                       cache_length)
            else:
                attended = gqa_decode_attention_native_out(query, keys, values, attention_mask, self.scaling,
                                                           cache_length, buffers.attention_output,
                                                           buffers.attention_workspace)
            merged = attended.transpose(1, 2).contiguous().reshape(*lead, -1).contiguous()
            return _project(self.o_proj, merged, buffers, "attention_projection_output",
                            self.use_cublaslt_projection), None
        if fused is not None:
            # the cache row is already written; the eager route would write it again
            raise RuntimeError("fused packed-QKV cache update requires native GQA decode attention")
        attended, weights = self._eager_attention(query, keys, values, attention_mask)
        return self.o_proj(attended.reshape(*lead, -1).contiguous()), weights


class FluxLlamaDecoderLayer(LlamaDecoderLayer):
    """Decoder layer whose residual add and post-attention RMSNorm are one
    ``residual_rmsnorm`` op (``smollm2_flux.py:683-787``)."""

    def __init__(self, source: LlamaDecoderLayer, *, use_rmsnorm: bool = True, use_residual_rmsnorm: bool = True,
                 use_rope: bool = True, use_softmax: bool = True, fuse_attention_scores: bool = True,
                 use_gqa_decode_attention: bool = False, use_packed_qkv_rope_cache: bool = False,
                 use_cublaslt_projection: bool = False, use_packed_mlp: bool = False,
                 use_packed_swiglu: bool = False, fuse_gate_up_swiglu: bool = False,
                 use_packed_qkv: bool = False) -> None:
        nn.Module.__init__(self)
        plan = LayerPlan(rmsnorm=use_rmsnorm, residual_rmsnorm=use_residual_rmsnorm, rope=use_rope,
                         softmax=use_softmax, fuse_attention_scores=fuse_attention_scores,
                         gqa_decode_attention=use_gqa_decode_attention, packed_qkv=use_packed_qkv,
                         packed_qkv_rope_cache=use_packed_qkv_rope_cache,
                         cublaslt_projection=use_cublaslt_projection, packed_mlp=use_packed_mlp,
                         packed_swiglu=use_packed_swiglu, fused_gate_up_swiglu=fuse_gate_up_swiglu)
        self.hidden_size = source.hidden_size
        self.use_residual_rmsnorm = use_residual_rmsnorm
        for name, module in _flux_submodules(source, plan).items():
            setattr(self, name, module)

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None, use_cache=False,
                position_embeddings=None, **kwargs: Any):
        residual = hidden_states
        attended, _ = self.self_attn(hidden_states=self.input_layernorm(hidden_states), attention_mask=attention_mask,
                                     position_ids=position_ids, past_key_values=past_key_values,
                                     use_cache=use_cache, position_embeddings=position_embeddings, **kwargs)
        if not self.use_residual_rmsnorm:
            residual = residual + attended
            return residual + self.mlp(self.post_attention_layernorm(residual))
        norm = self.post_attention_layernorm
        buffers = _scratch(self)
        if buffers is None:
            normed, residual = residual_rmsnorm_native(attended, residual, norm.weight, norm.variance_epsilon)
        else:
            normed, residual = residual_rmsnorm_native_out(attended, residual, norm.weight, norm.variance_epsilon,
                                                           buffers.norm_output, buffers.residual_output)
        return residual + self.mlp(normed)


def _flux_submodules(layer: LlamaDecoderLayer, plan: LayerPlan) -> dict[str, nn.Module]:
    """``layer``'s attention, MLP and norms as ``plan`` runs them: Flux modules
    where the plan replaces one (sharing the source parameters, or packing
    them), the source module otherwise.  ``layer`` itself is left unchanged."""
    attention, mlp = layer.self_attn, layer.mlp
    norms = (layer.input_layernorm, layer.post_attention_layernorm)
    if plan.replaces_attention:
        attention = FluxLlamaAttention(
            attention, use_rope=plan.rope, use_softmax=plan.softmax,
            fuse_attention_scores=plan.fuse_attention_scores, use_gqa_decode_attention=plan.gqa_decode_attention,
            use_packed_qkv=plan.packed_qkv, use_packed_qkv_rope_cache=plan.packed_qkv_rope_cache,
            use_cublaslt_projection=plan.cublaslt_projection)
    if plan.packed_mlp:
        mlp = FluxPackedLlamaMLP(mlp, use_packed_swiglu=plan.packed_swiglu,
                                 fuse_gate_up_swiglu=plan.fused_gate_up_swiglu)
    if plan.rmsnorm:
        norms = tuple(FluxRMSNorm(norm) for norm in norms)
    return {"self_attn": attention, "mlp": mlp, "input_layernorm": norms[0], "post_attention_layernorm": norms[1]}


# ---------------------------------------------------------------- enabling


def _validate_categories(selected: frozenset[str]) -> None:
    unknown = selected - FINAL_FLUX_OPERATOR_CATEGORIES
    if unknown:
        raise ValueError(f"unknown Flux operator categories: {sorted(unknown)}")
    if not selected:
        raise ValueError("at least one Flux operator category must be selected")
    for category, needs, message in _CATEGORY_RULES:
        if category in selected and not needs <= selected:
            raise ValueError(message)


def _validate_model(model: nn.Module) -> LlamaForCausalLM:
    if not isinstance(model, LlamaForCausalLM):
        raise TypeError("Flux SmolLM2 integration requires LlamaForCausalLM")
    if model.training:
        raise ValueError("Flux custom operators are inference-only; call model.eval() first")
    if getattr(model, "_flux_ops_enabled", False):
        raise ValueError("Flux custom operators are already enabled on this model")
    dtypes = {p.dtype for p in model.parameters() if p.is_floating_point()}
    if dtypes != {torch.float32}:
        raise TypeError("Flux SmolLM2 integration currently requires all floating-point parameters to be "
                        f"torch.float32, found {sorted(map(str, dtypes))}")
    if not all(isinstance(layer, LlamaDecoderLayer) for layer in model.model.layers):
        raise TypeError("model contains a decoder layer unsupported by Flux integration")
    if not isinstance(model.model.norm, LlamaRMSNorm):
        raise TypeError("model final norm is not LlamaRMSNorm")
    return model


def _missing_native_operators(selected: frozenset[str], fuse_attention_scores: bool) -> list[str]:
    active = set(selected)
    if "softmax" in selected and fuse_attention_scores:
        active.add("softmax+scores")
    probes = globals()
    return [name for category, name, probe in _NATIVE_PROBES if category in active and not probes[probe]()]


def enable_flux_ops(model: nn.Module, *, operators: Collection[str] = FLUX_OPERATOR_CATEGORIES,
                    fuse_attention_scores: bool = True) -> LlamaForCausalLM:
    """Switch an evaluated FP32 Llama causal LM to Flux operators in place and
    return the same instance (``smollm2_flux.py:869-1034``)."""
    selected = frozenset(operators)
    _validate_categories(selected)
    llama = _validate_model(model)
    missing = _missing_native_operators(selected, fuse_attention_scores)
    if missing:
        raise RuntimeError("Flux native operators are not built: " + ", ".join(missing)
                           + ". Build the extension before enabling the model path.")
    plan = LayerPlan.from_categories(selected, fuse_attention_scores)
    layers = llama.model.layers
    for index in range(len(layers)):  # one layer at a time: packed copies never double the whole model
        if plan.residual_rmsnorm:
            layers[index] = FluxLlamaDecoderLayer(
                layers[index], use_rmsnorm=plan.rmsnorm, use_residual_rmsnorm=True, use_rope=plan.rope,
                use_softmax=plan.softmax, fuse_attention_scores=plan.fuse_attention_scores,
                use_gqa_decode_attention=plan.gqa_decode_attention, use_packed_qkv=plan.packed_qkv,
                use_packed_qkv_rope_cache=plan.packed_qkv_rope_cache,
                use_cublaslt_projection=plan.cublaslt_projection, use_packed_mlp=plan.packed_mlp,
                use_packed_swiglu=plan.packed_swiglu, fuse_gate_up_swiglu=plan.fused_gate_up_swiglu)
        else:
            for name, module in _flux_submodules(layers[index], plan).items():
                setattr(layers[index], name, module)
    if plan.rmsnorm:
        llama.model.norm = FluxRMSNorm(llama.model.norm)
    for module in (llama, llama.model):  # let transformers re-install its output hooks on the new modules
        if hasattr(module, "_output_capturing_hooks_installed"):
            module._output_capturing_hooks_installed = False
    markers = {
        "ops_enabled": True,
        "operator_categories": tuple(sorted(selected)),
        "attention_score_fusion_enabled": plan.softmax and plan.fuse_attention_scores,
        "gqa_decode_attention_enabled": plan.gqa_decode_attention,
        "packed_mlp_enabled": plan.packed_mlp,
        "packed_swiglu_enabled": plan.packed_swiglu,
        "packed_qkv_enabled": plan.packed_qkv,
        "packed_qkv_rope_cache_enabled": plan.packed_qkv_rope_cache,
        "cublaslt_projection_enabled": plan.cublaslt_projection,
        "fused_gate_up_swiglu_enabled": plan.fused_gate_up_swiglu,
    }
    for name, value in markers.items():
        setattr(llama, f"_flux_{name}", value)
    return llama


def flux_operator_counts(model: nn.Module) -> dict[str, int]:
    """How many Flux modules of each kind are installed (diagnostics;
    ``smollm2_flux.py:1037-1077``)."""
    modules = list(model.modules())
    attention = [m for m in modules if isinstance(m, FluxLlamaAttention)]
    mlps = [m for m in modules if isinstance(m, FluxPackedLlamaMLP)]

    def count(kind) -> int:
        return sum(isinstance(m, kind) for m in modules)

    return {
        "decoder_layers": count(FluxLlamaDecoderLayer),
        "rmsnorm_modules": count(FluxRMSNorm),
        "attention_modules": len(attention),
        "packed_mlp_modules": len(mlps),
        "packed_qkv_modules": sum(m.use_packed_qkv for m in attention),
        "gqa_decode_attention_modules": sum(m.use_gqa_decode_attention for m in attention),
        "packed_qkv_rope_cache_modules": sum(m.use_packed_qkv_rope_cache for m in attention),
        "cublaslt_projection_modules": sum(m.use_cublaslt_projection for m in attention),
        "fused_gate_up_swiglu_modules": sum(m.fuse_gate_up_swiglu for m in mlps),
    }


__all__ = [
    "FINAL_FLUX_OPERATOR_CATEGORIES", "FLUX_OPERATOR_CATEGORIES", "FLUX_CUBLASLT_PROJECTION_CATEGORY",
    "FLUX_GQA_DECODE_ATTENTION_CATEGORY", "FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY", "FLUX_PACKED_MLP_CATEGORY",
    "FLUX_PACKED_QKV_CATEGORY", "FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY", "FLUX_PACKED_SWIGLU_CATEGORY",
    "FluxLlamaAttention", "FluxLlamaDecoderLayer", "FluxPackedLlamaMLP", "FluxRMSNorm", "LayerPlan",
    "enable_flux_ops", "flux_operator_counts",
]
