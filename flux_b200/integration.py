"""``enable_flux_ops``: the reference's operator-category surface on flux_b200.

Mirrors ``flux/model/smollm2_flux.py`` (module replacement per model instance,
packed QKV / gate-up parameters with state-dict hooks that keep the standard
Llama checkpoint keys, decode-only fused branches) with every native call
routed to the ``torch.ops.flux.*`` kernels of :mod:`flux_b200.operators`.
The native calls are looked up as module globals at call time, so a caller may
monkeypatch them (the reference tests do, ``tests/test_system.py:57-133``).
"""

from __future__ import annotations

from collections.abc import Collection
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

# Categories (smollm2_flux.py:58-80).
FLUX_OPERATOR_CATEGORIES = frozenset({"rmsnorm", "residual_rmsnorm", "rope", "softmax"})
FLUX_PACKED_MLP_CATEGORY = "mlp"
FLUX_PACKED_SWIGLU_CATEGORY = "packed_swiglu"
FLUX_PACKED_QKV_CATEGORY = "qkv"
FLUX_GQA_DECODE_ATTENTION_CATEGORY = "gqa_decode_attention"
FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY = "packed_qkv_rope_cache"
FLUX_CUBLASLT_PROJECTION_CATEGORY = "cublaslt_projection"
FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY = "fused_gate_up_swiglu"
_SUPPORTED_OPERATOR_CATEGORIES = FLUX_OPERATOR_CATEGORIES | {
    FLUX_GQA_DECODE_ATTENTION_CATEGORY,
    FLUX_PACKED_MLP_CATEGORY,
    FLUX_PACKED_SWIGLU_CATEGORY,
    FLUX_PACKED_QKV_CATEGORY,
    FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY,
    FLUX_CUBLASLT_PROJECTION_CATEGORY,
    FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY,
}
FINAL_FLUX_OPERATOR_CATEGORIES = _SUPPORTED_OPERATOR_CATEGORIES
_GQA_DECODE_GRAPH_MINIMUM_CAPACITY = 513
_DECODE_PROJECTION = CublasLtAlgorithm(index=-1, algorithm_id=13, tile_id=0, split_k=1, reduction_scheme=0,
                                       cta_swizzle=0, custom_option=91, stages_id=0, workspace_bytes=0,
                                       waves_count=0.0)
_DECODE_PROJECTION_SHAPES = {(960, 576), (576, 576)}


def _decode_projection_out(input, weight, output, workspace):
    """Exact decode projection shapes use the native GEMV; others stay nn.Linear
    (``smollm2_flux.py:100-116``)."""
    if tuple(weight.shape) not in _DECODE_PROJECTION_SHAPES:
        return torch.nn.functional.linear(input, weight)
    return cublaslt_linear_config_out(input, weight, output, workspace, _DECODE_PROJECTION)


def _packed_parameter(sources: list[torch.Tensor], requires_grad: bool) -> nn.Parameter:
    return nn.Parameter(torch.cat(sources, dim=0), requires_grad=requires_grad)


class FluxPackedLlamaMLP(nn.Module):
    """MLP owning one ``[gate; up]`` parameter (``smollm2_flux.py:119-235``).

    ``state_dict`` still reports ``gate_proj.weight`` / ``up_proj.weight``."""

    def __init__(self, source: LlamaMLP, *, use_packed_swiglu: bool = False,
                 fuse_gate_up_swiglu: bool = False) -> None:
        super().__init__()
        if source.gate_proj.bias is not None or source.up_proj.bias is not None:
            raise ValueError("Flux packed MLP requires bias-free gate/up projections")
        if source.gate_proj.weight.requires_grad != source.up_proj.weight.requires_grad:
            raise ValueError("gate/up projection weights must agree on requires_grad")
        self.config = source.config
        self.hidden_size = source.hidden_size
        self.intermediate_size = source.intermediate_size
        self.act_fn = source.act_fn
        self.down_proj = source.down_proj
        self.use_packed_swiglu = use_packed_swiglu
        self.fuse_gate_up_swiglu = fuse_gate_up_swiglu
        self.gate_up_proj = nn.Linear(self.hidden_size, 2 * self.intermediate_size, bias=False, device="meta",
                                      dtype=source.gate_proj.weight.dtype)
        self.gate_up_proj.weight = _packed_parameter([source.gate_proj.weight, source.up_proj.weight],
                                                     source.gate_proj.weight.requires_grad)
        self.register_state_dict_post_hook(FluxPackedLlamaMLP._unpack_state_dict_hook)
        self.register_load_state_dict_pre_hook(FluxPackedLlamaMLP._pack_state_dict_hook)

    @staticmethod
    def _unpack_state_dict_hook(module, state_dict, prefix, _local_metadata) -> None:
        packed = state_dict.pop(prefix + "gate_up_proj.weight", None)
        if packed is None:
            return
        gate, up = packed.split(module.intermediate_size, dim=0)
        state_dict[prefix + "gate_proj.weight"] = gate
        state_dict[prefix + "up_proj.weight"] = up

    @staticmethod
    def _pack_state_dict_hook(_module, state_dict, prefix, *_args) -> None:
        packed, gate, up = (prefix + n for n in ("gate_up_proj.weight", "gate_proj.weight", "up_proj.weight"))
        if packed in state_dict or gate not in state_dict or up not in state_dict:
            return
        state_dict[packed] = torch.cat((state_dict.pop(gate), state_dict.pop(up)), dim=0)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        scratch = getattr(self, "_flux_decode_scratch", None)
        if self.fuse_gate_up_swiglu and scratch is not None:
            return self.down_proj(packed_gate_up_swiglu_native_out(hidden_states, self.gate_up_proj.weight,
                                                                   scratch.swiglu_output))
        gate_up = self.gate_up_proj(hidden_states)
        if self.use_packed_swiglu:
            if scratch is not None:
                return self.down_proj(packed_swiglu_native_out(gate_up, scratch.swiglu_output))
            return self.down_proj(packed_swiglu_native(gate_up))
        gate, up = gate_up.chunk(2, dim=-1)
        return self.down_proj(self.act_fn(gate) * up)


class FluxRMSNorm(LlamaRMSNorm):
    """``LlamaRMSNorm`` on ``torch.ops.flux.rmsnorm``; reuses the source Parameter
    so names and tying are unchanged (``smollm2_flux.py:238-263``)."""

    def __init__(self, source: LlamaRMSNorm) -> None:
        nn.Module.__init__(self)
        self.weight = source.weight
        self.variance_epsilon = source.variance_epsilon

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        scratch = getattr(self, "_flux_decode_scratch", None)
        if scratch is not None:
            return rms_norm_native_out(hidden_states, self.weight, self.variance_epsilon, scratch.norm_output)
        return rms_norm_native(hidden_states, self.weight, self.variance_epsilon)


def _mask_broadcasts(mask, target) -> bool:
    return (mask.ndim == 4 and mask.dtype == torch.float32
            and all(m in (1, t) for m, t in zip(mask.shape, target, strict=True)))


class FluxLlamaAttention(LlamaAttention):
    """Llama eager attention with Flux operators (``smollm2_flux.py:266-680``)."""

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
        projections = (source.q_proj, source.k_proj, source.v_proj)
        if use_packed_qkv:
            if any(p.bias is not None for p in projections):
                raise ValueError("Flux packed QKV requires bias-free projections")
            if len({p.in_features for p in projections}) != 1:
                raise ValueError("Q/K/V projections must have the same input width")
            if len({p.weight.dtype for p in projections}) != 1:
                raise ValueError("Q/K/V projection weights must have the same dtype")
            if len({p.weight.device for p in projections}) != 1:
                raise ValueError("Q/K/V projection weights must be on the same device")
            if len({p.weight.requires_grad for p in projections}) != 1:
                raise ValueError("Q/K/V projection weights must agree on requires_grad")
            self.query_width = source.q_proj.out_features
            self.key_width = source.k_proj.out_features
            self.value_width = source.v_proj.out_features
            self.query_heads = self.query_width // self.head_dim
            self.key_value_heads = self.key_width // self.head_dim
            if self.query_width % self.head_dim or self.key_width % self.head_dim:
                raise ValueError("Q/K projection widths must be divisible by head_dim")
            if self.value_width != self.key_width:
                raise ValueError("K/V projection widths must match")
            width = self.query_width + self.key_width + self.value_width
            self.packed_qkv = nn.Linear(source.q_proj.in_features, width, bias=False, device="meta",
                                        dtype=source.q_proj.weight.dtype)
            self.packed_qkv.weight = _packed_parameter([p.weight for p in projections],
                                                       source.q_proj.weight.requires_grad)
            self.register_state_dict_post_hook(FluxLlamaAttention._unpack_qkv_state_dict_hook)
            self.register_load_state_dict_pre_hook(FluxLlamaAttention._pack_qkv_state_dict_hook)
        else:
            self.q_proj, self.k_proj, self.v_proj = projections
        self.o_proj = source.o_proj

    @staticmethod
    def _unpack_qkv_state_dict_hook(module, state_dict, prefix, _local_metadata) -> None:
        packed = state_dict.pop(prefix + "packed_qkv.weight", None)
        if packed is None:
            return
        q, k, v = packed.split((module.query_width, module.key_width, module.value_width), dim=0)
        state_dict[prefix + "q_proj.weight"] = q
        state_dict[prefix + "k_proj.weight"] = k
        state_dict[prefix + "v_proj.weight"] = v

    @staticmethod
    def _pack_qkv_state_dict_hook(_module, state_dict, prefix, *_args) -> None:
        packed = prefix + "packed_qkv.weight"
        keys = tuple(prefix + n for n in ("q_proj.weight", "k_proj.weight", "v_proj.weight"))
        if packed in state_dict or not all(k in state_dict for k in keys):
            return
        state_dict[packed] = torch.cat(tuple(state_dict.pop(k) for k in keys), dim=0)

    def project_qkv(self, hidden_states: torch.Tensor):
        """Head-major Q/K/V views of one projection (no extra allocation)."""
        input_shape = hidden_states.shape[:-1]
        if self.use_packed_qkv:
            q, k, v = self.packed_qkv(hidden_states).split((self.query_width, self.key_width, self.value_width),
                                                           dim=-1)
            return (q.view(*input_shape, self.query_heads, self.head_dim).transpose(1, 2),
                    k.view(*input_shape, self.key_value_heads, self.head_dim).transpose(1, 2),
                    v.view(*input_shape, self.key_value_heads, self.head_dim).transpose(1, 2))
        shape = (*input_shape, -1, self.head_dim)
        return (self.q_proj(hidden_states).view(shape).transpose(1, 2),
                self.k_proj(hidden_states).view(shape).transpose(1, 2),
                self.v_proj(hidden_states).view(shape).transpose(1, 2))

    def _fused_cache_layer(self, hidden_states, cos, sin, attention_mask, past_key_values, kwargs):
        """The StaticCache layer when the packed-QKV/RoPE/cache branch applies
        (``smollm2_flux.py:441-489``), else None."""
        if not self.use_packed_qkv_rope_cache or not isinstance(past_key_values, StaticCache):
            return None
        layer = past_key_values.layers[self.layer_idx]
        length = getattr(layer, "cumulative_length", None)
        keys, values = getattr(layer, "keys", None), getattr(layer, "values", None)
        device = hidden_states.device
        ok = (getattr(layer, "is_initialized", False) and tuple(hidden_states.shape) == (1, 1, 576)
              and hidden_states.dtype == torch.float32 and device.type == "cuda"
              and tuple(cos.shape) == tuple(sin.shape) == (1, 1, 64) and cos.dtype == sin.dtype == torch.float32
              and cos.device == sin.device == device
              and self.query_width == 576 and self.key_width == self.value_width == 192
              and self.query_heads == 9 and self.key_value_heads == 3 and self.head_dim == 64
              and keys is not None and values is not None and keys.shape == values.shape
              and keys.shape[0] == 1 and keys.shape[1] == 3
              and _GQA_DECODE_GRAPH_MINIMUM_CAPACITY <= keys.shape[2] <= 8192 and keys.shape[3] == 64
              and keys.dtype == values.dtype == torch.float32 and keys.device == values.device == device
              and length is not None and length.shape == () and length.dtype == torch.int64
              and length.device == device
              and (attention_mask is None or (attention_mask.device == device
                                              and _mask_broadcasts(attention_mask, (1, 9, 1, keys.shape[2]))))
              and not kwargs.get("output_attentions", False))
        return (layer, length) if ok else None

    def forward(self, hidden_states: torch.Tensor, position_embeddings=None, attention_mask=None,
                past_key_values=None, **kwargs: Any):
        if position_embeddings is None:
            raise ValueError("position_embeddings must be provided")
        cos, sin = position_embeddings
        input_shape = hidden_states.shape[:-1]
        scratch = getattr(self, "_flux_decode_scratch", None)
        cache_length = None
        fused = self._fused_cache_layer(hidden_states, cos, sin, attention_mask, past_key_values, kwargs)
        if fused is not None:
            layer, cache_length = fused
            if (self.use_cublaslt_projection and scratch is not None
                    and scratch.qkv_projection_output is not None and scratch.projection_workspace is not None):
                packed = _decode_projection_out(hidden_states, self.packed_qkv.weight, scratch.qkv_projection_output,
                                                scratch.projection_workspace)
            else:
                packed = self.packed_qkv(hidden_states)
            if scratch is None:
                query_states = packed_qkv_rope_cache_native(packed, cos, sin, layer.keys, layer.values, cache_length)
            else:
                query_states = packed_qkv_rope_cache_native_out(packed, cos, sin, layer.keys, layer.values,
                                                                cache_length, scratch.query_output)
            key_states, value_states = layer.keys, layer.values
        else:
            query_states, key_states, value_states = self.project_qkv(hidden_states)
            if self.use_rope:
                query_states, key_states = rope_native(query_states, key_states, cos, sin)
            else:
                query_states, key_states = apply_rotary_pos_emb(query_states, key_states, cos, sin)
            if past_key_values is not None:
                key_states, value_states = past_key_values.update(key_states, value_states, self.layer_idx)
                cache_length = getattr(past_key_values.layers[self.layer_idx], "cumulative_length", None)

        capacity = key_states.shape[-2]
        if (self.use_gqa_decode_attention and past_key_values is not None
                and query_states.shape[0] == 1 and query_states.shape[-2] == 1
                and query_states.dtype == key_states.dtype == value_states.dtype == torch.float32
                and query_states.ndim == key_states.ndim == value_states.ndim == 4
                and key_states.shape == value_states.shape and query_states.shape[0] == key_states.shape[0]
                and query_states.shape[-1] == key_states.shape[-1] and key_states.shape[1] > 0
                and query_states.shape[1] % key_states.shape[1] == 0 and capacity <= 8192
                and (cache_length is None or capacity >= _GQA_DECODE_GRAPH_MINIMUM_CAPACITY)
                and (attention_mask is None or (attention_mask.device == query_states.device and _mask_broadcasts(
                    attention_mask, (query_states.shape[0], query_states.shape[1], 1, capacity))))
                and not kwargs.get("output_attentions", False)):
            if scratch is None:
                attn = gqa_decode_attention_native(query_states, key_states, value_states, attention_mask,
                                                   self.scaling, cache_length)
            else:
                attn = gqa_decode_attention_native_out(query_states, key_states, value_states, attention_mask,
                                                       self.scaling, cache_length, scratch.attention_output,
                                                       scratch.attention_workspace)
            attn = attn.transpose(1, 2).contiguous().reshape(*input_shape, -1).contiguous()
            if (self.use_cublaslt_projection and scratch is not None
                    and scratch.attention_projection_output is not None and scratch.projection_workspace is not None):
                return _decode_projection_out(attn, self.o_proj.weight, scratch.attention_projection_output,
                                              scratch.projection_workspace), None
            return self.o_proj(attn), None
        if fused is not None:
            raise RuntimeError("fused packed-QKV cache update requires native GQA decode attention")

        # Llama eager attention around the Flux softmax (smollm2_flux.py:636-680).
        key_states = repeat_kv(key_states, self.num_key_value_groups)
        value_states = repeat_kv(value_states, self.num_key_value_groups)
        weights = torch.matmul(query_states, key_states.transpose(2, 3))
        if self.use_softmax and self.fuse_attention_scores and attention_mask is not None \
                and query_states.shape[-2] > 1:
            weights = attention_score_softmax_native(weights, attention_mask, self.scaling)
        elif self.use_softmax:
            weights = weights * self.scaling
            if attention_mask is not None:
                weights = weights + attention_mask
            weights = softmax_native(weights)
        else:
            weights = weights * self.scaling
            if attention_mask is not None:
                weights = weights + attention_mask
            weights = torch.nn.functional.softmax(weights, dim=-1, dtype=torch.float32).to(query_states.dtype)
            weights = torch.nn.functional.dropout(weights, p=self.attention_dropout, training=self.training)
        out = torch.matmul(weights, value_states).transpose(1, 2).contiguous()
        return self.o_proj(out.reshape(*input_shape, -1).contiguous()), weights


class FluxLlamaDecoderLayer(LlamaDecoderLayer):
    """Decoder layer with the fused residual RMSNorm (``smollm2_flux.py:683-787``)."""

    def __init__(self, source: LlamaDecoderLayer, *, use_rmsnorm: bool = True, use_residual_rmsnorm: bool = True,
                 use_rope: bool = True, use_softmax: bool = True, fuse_attention_scores: bool = True,
                 use_gqa_decode_attention: bool = False, use_packed_qkv_rope_cache: bool = False,
                 use_cublaslt_projection: bool = False, use_packed_mlp: bool = False,
                 use_packed_swiglu: bool = False, fuse_gate_up_swiglu: bool = False,
                 use_packed_qkv: bool = False) -> None:
        nn.Module.__init__(self)
        self.hidden_size = source.hidden_size
        if use_softmax or use_rope or use_gqa_decode_attention or use_packed_qkv:
            self.self_attn = FluxLlamaAttention(
                source.self_attn, use_rope=use_rope, use_softmax=use_softmax,
                fuse_attention_scores=fuse_attention_scores, use_gqa_decode_attention=use_gqa_decode_attention,
                use_packed_qkv_rope_cache=use_packed_qkv_rope_cache, use_cublaslt_projection=use_cublaslt_projection,
                use_packed_qkv=use_packed_qkv)
        else:
            self.self_attn = source.self_attn
        self.mlp = (FluxPackedLlamaMLP(source.mlp, use_packed_swiglu=use_packed_swiglu,
                                       fuse_gate_up_swiglu=fuse_gate_up_swiglu) if use_packed_mlp else source.mlp)
        self.input_layernorm = FluxRMSNorm(source.input_layernorm) if use_rmsnorm else source.input_layernorm
        self.post_attention_layernorm = (FluxRMSNorm(source.post_attention_layernorm) if use_rmsnorm
                                         else source.post_attention_layernorm)
        self.use_residual_rmsnorm = use_residual_rmsnorm

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None, use_cache=False,
                position_embeddings=None, **kwargs: Any):
        residual = hidden_states
        hidden_states = self.input_layernorm(hidden_states)
        attention_output, _ = self.self_attn(hidden_states=hidden_states, attention_mask=attention_mask,
                                             position_ids=position_ids, past_key_values=past_key_values,
                                             use_cache=use_cache, position_embeddings=position_embeddings, **kwargs)
        if self.use_residual_rmsnorm:
            scratch = getattr(self, "_flux_decode_scratch", None)
            weight = self.post_attention_layernorm.weight
            eps = self.post_attention_layernorm.variance_epsilon
            if scratch is None:
                hidden_states, residual = residual_rmsnorm_native(attention_output, residual, weight, eps)
            else:
                hidden_states, residual = residual_rmsnorm_native_out(attention_output, residual, weight, eps,
                                                                      scratch.norm_output, scratch.residual_output)
        else:
            residual = residual + attention_output
            hidden_states = self.post_attention_layernorm(residual)
        return residual + self.mlp(hidden_states)


def _check_model(model: nn.Module) -> LlamaForCausalLM:
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


def _check_native_ops(operators: frozenset[str], *, fuse_attention_scores: bool) -> None:
    """``smollm2_flux.py:813-866``; the probes are module globals (patchable)."""
    g = globals()
    needs = [
        ("rmsnorm", "rmsnorm", "native_rmsnorm_is_available"),
        ("residual_rmsnorm", "residual_rmsnorm", "native_residual_rmsnorm_is_available"),
        ("softmax", "softmax", "native_softmax_is_available"),
        ("rope", "rope", "native_rope_is_available"),
        (FLUX_PACKED_SWIGLU_CATEGORY, "packed_swiglu", "native_packed_swiglu_is_available"),
    ]
    missing = [name for category, name, probe in needs if category in operators and not g[probe]()]
    if "softmax" in operators and fuse_attention_scores and not g["native_attention_score_softmax_is_available"]():
        missing.append("attention_score_softmax")
    for category, name, probe in (
            (FLUX_GQA_DECODE_ATTENTION_CATEGORY, "gqa_decode_attention", "native_gqa_decode_attention_is_available"),
            (FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY, "packed_qkv_rope_cache",
             "native_packed_qkv_rope_cache_is_available"),
            (FLUX_CUBLASLT_PROJECTION_CATEGORY, "cublaslt_projection", "native_cublaslt_linear_is_available"),
            (FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY, "gate_up_gemv", "native_packed_gate_up_gemv_is_available")):
        if category in operators and not g[probe]():
            missing.append(name)
    if missing:
        raise RuntimeError("Flux native operators are not built: " + ", ".join(missing)
                           + ". Build the extension before enabling the model path.")


def enable_flux_ops(model: nn.Module, *, operators: Collection[str] = FLUX_OPERATOR_CATEGORIES,
                    fuse_attention_scores: bool = True) -> LlamaForCausalLM:
    """Replace supported modules of an evaluated FP32 Llama causal LM in place
    (``smollm2_flux.py:869-1034``); returns the same model instance."""
    selected = frozenset(operators)
    unknown = selected - _SUPPORTED_OPERATOR_CATEGORIES
    if unknown:
        raise ValueError(f"unknown Flux operator categories: {sorted(unknown)}")
    if not selected:
        raise ValueError("at least one Flux operator category must be selected")
    if FLUX_PACKED_SWIGLU_CATEGORY in selected and FLUX_PACKED_MLP_CATEGORY not in selected:
        raise ValueError('"packed_swiglu" requires the "mlp" operator category')
    if FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY in selected and not {
            "rope", FLUX_PACKED_QKV_CATEGORY, FLUX_GQA_DECODE_ATTENTION_CATEGORY}.issubset(selected):
        raise ValueError('"packed_qkv_rope_cache" requires the "rope", "qkv", and "gqa_decode_attention" '
                         'operator categories')
    if FLUX_CUBLASLT_PROJECTION_CATEGORY in selected and FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY not in selected:
        raise ValueError('"cublaslt_projection" requires the "packed_qkv_rope_cache" operator category')
    if FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY in selected and not {
            FLUX_PACKED_MLP_CATEGORY, FLUX_PACKED_SWIGLU_CATEGORY}.issubset(selected):
        raise ValueError('"fused_gate_up_swiglu" requires the "mlp" and "packed_swiglu" operator categories')
    llama = _check_model(model)
    _check_native_ops(selected, fuse_attention_scores=fuse_attention_scores)
    flags = dict(
        use_rope="rope" in selected, use_softmax="softmax" in selected, fuse_attention_scores=fuse_attention_scores,
        use_gqa_decode_attention=FLUX_GQA_DECODE_ATTENTION_CATEGORY in selected,
        use_packed_qkv_rope_cache=FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY in selected,
        use_cublaslt_projection=FLUX_CUBLASLT_PROJECTION_CATEGORY in selected,
        use_packed_qkv=FLUX_PACKED_QKV_CATEGORY in selected)
    if "residual_rmsnorm" in selected:
        # One layer at a time, so packed copies never duplicate the whole model.
        for index in range(len(llama.model.layers)):
            llama.model.layers[index] = FluxLlamaDecoderLayer(
                llama.model.layers[index], use_rmsnorm="rmsnorm" in selected, use_residual_rmsnorm=True,
                use_packed_mlp=FLUX_PACKED_MLP_CATEGORY in selected,
                use_packed_swiglu=FLUX_PACKED_SWIGLU_CATEGORY in selected,
                fuse_gate_up_swiglu=FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY in selected, **flags)
    else:
        for layer in llama.model.layers:
            if flags["use_softmax"] or flags["use_rope"] or flags["use_packed_qkv"] \
                    or flags["use_gqa_decode_attention"]:
                layer.self_attn = FluxLlamaAttention(
                    layer.self_attn, **{k: v for k, v in flags.items()})
            if "rmsnorm" in selected:
                layer.input_layernorm = FluxRMSNorm(layer.input_layernorm)
                layer.post_attention_layernorm = FluxRMSNorm(layer.post_attention_layernorm)
            if FLUX_PACKED_MLP_CATEGORY in selected:
                layer.mlp = FluxPackedLlamaMLP(layer.mlp, use_packed_swiglu=FLUX_PACKED_SWIGLU_CATEGORY in selected,
                                               fuse_gate_up_swiglu=FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY in selected)
    if "rmsnorm" in selected:
        llama.model.norm = FluxRMSNorm(llama.model.norm)
    for module in (llama, llama.model):
        if hasattr(module, "_output_capturing_hooks_installed"):
            module._output_capturing_hooks_installed = False
    llama._flux_ops_enabled = True
    llama._flux_operator_categories = tuple(sorted(selected))
    llama._flux_attention_score_fusion_enabled = "softmax" in selected and fuse_attention_scores
    llama._flux_gqa_decode_attention_enabled = FLUX_GQA_DECODE_ATTENTION_CATEGORY in selected
    llama._flux_packed_mlp_enabled = FLUX_PACKED_MLP_CATEGORY in selected
    llama._flux_packed_swiglu_enabled = FLUX_PACKED_SWIGLU_CATEGORY in selected
    llama._flux_packed_qkv_enabled = FLUX_PACKED_QKV_CATEGORY in selected
    llama._flux_packed_qkv_rope_cache_enabled = FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY in selected
    llama._flux_cublaslt_projection_enabled = FLUX_CUBLASLT_PROJECTION_CATEGORY in selected
    llama._flux_fused_gate_up_swiglu_enabled = FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY in selected
    return llama


def flux_operator_counts(model: nn.Module) -> dict[str, int]:
    """Installed Flux modules, for diagnostics (``smollm2_flux.py:1037-1077``)."""
    modules = list(model.modules())
    attn = [m for m in modules if isinstance(m, FluxLlamaAttention)]
    mlps = [m for m in modules if isinstance(m, FluxPackedLlamaMLP)]
    return {
        "decoder_layers": sum(isinstance(m, FluxLlamaDecoderLayer) for m in modules),
        "rmsnorm_modules": sum(isinstance(m, FluxRMSNorm) for m in modules),
        "attention_modules": len(attn),
        "packed_mlp_modules": len(mlps),
        "packed_qkv_modules": sum(m.use_packed_qkv for m in attn),
        "gqa_decode_attention_modules": sum(m.use_gqa_decode_attention for m in attn),
        "packed_qkv_rope_cache_modules": sum(m.use_packed_qkv_rope_cache for m in attn),
        "cublaslt_projection_modules": sum(m.use_cublaslt_projection for m in attn),
        "fused_gate_up_swiglu_modules": sum(m.fuse_gate_up_swiglu for m in mlps),
    }


__all__ = [
    "FINAL_FLUX_OPERATOR_CATEGORIES", "FLUX_OPERATOR_CATEGORIES", "FLUX_CUBLASLT_PROJECTION_CATEGORY",
    "FLUX_GQA_DECODE_ATTENTION_CATEGORY", "FLUX_FUSED_GATE_UP_SWIGLU_CATEGORY", "FLUX_PACKED_MLP_CATEGORY",
    "FLUX_PACKED_QKV_CATEGORY", "FLUX_PACKED_QKV_ROPE_CACHE_CATEGORY", "FLUX_PACKED_SWIGLU_CATEGORY",
    "FluxLlamaAttention", "FluxLlamaDecoderLayer", "FluxPackedLlamaMLP", "FluxRMSNorm", "enable_flux_ops",
    "flux_operator_counts",
]
