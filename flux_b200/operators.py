"""``torch.ops.flux.*`` over the flux_b200 C ABI.

Registers the reference's operator schemas verbatim (the ``TORCH_LIBRARY``
blocks of ``csrc/*/*_torch.cpp``) with CUDA kernels from ``libfluxb200.so``,
FakeTensor kernels, and the reference's argument checks and error messages.
A CPU call is validated and then rejected: flux_b200 has no CPU compute path.
The Python entry points keep the reference names of ``flux/ops/native_*.py``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from flux_b200 import _native

FLT_MAX = 3.4028234663852886e38

_LIB = torch.library.Library("flux", "DEF")

_SCHEMAS = {
    # csrc/rmsnorm/rmsnorm_torch.cpp:152-158
    "rmsnorm": "rmsnorm(Tensor input, Tensor weight, float epsilon) -> Tensor",
    "rmsnorm_out": "rmsnorm_out(Tensor input, Tensor weight, float epsilon, Tensor(a!) output) -> Tensor(a!)",
    # csrc/residual_rmsnorm/residual_rmsnorm_torch.cpp:184-192
    "residual_rmsnorm": ("residual_rmsnorm(Tensor hidden, Tensor residual, Tensor weight, float epsilon) -> "
                         "(Tensor norm_out, Tensor residual_out)"),
    "residual_rmsnorm_out": ("residual_rmsnorm_out(Tensor hidden, Tensor residual, Tensor weight, float epsilon, "
                             "Tensor(a!) norm_out, Tensor(b!) residual_out) -> (Tensor(a!), Tensor(b!))"),
    # csrc/packed_swiglu/packed_swiglu_torch.cpp:125-128
    "packed_swiglu": "packed_swiglu(Tensor packed) -> Tensor",
    "packed_swiglu_out": "packed_swiglu_out(Tensor packed, Tensor(a!) output) -> Tensor(a!)",
    # csrc/softmax/softmax_torch.cpp:83-85
    "softmax": "softmax(Tensor input) -> Tensor",
    # csrc/attention_score_softmax/attention_score_softmax_torch.cpp:119-122
    "attention_score_softmax": ("attention_score_softmax(Tensor scores, Tensor additive_attention_mask, "
                                "float scale) -> Tensor"),
    # csrc/rope/rope_torch.cpp:133-136
    "rope": "rope(Tensor query, Tensor key, Tensor cos, Tensor sin) -> (Tensor, Tensor)",
    # csrc/packed_qkv_rope_cache/packed_qkv_rope_cache_torch.cpp:173-182
    "packed_qkv_rope_cache": ("packed_qkv_rope_cache(Tensor packed_qkv, Tensor cos, Tensor sin, "
                              "Tensor(a!) key_cache, Tensor(b!) value_cache, Tensor(c!) cache_length) -> Tensor"),
    "packed_qkv_rope_cache_out": ("packed_qkv_rope_cache_out(Tensor packed_qkv, Tensor cos, Tensor sin, "
                                  "Tensor(a!) key_cache, Tensor(b!) value_cache, Tensor(c!) cache_length, "
                                  "Tensor(d!) query_output) -> Tensor(d!)"),
    # csrc/gqa_decode_attention/gqa_decode_attention_torch.cpp:337-345
    "gqa_decode_attention": ("gqa_decode_attention(Tensor query, Tensor key_cache, Tensor value_cache, "
                             "Tensor? additive_attention_mask, float scale, Tensor? cache_length=None) -> Tensor"),
    "gqa_decode_attention_out": ("gqa_decode_attention_out(Tensor query, Tensor key_cache, Tensor value_cache, "
                                 "Tensor? additive_attention_mask, float scale, Tensor? cache_length, "
                                 "Tensor(a!) output, Tensor(b!) workspace) -> Tensor(a!)"),
    # csrc/packed_gate_up_gemv/packed_gate_up_gemv_torch.cpp:70-73
    "packed_gate_up_swiglu_out": "packed_gate_up_swiglu_out(Tensor input, Tensor weight, Tensor(a!) output) -> Tensor(a!)",
    # csrc/cublaslt_linear/cublaslt_linear_torch.cpp:516-523
    "cublaslt_algorithm_info": ("cublaslt_algorithm_info(Tensor input, Tensor weight, int max_workspace_bytes, "
                                "int max_algorithms=16) -> Tensor"),
    "cublaslt_linear_out": ("cublaslt_linear_out(Tensor input, Tensor weight, Tensor(a!) output, Tensor(b!) workspace, "
                            "int algorithm_index, int max_workspace_bytes) -> Tensor(a!)"),
    "cublaslt_linear_config_out": ("cublaslt_linear_config_out(Tensor input, Tensor weight, Tensor(a!) output, "
                                   "Tensor(b!) workspace, int algorithm_id, int tile_id, int split_k, "
                                   "int reduction_scheme, int cta_swizzle, int custom_option, int stages_id) "
                                   "-> Tensor(a!)"),
}

for _schema in _SCHEMAS.values():
    _LIB.define(_schema)


# ------------------------------------------------------------------ helpers


def _check(condition: bool, message: str) -> None:
    if not condition:
        raise RuntimeError(message)


def _no_grad(op: str, *tensors) -> None:
    _check(not torch.is_grad_enabled() or not any(t is not None and t.requires_grad for t in tensors),
           f"flux::{op} is inference-only; use torch.no_grad() or torch.inference_mode() for tensors that "
           "require gradients")


def _overlaps(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.device != b.device or a.numel() == 0 or b.numel() == 0:
        return False
    if a.untyped_storage().data_ptr() != b.untyped_storage().data_ptr():
        return False
    a0 = a.data_ptr()
    a1 = a0 + a.element_size() * (1 + sum((s - 1) * st for s, st in zip(a.shape, a.stride())))
    b0 = b.data_ptr()
    b1 = b0 + b.element_size() * (1 + sum((s - 1) * st for s, st in zip(b.shape, b.stride())))
    return a0 < b1 and b0 < a1


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: torch.Tensor) -> int:
    """The caller's current CUDA stream on the tensor's device (raw handle)."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index if t.device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def _cuda_only(op: str) -> None:
    raise RuntimeError(f"flux::{op}: CUDA tensors are required; flux_b200 has no CPU implementation")


def _lib():
    return _native.load()


def _impl(name: str, cuda_fn, cpu_validate) -> None:
    _LIB.impl(name, cuda_fn, "CUDA")

    def cpu(*args, **kwargs):
        cpu_validate(*args, **kwargs)
        _cuda_only(name)

    _LIB.impl(name, cpu, "CPU")


# ------------------------------------------------------------------ RMSNorm


def _validate_rmsnorm(input, weight, epsilon, *_):
    """``csrc/rmsnorm/rmsnorm_torch.cpp:18-52``."""
    _check(input.dim() >= 1, "flux::rmsnorm: input must have at least one dimension")
    _check(input.shape[-1] > 0, "flux::rmsnorm: input must have a non-empty final dimension")
    _check(input.numel() > 0, "flux::rmsnorm: input must contain at least one row")
    _check(input.dtype == torch.float32, "flux::rmsnorm: input must have dtype torch.float32")
    _check(weight.dtype == torch.float32, "flux::rmsnorm: weight must have dtype torch.float32")
    _check(weight.dim() == 1, "flux::rmsnorm: weight must be one-dimensional")
    _check(weight.shape[0] == input.shape[-1], "flux::rmsnorm: weight length must equal input.size(-1)")
    _check(weight.device == input.device, "flux::rmsnorm: input and weight must be on the same device")
    _check(0.0 < epsilon <= FLT_MAX, "flux::rmsnorm: epsilon must be a positive finite FP32 value")
    _no_grad("rmsnorm", input, weight)


def _rmsnorm_launch(input, weight, epsilon, output):
    rows = input.numel() // input.shape[-1]
    _native.check(_lib().fx_rmsnorm_f32(input.data_ptr(), weight.data_ptr(), output.data_ptr(), rows,
                                        input.shape[-1], float(epsilon), _stream(input)))
    return output


def _rmsnorm_cuda(input, weight, epsilon):
    _validate_rmsnorm(input, weight, epsilon)
    _check(input.is_cuda, "flux::rmsnorm: CUDA dispatch requires CUDA tensors")
    with torch.cuda.device(input.device):
        x, w = input.contiguous(), weight.contiguous()
        return _rmsnorm_launch(x, w, epsilon, torch.empty(input.shape, dtype=input.dtype, device=input.device))


def _validate_rmsnorm_out(input, weight, epsilon, output):
    _validate_rmsnorm(input, weight, epsilon)
    _check(input.is_contiguous() and weight.is_contiguous(), "flux::rmsnorm_out: input and weight must be contiguous")
    _check(output.shape == input.shape, "flux::rmsnorm_out: output shape must match input")
    _check(output.dtype == torch.float32 and output.device == input.device,
           "flux::rmsnorm_out: output must be float32 on the input device")
    _check(output.is_contiguous(), "flux::rmsnorm_out: output must be contiguous")
    _check(not _overlaps(output, input) and not _overlaps(output, weight),
           "flux::rmsnorm_out: output must not alias an input")


def _rmsnorm_out_cuda(input, weight, epsilon, output):
    _validate_rmsnorm_out(input, weight, epsilon, output)
    _check(input.is_cuda, "flux::rmsnorm_out: CUDA dispatch requires CUDA tensors")
    with torch.cuda.device(input.device):
        return _rmsnorm_launch(input, weight, epsilon, output)


_impl("rmsnorm", _rmsnorm_cuda, _validate_rmsnorm)
_impl("rmsnorm_out", _rmsnorm_out_cuda, _validate_rmsnorm_out)


# --------------------------------------------------------- residual RMSNorm


def _validate_residual_rmsnorm(hidden, residual, weight, epsilon, *_):
    """``csrc/residual_rmsnorm/residual_rmsnorm_torch.cpp:19-63``."""
    op = "residual_rmsnorm"
    _check(hidden.dim() >= 1, f"flux::{op}: hidden must have at least one dimension")
    _check(hidden.shape[-1] > 0, f"flux::{op}: hidden must have a non-empty final dimension")
    _check(hidden.numel() > 0, f"flux::{op}: hidden must contain at least one row")
    _check(hidden.shape == residual.shape, f"flux::{op}: hidden and residual must have the same shape")
    _check(hidden.dtype == torch.float32, f"flux::{op}: hidden must have dtype torch.float32")
    _check(residual.dtype == torch.float32, f"flux::{op}: residual must have dtype torch.float32")
    _check(weight.dtype == torch.float32, f"flux::{op}: weight must have dtype torch.float32")
    _check(weight.dim() == 1, f"flux::{op}: weight must be one-dimensional")
    _check(weight.shape[0] == hidden.shape[-1], f"flux::{op}: weight length must equal hidden.size(-1)")
    _check(residual.device == hidden.device and weight.device == hidden.device,
           f"flux::{op}: hidden, residual, and weight must be on the same device")
    _check(0.0 <= epsilon <= FLT_MAX, f"flux::{op}: epsilon must be a non-negative finite FP32 value")
    _no_grad(op, hidden, residual, weight)


def _residual_launch(hidden, residual, weight, epsilon, norm_out, residual_out):
    rows = hidden.numel() // hidden.shape[-1]
    _native.check(_lib().fx_residual_rmsnorm_f32(hidden.data_ptr(), residual.data_ptr(), weight.data_ptr(),
                                                 norm_out.data_ptr(), residual_out.data_ptr(), rows,
                                                 hidden.shape[-1], float(epsilon), _stream(hidden)))
    return norm_out, residual_out


def _residual_rmsnorm_cuda(hidden, residual, weight, epsilon):
    _validate_residual_rmsnorm(hidden, residual, weight, epsilon)
    _check(hidden.is_cuda, "flux::residual_rmsnorm: CUDA dispatch requires CUDA tensors")
    with torch.cuda.device(hidden.device):
        h, r, w = hidden.contiguous(), residual.contiguous(), weight.contiguous()
        residual_out = torch.empty(hidden.shape, dtype=torch.float32, device=hidden.device)
        norm_out = torch.empty(hidden.shape, dtype=torch.float32, device=hidden.device)
        return _residual_launch(h, r, w, epsilon, norm_out, residual_out)


def _validate_residual_rmsnorm_out(hidden, residual, weight, epsilon, norm_out, residual_out):
    op = "residual_rmsnorm_out"
    _validate_residual_rmsnorm(hidden, residual, weight, epsilon)
    _check(hidden.is_contiguous() and residual.is_contiguous() and weight.is_contiguous(),
           f"flux::{op}: inputs must be contiguous")
    for output in (norm_out, residual_out):
        _check(output.shape == hidden.shape, f"flux::{op}: output shapes must match hidden")
        _check(output.dtype == torch.float32 and output.device == hidden.device and output.is_contiguous(),
               f"flux::{op}: outputs must be contiguous float32 on the input device")
        _check(not any(_overlaps(output, t) for t in (hidden, residual, weight)),
               f"flux::{op}: outputs must not alias inputs")
    _check(not _overlaps(norm_out, residual_out), f"flux::{op}: outputs must not alias each other")


def _residual_rmsnorm_out_cuda(hidden, residual, weight, epsilon, norm_out, residual_out):
    _validate_residual_rmsnorm_out(hidden, residual, weight, epsilon, norm_out, residual_out)
    _check(hidden.is_cuda, "flux::residual_rmsnorm_out: CUDA dispatch requires CUDA tensors")
    with torch.cuda.device(hidden.device):
        return _residual_launch(hidden, residual, weight, epsilon, norm_out, residual_out)


_impl("residual_rmsnorm", _residual_rmsnorm_cuda, _validate_residual_rmsnorm)
_impl("residual_rmsnorm_out", _residual_rmsnorm_out_cuda, _validate_residual_rmsnorm_out)


# ----------------------------------------------------------- packed SwiGLU


def _validate_packed_swiglu(packed, *_):
    """``csrc/packed_swiglu/packed_swiglu_torch.cpp:18-41``."""
    op = "packed_swiglu"
    _check(packed.dim() >= 1, f"flux::{op}: packed must have at least one dimension")
    _check(packed.shape[-1] > 0, f"flux::{op}: packed final dimension must be non-empty")
    _check(packed.shape[-1] % 2 == 0, f"flux::{op}: packed final dimension must be even")
    _check(packed.numel() > 0, f"flux::{op}: packed must contain at least one row")
    _check(packed.dtype == torch.float32, f"flux::{op}: packed must have dtype torch.float32")
    _check(packed.is_contiguous(), f"flux::{op}: packed must be contiguous; no implicit copy is performed")
    _no_grad(op, packed)


def _swiglu_launch(packed, output):
    rows = packed.numel() // packed.shape[-1]
    _native.check(_lib().fx_packed_swiglu_f32(packed.data_ptr(), output.data_ptr(), rows, packed.shape[-1] // 2,
                                              _stream(packed)))
    return output


def _packed_swiglu_cuda(packed):
    _validate_packed_swiglu(packed)
    _check(packed.is_cuda, "flux::packed_swiglu: CUDA dispatch requires a CUDA tensor")
    with torch.cuda.device(packed.device):
        out = torch.empty((*packed.shape[:-1], packed.shape[-1] // 2), dtype=torch.float32, device=packed.device)
        return _swiglu_launch(packed, out)


def _validate_packed_swiglu_out(packed, output):
    _validate_packed_swiglu(packed)
    _check(output.shape == (*packed.shape[:-1], packed.shape[-1] // 2),
           "flux::packed_swiglu_out: output shape is incorrect")
    _check(output.dtype == torch.float32 and output.device == packed.device and output.is_contiguous(),
           "flux::packed_swiglu_out: output must be contiguous float32 on the input device")
    _check(not _overlaps(output, packed), "flux::packed_swiglu_out: output must not alias packed")


def _packed_swiglu_out_cuda(packed, output):
    _validate_packed_swiglu_out(packed, output)
    _check(packed.is_cuda, "flux::packed_swiglu_out: CUDA dispatch requires a CUDA tensor")
    with torch.cuda.device(packed.device):
        return _swiglu_launch(packed, output)


_impl("packed_swiglu", _packed_swiglu_cuda, _validate_packed_swiglu)
_impl("packed_swiglu_out", _packed_swiglu_out_cuda, _validate_packed_swiglu_out)


# ----------------------------------------------------------------- softmax


def _validate_softmax(input):
    """``csrc/softmax/softmax_torch.cpp:16-34``."""
    _check(input.dim() >= 1, "flux::softmax: input must have at least one dimension")
    _check(input.shape[-1] > 0, "flux::softmax: input must have a non-empty final dimension")
    _check(input.numel() > 0, "flux::softmax: input must contain at least one row")
    _check(input.dtype == torch.float32, "flux::softmax: input must have dtype torch.float32")
    _no_grad("softmax", input)


def _softmax_cuda(input):
    _validate_softmax(input)
    _check(input.is_cuda, "flux::softmax: CUDA dispatch requires a CUDA tensor")
    with torch.cuda.device(input.device):
        x = input.contiguous()
        out = torch.empty(input.shape, dtype=torch.float32, device=input.device)
        _native.check(_lib().fx_softmax_f32(x.data_ptr(), out.data_ptr(), x.numel() // x.shape[-1], x.shape[-1],
                                            _stream(x)))
        return out


_impl("softmax", _softmax_cuda, _validate_softmax)


def _validate_attention_score_softmax(scores, mask, scale):
    """``csrc/attention_score_softmax/attention_score_softmax_torch.cpp:19-50``."""
    op = "attention_score_softmax"
    _check(scores.dim() == 4, f"flux::{op}: scores must be rank four")
    _check(mask.dim() == 4, f"flux::{op}: additive_attention_mask must be rank four")
    _check(scores.numel() > 0 and scores.shape[-1] > 0, f"flux::{op}: scores dimensions must be non-empty")
    _check(scores.dtype == torch.float32, f"flux::{op}: scores must have dtype torch.float32")
    _check(mask.dtype == torch.float32, f"flux::{op}: additive_attention_mask must have dtype torch.float32")
    _check(scores.device == mask.device, f"flux::{op}: tensor devices must match")
    _check(all(m in (1, s) for m, s in zip(mask.shape, scores.shape)),
           f"flux::{op}: additive_attention_mask is not broadcastable to scores")
    _check(math.isfinite(scale) and abs(scale) <= FLT_MAX, f"flux::{op}: scale must be a finite FP32 value")
    _no_grad(op, scores, mask)


def _attention_score_softmax_cuda(scores, mask, scale):
    _validate_attention_score_softmax(scores, mask, scale)
    _check(scores.is_cuda, "flux::attention_score_softmax: CUDA dispatch requires CUDA tensors")
    with torch.cuda.device(scores.device):
        s = scores.contiguous()
        out = torch.empty(scores.shape, dtype=torch.float32, device=scores.device)
        _native.check(_lib().fx_attention_score_softmax_f32(
            s.data_ptr(), _native.int64_array(s.shape), mask.data_ptr(), _native.int64_array(mask.shape),
            _native.int64_array(mask.stride()), float(scale), out.data_ptr(), _stream(s)))
        return out


_impl("attention_score_softmax", _attention_score_softmax_cuda, _validate_attention_score_softmax)


# -------------------------------------------------------------------- RoPE


def _validate_rope(query, key, cos, sin):
    """``csrc/rope/rope_torch.cpp:19-55``."""
    _check(query.dim() == 4 and key.dim() == 4, "flux::rope: query and key must be rank four")
    _check(cos.dim() == 3 and sin.dim() == 3, "flux::rope: cos and sin must be rank three")
    _check(query.dtype == torch.float32 and key.dtype == torch.float32,
           "flux::rope: query and key must have dtype torch.float32")
    _check(cos.dtype == torch.float32 and sin.dtype == torch.float32,
           "flux::rope: cos and sin must have dtype torch.float32")
    _check(query.device == key.device == cos.device == sin.device, "flux::rope: all tensors must be on the same device")
    _check(all(d > 0 for d in (*query.shape, *key.shape)), "flux::rope: tensor dimensions must be non-empty")
    _check(query.shape[-1] % 2 == 0, "flux::rope: head_dim must be even")
    _check(key.shape[0] == query.shape[0] and key.shape[2:] == query.shape[2:],
           "flux::rope: query and key batch, sequence, and head dimensions must match")
    _check(cos.shape == sin.shape, "flux::rope: cos and sin shapes must match")
    _check(cos.shape[0] in (1, query.shape[0]) and cos.shape[1:] == query.shape[2:],
           "flux::rope: cos and sin shapes are not broadcastable to query and key")
    _no_grad("rope", query, key, cos, sin)


def _rope_cuda(query, key, cos, sin):
    _validate_rope(query, key, cos, sin)
    _check(query.is_cuda, "flux::rope: CUDA dispatch requires CUDA tensors")
    with torch.cuda.device(query.device):
        q_out = torch.empty(query.shape, dtype=torch.float32, device=query.device)
        k_out = torch.empty(key.shape, dtype=torch.float32, device=query.device)
        b, hq, s, d = query.shape
        _native.check(_lib().fx_rope_f32(
            query.data_ptr(), _native.int64_array(query.stride()), key.data_ptr(), _native.int64_array(key.stride()),
            cos.data_ptr(), _native.int64_array(cos.stride()), sin.data_ptr(), _native.int64_array(sin.stride()),
            q_out.data_ptr(), k_out.data_ptr(), b, hq, key.shape[1], s, d, cos.shape[0], _stream(query)))
        return q_out, k_out


_impl("rope", _rope_cuda, _validate_rope)


# ------------------------------------------------- packed QKV / RoPE / cache


def _validate_packed_qkv(packed_qkv, cos, sin, key_cache, value_cache, cache_length, *_):
    """``csrc/packed_qkv_rope_cache/packed_qkv_rope_cache_torch.cpp:22-74``."""
    op = "packed_qkv_rope_cache"
    _check(packed_qkv.shape == (1, 1, 960), f"flux::{op}: packed_qkv must have shape [1, 1, 960]")
    _check(cos.shape == (1, 1, 64) and sin.shape == cos.shape, f"flux::{op}: cos and sin must have shape [1, 1, 64]")
    _check(key_cache.dim() == 4 and value_cache.dim() == 4 and key_cache.shape == value_cache.shape
           and key_cache.shape[0] == 1 and key_cache.shape[1] == 3 and key_cache.shape[2] > 0
           and key_cache.shape[3] == 64,
           f"flux::{op}: K/V cache must have matching shape [1, 3, capacity, 64]")
    _check(cache_length.dim() == 0 and cache_length.numel() == 1 and cache_length.dtype == torch.int64,
           f"flux::{op}: cache_length must be a scalar torch.int64 tensor")
    for t in (packed_qkv, cos, sin, key_cache, value_cache):
        _check(t.dtype == torch.float32, f"flux::{op}: data tensors must have dtype torch.float32")
        _check(t.device == packed_qkv.device, f"flux::{op}: all tensors must be on the same device")
    _check(cache_length.device == packed_qkv.device, f"flux::{op}: all tensors must be on the same device")
    _check(all(s > 0 for s in packed_qkv.stride()), f"flux::{op}: packed_qkv strides must be positive")
    _check(all(s > 0 for s in (*key_cache.stride(), *value_cache.stride())), f"flux::{op}: cache strides must be positive")
    _check(not torch.is_grad_enabled() or not any(
        t.requires_grad for t in (packed_qkv, cos, sin, key_cache, value_cache, cache_length)),
        f"flux::{op} is inference-only; use torch.no_grad() or torch.inference_mode()")


def _packed_qkv_launch(packed_qkv, cos, sin, key_cache, value_cache, cache_length, query_output):
    _native.check(_lib().fx_packed_qkv_rope_cache_f32(
        packed_qkv.data_ptr(), _native.int64_array(packed_qkv.stride()), cos.data_ptr(),
        _native.int64_array(cos.stride()), sin.data_ptr(), _native.int64_array(sin.stride()),
        key_cache.data_ptr(), _native.int64_array(key_cache.stride()), value_cache.data_ptr(),
        _native.int64_array(value_cache.stride()), key_cache.shape[2], cache_length.data_ptr(),
        cache_length.data_ptr(), query_output.data_ptr(), _stream(packed_qkv)))
    return query_output


def _packed_qkv_cuda(packed_qkv, cos, sin, key_cache, value_cache, cache_length):
    _validate_packed_qkv(packed_qkv, cos, sin, key_cache, value_cache, cache_length)
    _check(packed_qkv.is_cuda, "flux::packed_qkv_rope_cache: CUDA dispatch requires CUDA tensors")
    with torch.cuda.device(packed_qkv.device):
        out = torch.empty((1, 9, 1, 64), dtype=torch.float32, device=packed_qkv.device)
        return _packed_qkv_launch(packed_qkv, cos, sin, key_cache, value_cache, cache_length, out)


def _validate_packed_qkv_out(packed_qkv, cos, sin, key_cache, value_cache, cache_length, query_output):
    op = "packed_qkv_rope_cache_out"
    _validate_packed_qkv(packed_qkv, cos, sin, key_cache, value_cache, cache_length)
    _check(query_output.shape == (1, 9, 1, 64), f"flux::{op}: query_output must have shape [1, 9, 1, 64]")
    _check(query_output.dtype == torch.float32 and query_output.device == packed_qkv.device
           and query_output.is_contiguous(),
           f"flux::{op}: query_output must be contiguous float32 on the input device")
    _check(not any(_overlaps(query_output, t) for t in (packed_qkv, cos, sin, key_cache, value_cache, cache_length)),
           f"flux::{op}: query_output must not alias an input")


def _packed_qkv_out_cuda(packed_qkv, cos, sin, key_cache, value_cache, cache_length, query_output):
    _validate_packed_qkv_out(packed_qkv, cos, sin, key_cache, value_cache, cache_length, query_output)
    _check(packed_qkv.is_cuda, "flux::packed_qkv_rope_cache_out: CUDA dispatch requires CUDA tensors")
    with torch.cuda.device(packed_qkv.device):
        return _packed_qkv_launch(packed_qkv, cos, sin, key_cache, value_cache, cache_length, query_output)


_impl("packed_qkv_rope_cache", _packed_qkv_cuda, _validate_packed_qkv)
_impl("packed_qkv_rope_cache_out", _packed_qkv_out_cuda, _validate_packed_qkv_out)


# ----------------------------------------------------- GQA decode attention

GQA_MAX_CAPACITY = 131072


def _validate_gqa(query, key_cache, value_cache, mask, scale, cache_length=None, *_):
    """``csrc/gqa_decode_attention/gqa_decode_attention_torch.cpp:22-104``."""
    op = "gqa_decode_attention"
    _check(query.dim() == 4 and key_cache.dim() == 4 and value_cache.dim() == 4,
           f"flux::{op}: Q/K/V tensors must be rank four")
    _check(query.shape[2] == 1, f"flux::{op}: query length must be one")
    _check(query.shape[0] == 1, f"flux::{op}: batch size must be one")
    _check(query.dtype == key_cache.dtype == value_cache.dtype == torch.float32,
           f"flux::{op}: Q/K/V tensors must have dtype torch.float32")
    _check(query.device == key_cache.device == value_cache.device, f"flux::{op}: Q/K/V tensor devices must match")
    _check(key_cache.shape == value_cache.shape, f"flux::{op}: key/value cache shapes must match")
    _check(query.shape[1] > 0 and query.shape[3] > 0 and key_cache.shape[1] > 0 and key_cache.shape[2] > 0,
           f"flux::{op}: tensor dimensions must be non-empty")
    _check(query.shape[0] == key_cache.shape[0], f"flux::{op}: cache batch must match query")
    _check(query.shape[3] == key_cache.shape[3], f"flux::{op}: cache head dimension must match query")
    _check(query.shape[1] % key_cache.shape[1] == 0, f"flux::{op}: query heads must be divisible by KV heads")
    _check(math.isfinite(scale) and abs(scale) <= FLT_MAX, f"flux::{op}: scale must be a finite FP32 value")
    if mask is not None:
        _check(mask.dim() == 4, f"flux::{op}: additive_attention_mask must be rank four")
        _check(mask.dtype == torch.float32, f"flux::{op}: additive_attention_mask must be float32")
        _check(mask.device == query.device, f"flux::{op}: mask device must match query")
        target = (query.shape[0], query.shape[1], 1, key_cache.shape[2])
        _check(all(m in (1, t) for m, t in zip(mask.shape, target)), f"flux::{op}: mask is not broadcastable")
    if cache_length is not None:
        _check(cache_length.numel() == 1 and cache_length.dtype == torch.int64,
               f"flux::{op}: cache_length must be a scalar int64 tensor")
        _check(cache_length.device == query.device, f"flux::{op}: cache_length device must match query")
        if cache_length.device.type == "cpu":
            length = int(cache_length.item())
            _check(1 <= length <= key_cache.shape[2], f"flux::{op}: cache_length must be within cache capacity")
    _no_grad(op, query, key_cache, value_cache, mask)


def _gqa_launch(query, key_cache, value_cache, mask, scale, cache_length, output, workspace):
    b, hq, _, d = query.shape
    _native.check(_lib().fx_gqa_decode_attention_f32(
        query.data_ptr(), _native.int64_array(query.stride()), key_cache.data_ptr(),
        _native.int64_array(key_cache.stride()), value_cache.data_ptr(), _native.int64_array(value_cache.stride()),
        _p(mask), _native.int64_array(mask.shape) if mask is not None else None,
        _native.int64_array(mask.stride()) if mask is not None else None, _p(cache_length), output.data_ptr(),
        workspace.data_ptr(), workspace.numel(), float(scale), b, hq, key_cache.shape[1], key_cache.shape[2], d,
        _stream(query)))
    return output


def _gqa_cuda(query, key_cache, value_cache, mask, scale, cache_length=None):
    _validate_gqa(query, key_cache, value_cache, mask, scale, cache_length)
    _check(query.is_cuda, "flux::gqa_decode_attention: CUDA dispatch requires CUDA tensors")
    _check(key_cache.shape[2] <= GQA_MAX_CAPACITY,
           f"flux::gqa_decode_attention: CUDA cache capacity exceeds {GQA_MAX_CAPACITY} tokens")
    with torch.cuda.device(query.device):
        out = torch.empty(query.shape, dtype=torch.float32, device=query.device)
        floats = _lib().fx_gqa_decode_attention_workspace_floats(query.shape[0], query.shape[1], key_cache.shape[2],
                                                                 query.shape[3])
        ws = torch.empty(floats, dtype=torch.float32, device=query.device)
        return _gqa_launch(query, key_cache, value_cache, mask, scale, cache_length, out, ws)


def _validate_gqa_out(query, key_cache, value_cache, mask, scale, cache_length, output, workspace):
    op = "gqa_decode_attention_out"
    _validate_gqa(query, key_cache, value_cache, mask, scale, cache_length)
    _check(query.shape[3] == 64 and key_cache.shape[2] > 512,
           f"flux::{op}: stable workspace path requires head_dim=64 and capacity > 512")
    _check(output.shape == query.shape, f"flux::{op}: output shape must match query")
    _check(output.dtype == torch.float32 and output.device == query.device and output.is_contiguous(),
           f"flux::{op}: output must be contiguous float32 on the query device")
    chunks = (key_cache.shape[2] + 127) // 128
    _check(tuple(workspace.shape) == (query.shape[0], query.shape[1], chunks, query.shape[3] + 2),
           f"flux::{op}: workspace shape is incorrect")
    _check(workspace.dtype == torch.float32 and workspace.device == query.device and workspace.is_contiguous(),
           f"flux::{op}: workspace must be contiguous float32 on the query device")
    _check(not _overlaps(output, workspace), f"flux::{op}: output and workspace must not alias")
    for t in (query, key_cache, value_cache):
        _check(not _overlaps(output, t) and not _overlaps(workspace, t), f"flux::{op}: outputs must not alias Q/K/V")
    if mask is not None:
        _check(not _overlaps(output, mask) and not _overlaps(workspace, mask),
               f"flux::{op}: outputs must not alias the mask")
    if cache_length is not None:
        _check(not _overlaps(output, cache_length) and not _overlaps(workspace, cache_length),
               f"flux::{op}: outputs must not alias cache_length")


def _gqa_out_cuda(query, key_cache, value_cache, mask, scale, cache_length, output, workspace):
    _validate_gqa_out(query, key_cache, value_cache, mask, scale, cache_length, output, workspace)
    _check(query.is_cuda, "flux::gqa_decode_attention_out: CUDA dispatch requires CUDA tensors")
    _check(key_cache.shape[2] <= GQA_MAX_CAPACITY,
           f"flux::gqa_decode_attention_out: CUDA cache capacity exceeds {GQA_MAX_CAPACITY} tokens")
    with torch.cuda.device(query.device):
        return _gqa_launch(query, key_cache, value_cache, mask, scale, cache_length, output, workspace)


_impl("gqa_decode_attention", _gqa_cuda, _validate_gqa)
_impl("gqa_decode_attention_out", _gqa_out_cuda, _validate_gqa_out)


# ------------------------------------------------------- gate/up + SwiGLU


def _validate_gate_up(input, weight, output):
    """``csrc/packed_gate_up_gemv/packed_gate_up_gemv_torch.cpp:17-47``."""
    op = "packed_gate_up_gemv"
    _check(input.is_cuda and weight.is_cuda and input.device == weight.device,
           f"flux::{op}: input and weight must be CUDA tensors on the same device")
    _check(input.shape == (1, 1, 576), f"flux::{op}: input must have shape [1, 1, 576]")
    _check(weight.shape == (3072, 576), f"flux::{op}: weight must have shape [3072, 576]")
    _check(input.dtype == torch.float32 and weight.dtype == torch.float32,
           f"flux::{op}: input and weight must have dtype torch.float32")
    _check(input.is_contiguous() and weight.is_contiguous(), f"flux::{op}: input and weight must be contiguous")
    _check(not torch.is_grad_enabled() or not (input.requires_grad or weight.requires_grad),
           f"flux::{op} is inference-only; use torch.no_grad() or torch.inference_mode()")
    _check(output.is_cuda and output.device == input.device,
           "flux::packed_gate_up_gemv_out: output must be CUDA on the input device")
    _check(output.shape == (1, 1, 1536), "flux::packed_gate_up_gemv_out: output shape is incorrect")
    _check(output.dtype == torch.float32 and output.is_contiguous(),
           "flux::packed_gate_up_gemv_out: output must be contiguous float32")
    _check(not _overlaps(output, input) and not _overlaps(output, weight),
           "flux::packed_gate_up_gemv_out: output must not alias an input")


def _gate_up_cuda(input, weight, output):
    _validate_gate_up(input, weight, output)
    with torch.cuda.device(input.device):
        _native.check(_lib().fx_packed_gate_up_swiglu_f32(input.data_ptr(), weight.data_ptr(), output.data_ptr(),
                                                          1536, 576, _stream(input)))
        return output


_impl("packed_gate_up_swiglu_out", _gate_up_cuda, _validate_gate_up)


# ------------------------------------------------ projection (cuBLASLt op)


def _validate_linear(input, weight, max_workspace_bytes):
    """``csrc/cublaslt_linear/cublaslt_linear_torch.cpp:255-281`` (M = 1 only)."""
    op = "cublaslt_linear"
    _check(input.is_cuda and weight.is_cuda, f"flux::{op}: input and weight must be CUDA tensors")
    _check(input.device == weight.device, f"flux::{op}: tensor devices must match")
    _check(input.dtype == torch.float32 and weight.dtype == torch.float32, f"flux::{op}: input and weight must be float32")
    _check(input.dim() >= 1 and weight.dim() == 2,
           f"flux::{op}: input must have at least one dimension and weight must be rank two")
    _check(input.shape[-1] > 0 and weight.shape[0] > 0 and input.shape[-1] == weight.shape[1],
           f"flux::{op}: weight shape must be [N, input.size(-1)]")
    _check(input.numel() == input.shape[-1], f"flux::{op}: only M=1 inputs are supported")
    _check(input.is_contiguous() and weight.is_contiguous(),
           f"flux::{op}: input and weight must be contiguous; no implicit copy is performed")
    _check(max_workspace_bytes >= 0, f"flux::{op}: max_workspace_bytes must be non-negative")
    _check(not torch.is_grad_enabled() or not (input.requires_grad or weight.requires_grad),
           f"flux::{op} is inference-only; use torch.no_grad() or torch.inference_mode()")


def _validate_linear_out(input, weight, output, workspace, max_workspace_bytes):
    op = "cublaslt_linear_out"
    _validate_linear(input, weight, max_workspace_bytes)
    _check(output.is_cuda and output.device == input.device and output.dtype == torch.float32
           and output.is_contiguous(),
           f"flux::{op}: output must be contiguous float32 CUDA on the input device")
    _check(output.dim() == input.dim() and output.numel() == weight.shape[0],
           f"flux::{op}: output must preserve the input rank with final width weight.size(0)")
    _check(workspace.is_cuda and workspace.device == input.device and workspace.dtype == torch.uint8
           and workspace.is_contiguous(),
           f"flux::{op}: workspace must be contiguous uint8 CUDA on the input device")
    _check(workspace.numel() <= max_workspace_bytes, f"flux::{op}: workspace exceeds max_workspace_bytes")
    _check(not any(_overlaps(output, t) for t in (input, weight, workspace)),
           f"flux::{op}: output must not alias an input or the workspace")


def _linear_launch(input, weight, output):
    _native.check(_lib().fx_linear_f32(input.data_ptr(), weight.data_ptr(), output.data_ptr(), 1, weight.shape[1],
                                       weight.shape[0], _stream(input)))
    return output


def _linear_out_cuda(input, weight, output, workspace, algorithm_index, max_workspace_bytes):
    _validate_linear_out(input, weight, output, workspace, max_workspace_bytes)
    _check(algorithm_index == 0, "flux::cublaslt_linear_out: algorithm_index must be 0 (one flux_b200 GEMV)")
    with torch.cuda.device(input.device):
        return _linear_launch(input, weight, output)


def _linear_config_out_cuda(input, weight, output, workspace, algorithm_id, tile_id, split_k, reduction_scheme,
                            cta_swizzle, custom_option, stages_id):
    # The cuBLASLt configuration fields select among library kernels; flux_b200
    # has one hand-written GEMV for this shape, so they are accepted and ignored.
    del algorithm_id, tile_id, split_k, reduction_scheme, cta_swizzle, custom_option, stages_id
    _validate_linear_out(input, weight, output, workspace, max(workspace.numel(), 0))
    with torch.cuda.device(input.device):
        return _linear_launch(input, weight, output)


def _algorithm_info_cuda(input, weight, max_workspace_bytes, max_algorithms=16):
    _validate_linear(input, weight, max_workspace_bytes)
    _check(1 <= max_algorithms <= 64, "flux::cublaslt_algorithm_info: max_algorithms must be in [1, 64]")
    # One entry: the flux_b200 GEMV (no workspace, one wave).
    return torch.tensor([[0, 0, 0, 1, 0, 0, 0, 0, 0, 1_000_000]], dtype=torch.int64)


_LIB.impl("cublaslt_algorithm_info", _algorithm_info_cuda, "CUDA")
_LIB.impl("cublaslt_linear_out", _linear_out_cuda, "CUDA")
_LIB.impl("cublaslt_linear_config_out", _linear_config_out_cuda, "CUDA")


# ------------------------------------------------------------------- fakes


@torch.library.register_fake("flux::rmsnorm")
def _rmsnorm_fake(input, weight, epsilon):
    _validate_rmsnorm(input, weight, epsilon)
    return torch.empty_like(input, memory_format=torch.contiguous_format)


@torch.library.register_fake("flux::rmsnorm_out")
def _rmsnorm_out_fake(input, weight, epsilon, output):
    return output


@torch.library.register_fake("flux::residual_rmsnorm")
def _residual_rmsnorm_fake(hidden, residual, weight, epsilon):
    _validate_residual_rmsnorm(hidden, residual, weight, epsilon)
    return (torch.empty_like(hidden, memory_format=torch.contiguous_format),
            torch.empty_like(hidden, memory_format=torch.contiguous_format))


@torch.library.register_fake("flux::residual_rmsnorm_out")
def _residual_rmsnorm_out_fake(hidden, residual, weight, epsilon, norm_out, residual_out):
    return norm_out, residual_out


@torch.library.register_fake("flux::packed_swiglu")
def _packed_swiglu_fake(packed):
    _validate_packed_swiglu(packed)
    return packed.new_empty((*packed.shape[:-1], packed.shape[-1] // 2))


@torch.library.register_fake("flux::packed_swiglu_out")
def _packed_swiglu_out_fake(packed, output):
    return output


@torch.library.register_fake("flux::softmax")
def _softmax_fake(input):
    _validate_softmax(input)
    return torch.empty_like(input, memory_format=torch.contiguous_format)


@torch.library.register_fake("flux::attention_score_softmax")
def _attention_score_softmax_fake(scores, mask, scale):
    _validate_attention_score_softmax(scores, mask, scale)
    return torch.empty_like(scores, memory_format=torch.contiguous_format)


@torch.library.register_fake("flux::rope")
def _rope_fake(query, key, cos, sin):
    _validate_rope(query, key, cos, sin)
    return (torch.empty_like(query, memory_format=torch.contiguous_format),
            torch.empty_like(key, memory_format=torch.contiguous_format))


@torch.library.register_fake("flux::packed_qkv_rope_cache")
def _packed_qkv_fake(packed_qkv, cos, sin, key_cache, value_cache, cache_length):
    return packed_qkv.new_empty((1, 9, 1, 64))


@torch.library.register_fake("flux::packed_qkv_rope_cache_out")
def _packed_qkv_out_fake(packed_qkv, cos, sin, key_cache, value_cache, cache_length, query_output):
    return query_output


@torch.library.register_fake("flux::gqa_decode_attention")
def _gqa_fake(query, key_cache, value_cache, mask, scale, cache_length=None):
    _validate_gqa(query, key_cache, value_cache, mask, scale, None)
    return torch.empty_like(query, memory_format=torch.contiguous_format)


@torch.library.register_fake("flux::gqa_decode_attention_out")
def _gqa_out_fake(query, key_cache, value_cache, mask, scale, cache_length, output, workspace):
    return output


@torch.library.register_fake("flux::packed_gate_up_swiglu_out")
def _gate_up_fake(input, weight, output):
    return output


@torch.library.register_fake("flux::cublaslt_linear_out")
def _linear_out_fake(input, weight, output, workspace, algorithm_index, max_workspace_bytes):
    return output


@torch.library.register_fake("flux::cublaslt_linear_config_out")
def _linear_config_out_fake(input, weight, output, workspace, algorithm_id, tile_id, split_k, reduction_scheme,
                            cta_swizzle, custom_option, stages_id):
    return output


# --------------------------------------- Python entry points (flux/ops/native_*.py)


def _require_native(what: str) -> None:
    if not _native.is_available():
        raise RuntimeError(f"Flux native {what} is not built: {_native.load_error()}")


def native_rmsnorm_load_error():
    return _native.load_error()


def _available() -> bool:
    return _native.is_available()


native_rmsnorm_is_available = _available
native_residual_rmsnorm_is_available = _available
native_packed_swiglu_is_available = _available
native_softmax_is_available = _available
native_attention_score_softmax_is_available = _available
native_rope_is_available = _available
native_packed_qkv_rope_cache_is_available = _available
native_gqa_decode_attention_is_available = _available
native_packed_gate_up_gemv_is_available = _available
native_cublaslt_linear_is_available = _available
native_softmax_load_error = native_rmsnorm_load_error
native_rope_load_error = native_rmsnorm_load_error
native_packed_qkv_rope_cache_load_error = native_rmsnorm_load_error


def rms_norm_native(input, weight, epsilon):
    _require_native("RMSNorm")
    return torch.ops.flux.rmsnorm(input, weight, epsilon)


def rms_norm_native_out(input, weight, epsilon, output):
    _require_native("RMSNorm")
    return torch.ops.flux.rmsnorm_out(input, weight, epsilon, output)


def residual_rmsnorm_native(hidden, residual, weight, epsilon):
    _require_native("residual RMSNorm")
    return torch.ops.flux.residual_rmsnorm(hidden, residual, weight, epsilon)


def residual_rmsnorm_native_out(hidden, residual, weight, epsilon, norm_out, residual_out):
    _require_native("residual RMSNorm")
    return torch.ops.flux.residual_rmsnorm_out(hidden, residual, weight, epsilon, norm_out, residual_out)


def packed_swiglu_native(packed):
    _require_native("packed SwiGLU")
    return torch.ops.flux.packed_swiglu(packed)


def packed_swiglu_native_out(packed, output):
    _require_native("packed SwiGLU")
    return torch.ops.flux.packed_swiglu_out(packed, output)


def softmax_native(input):
    _require_native("softmax")
    return torch.ops.flux.softmax(input)


def attention_score_softmax_native(scores, additive_attention_mask, scale):
    _require_native("attention score softmax")
    return torch.ops.flux.attention_score_softmax(scores, additive_attention_mask, scale)


def rope_native(query, key, cos, sin):
    _require_native("RoPE")
    return torch.ops.flux.rope(query, key, cos, sin)


def packed_qkv_rope_cache_native(packed_qkv, cos, sin, key_cache, value_cache, cache_length):
    _require_native("packed QKV/RoPE/cache")
    return torch.ops.flux.packed_qkv_rope_cache(packed_qkv, cos, sin, key_cache, value_cache, cache_length)


def packed_qkv_rope_cache_native_out(packed_qkv, cos, sin, key_cache, value_cache, cache_length, query_output):
    _require_native("packed QKV/RoPE/cache")
    return torch.ops.flux.packed_qkv_rope_cache_out(packed_qkv, cos, sin, key_cache, value_cache, cache_length,
                                                    query_output)


def gqa_decode_attention_native(query, key_cache, value_cache, additive_attention_mask, scale, cache_length=None):
    _require_native("GQA decode attention")
    return torch.ops.flux.gqa_decode_attention(query, key_cache, value_cache, additive_attention_mask, scale,
                                               cache_length)


def gqa_decode_attention_native_out(query, key_cache, value_cache, additive_attention_mask, scale, cache_length,
                                    output, workspace):
    _require_native("GQA decode attention")
    return torch.ops.flux.gqa_decode_attention_out(query, key_cache, value_cache, additive_attention_mask, scale,
                                                   cache_length, output, workspace)


def packed_gate_up_swiglu_native_out(input, weight, output):
    _require_native("gate/up GEMV")
    return torch.ops.flux.packed_gate_up_swiglu_out(input, weight, output)


@dataclass(frozen=True)
class CublasLtAlgorithm:
    """Projection configuration record (``flux/ops/native_cublaslt_linear.py:16-28``).

    flux_b200 runs its own GEMV for every configuration; the fields are kept so
    code written against the reference keeps working."""

    index: int
    algorithm_id: int
    tile_id: int
    split_k: int
    reduction_scheme: int
    cta_swizzle: int
    custom_option: int
    stages_id: int
    workspace_bytes: int
    waves_count: float


def cublaslt_algorithms(input, weight, *, max_workspace_bytes: int, max_algorithms: int = 16):
    _require_native("projection")
    rows = torch.ops.flux.cublaslt_algorithm_info(input, weight, max_workspace_bytes, max_algorithms).tolist()
    return tuple(CublasLtAlgorithm(index=r[0], algorithm_id=r[1], tile_id=r[2], split_k=r[3], reduction_scheme=r[4],
                                   cta_swizzle=r[5], custom_option=r[6], stages_id=r[7], workspace_bytes=r[8],
                                   waves_count=r[9] / 1_000_000.0) for r in rows)


def cublaslt_linear_out(input, weight, output, workspace, *, algorithm_index: int, max_workspace_bytes: int):
    _require_native("projection")
    return torch.ops.flux.cublaslt_linear_out(input, weight, output, workspace, algorithm_index, max_workspace_bytes)


def cublaslt_linear_config_out(input, weight, output, workspace, algorithm: CublasLtAlgorithm):
    _require_native("projection")
    return torch.ops.flux.cublaslt_linear_config_out(
        input, weight, output, workspace, algorithm.algorithm_id, algorithm.tile_id, algorithm.split_k,
        algorithm.reduction_scheme, algorithm.cta_swizzle, algorithm.custom_option, algorithm.stages_id)


__all__ = [name for name in dir() if name.endswith(("_native", "_native_out", "_is_available", "_load_error"))] + [
    "CublasLtAlgorithm", "cublaslt_algorithms", "cublaslt_linear_config_out", "cublaslt_linear_out",
]
