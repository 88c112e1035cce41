"""Native SmolLM2 decode / prefill runtimes (drop-in for ``flux/runtime``).

Python owners mirroring ``flux/runtime/native_smollm2.py`` over the C ABI
(``fx_decode_*`` / ``fx_prefill_*``).  The native objects own the compact
30-layer cache, the stable token/logit/state buffers, the workspace and the
captured CUDA graph; they are exposed here as zero-copy torch tensors whose
addresses never change.  Weights stay borrowed from the model (as the
reference's ``at::Tensor`` members do).

Differences from the reference, all deliberate: the cache capacity limit is
131072 rows instead of 8192 (the decode kernels chunk the valid length), and
the objects are plain Python classes over ctypes rather than
``torch.classes.flux`` TorchScript classes.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Any, Sequence

import torch
from torch import nn
from transformers import DynamicCache

from flux_b200 import _native

MAX_CAPACITY = 131072
HIDDEN, INTER, LAYERS = 576, 1536, 30

_ADDRESS_NAMES = (
    "input_token", "logits", "generated_tokens", "device_generation_step", "key_cache", "value_cache",
    "device_position", "device_cache_length", "workspace", "hidden_a", "hidden_b", "final_norm_output",
    "attention_workspace",
)
_PREFILL_ADDRESS_NAMES = ("prefill_logits", "prefill_workspace", "streaming_attention_output",
                          "final_hidden") + _ADDRESS_NAMES


@dataclass(frozen=True)
class NativeDecodeRuntimeMemory:
    """Persistent memory attributable to the native decode runtime."""

    cache_bytes: int
    workspace_bytes: int
    stable_buffer_bytes: int
    referenced_weight_bytes: int
    graph_resource_bytes: int | None = None

    @property
    def owned_tensor_bytes(self) -> int:
        return self.cache_bytes + self.workspace_bytes + self.stable_buffer_bytes


@dataclass(frozen=True)
class NativePrefillRuntimeMemory:
    """Persistent native prefill memory plus the decode storage it feeds."""

    cache_bytes: int
    prefill_workspace_bytes: int
    decode_workspace_bytes: int
    stable_buffer_bytes: int
    referenced_weight_bytes: int

    @property
    def owned_tensor_bytes(self) -> int:
        return self.cache_bytes + self.prefill_workspace_bytes + self.decode_workspace_bytes + self.stable_buffer_bytes


def native_smollm2_runtime_is_available() -> bool:
    available = _native.is_available()
    if available:
        _native.load_torch_classes()  # torch.classes.flux.* for callers that build the objects directly
    return available


def native_smollm2_prefill_is_available() -> bool:
    available = _native.is_available()
    if available:
        _native.load_torch_classes()
    return available


# ------------------------------------------------------- device buffer views


class _DeviceView:
    """``__cuda_array_interface__`` record that keeps the owning runtime alive."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str, owner: Any):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 2, "strides": None}
        self._owner = owner


def _view(ptr: int, shape, dtype: torch.dtype, owner, device: torch.device) -> torch.Tensor:
    typestr = {torch.float32: "<f4", torch.int64: "<i8", torch.uint8: "|u1"}[dtype]
    return torch.as_tensor(_DeviceView(ptr, shape, typestr, owner), device=device)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """The caller's current CUDA stream on `device` as a raw handle (queried
    on every call, so it follows `torch.cuda.stream(...)` contexts)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _check_tensor(tensor: torch.Tensor, device, dtype, shape, name: str, prefix: str) -> None:
    """``check_tensor`` of ``native_decode_runtime_cuda.cu:53-68``."""
    if tensor is None:
        raise RuntimeError(f"{prefix}: {name} is undefined")
    if tensor.device != device:
        raise RuntimeError(f"{prefix}: {name} must be on {device}")
    if tensor.dtype != dtype:
        raise RuntimeError(f"{prefix}: {name} has the wrong dtype")
    if tuple(tensor.shape) != tuple(shape):
        raise RuntimeError(f"{prefix}: {name} has shape {list(tensor.shape)}, expected {list(shape)}")
    if not tensor.is_contiguous():
        raise RuntimeError(f"{prefix}: {name} must be contiguous")


def _model_weights(model: nn.Module) -> dict[str, Any]:
    layers = list(model.model.layers)
    return {
        "embedding": model.model.embed_tokens.weight,
        "final_norm": model.model.norm.weight,
        "lm_head": model.lm_head.weight,
        "input_norm": [layer.input_layernorm.weight for layer in layers],
        "packed_qkv": [layer.self_attn.packed_qkv.weight for layer in layers],
        "o_proj": [layer.self_attn.o_proj.weight for layer in layers],
        "post_norm": [layer.post_attention_layernorm.weight for layer in layers],
        "gate_up": [layer.mlp.gate_up_proj.weight for layer in layers],
        "down": [layer.mlp.down_proj.weight for layer in layers],
        "epsilons": [float(layer.input_layernorm.variance_epsilon) for layer in layers],
        "scales": [float(layer.self_attn.scaling) for layer in layers],
    }


def _model_desc(weights: dict[str, Any], cos: torch.Tensor, sin: torch.Tensor, capacity: int,
                prefix: str) -> _native.ModelDesc:
    """Validate shapes the way the reference constructors do and fill ``fx_model_desc``."""
    embedding = weights["embedding"]
    device = embedding.device
    vocab = int(embedding.shape[0]) if embedding.dim() == 2 else 0
    if vocab <= 0:
        raise RuntimeError(f"{prefix}: vocabulary must be non-empty")
    for key in ("input_norm", "packed_qkv", "o_proj", "post_norm", "gate_up", "down", "epsilons", "scales"):
        if len(weights[key]) != LAYERS:
            raise RuntimeError(f"{prefix}: exactly 30 complete layer descriptors are required")
    f32 = torch.float32
    _check_tensor(embedding, device, f32, (vocab, HIDDEN), "embedding weight", prefix)
    _check_tensor(weights["lm_head"], device, f32, (vocab, HIDDEN), "LM-head weight", prefix)
    _check_tensor(weights["final_norm"], device, f32, (HIDDEN,), "final norm weight", prefix)
    _check_tensor(cos, device, f32, (capacity, 64), "RoPE cosine table", prefix)
    _check_tensor(sin, device, f32, (capacity, 64), "RoPE sine table", prefix)
    checks = (("input_norm", (HIDDEN,), "layer input norm weight"), ("packed_qkv", (960, HIDDEN), "layer packed QKV weight"),
              ("o_proj", (HIDDEN, HIDDEN), "layer attention output weight"),
              ("post_norm", (HIDDEN,), "layer post-attention norm weight"),
              ("gate_up", (2 * INTER, HIDDEN), "layer gate/up weight"), ("down", (HIDDEN, INTER), "layer down weight"))
    for key, shape, name in checks:
        for tensor in weights[key]:
            _check_tensor(tensor, device, f32, shape, name, prefix)
    epsilons = weights["epsilons"]
    for eps in epsilons:
        if not (eps > 0.0 and eps == eps and eps != float("inf")):
            raise RuntimeError(f"{prefix}: every RMSNorm epsilon must be positive")
    if len(set(epsilons)) != 1:
        raise RuntimeError(f"{prefix}: every layer must share one RMSNorm epsilon")
    for scale in weights["scales"]:
        if not (scale == scale and abs(scale) != float("inf")):
            raise RuntimeError(f"{prefix}: every attention scale must be finite")
    desc = _native.ModelDesc()
    desc.device = device.index if device.index is not None else torch.cuda.current_device()
    desc.vocab = vocab
    desc.capacity = capacity
    desc.epsilon = epsilons[0]
    desc.embedding = embedding.data_ptr()
    desc.final_norm = weights["final_norm"].data_ptr()
    desc.lm_head = weights["lm_head"].data_ptr()
    desc.rope_cos = cos.data_ptr()
    desc.rope_sin = sin.data_ptr()
    for layer in range(LAYERS):
        desc.input_norm[layer] = weights["input_norm"][layer].data_ptr()
        desc.packed_qkv[layer] = weights["packed_qkv"][layer].data_ptr()
        desc.o_proj[layer] = weights["o_proj"][layer].data_ptr()
        desc.post_norm[layer] = weights["post_norm"][layer].data_ptr()
        desc.gate_up[layer] = weights["gate_up"][layer].data_ptr()
        desc.down[layer] = weights["down"][layer].data_ptr()
        desc.attention_scale[layer] = weights["scales"][layer]
    return desc


def _rope_tables(model: nn.Module, positions: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin from the model's own ``rotary_emb`` (``native_smollm2.py:131-138``)."""
    ids = torch.arange(positions, dtype=torch.long, device=device).unsqueeze(0)
    seed = model.model.embed_tokens.weight[:1].view(1, 1, HIDDEN)
    with torch.inference_mode():
        cos, sin = model.model.rotary_emb(seed, ids)
    return cos.reshape(positions, 64).contiguous(), sin.reshape(positions, 64).contiguous()


# ------------------------------------------------------------ native objects


class _OwnedHandle:
    """Owns one native handle and destroys it when the last view goes away.

    Tensor views of runtime memory reference this object (never the Python
    runtime wrapper), so there is no reference cycle and a tensor that
    outlives its runtime keeps the memory valid.  ``keepalive`` holds the
    borrowed weight tensors for as long as the native object may read them."""

    def __init__(self, ptr: int, destroy: str, keepalive: tuple = ()):
        self.ptr = ptr
        # Bound now: at interpreter shutdown module globals may already be gone.
        self._destroy = getattr(_native.load(), destroy)
        self._keepalive = keepalive

    def __del__(self):
        ptr, self.ptr = self.ptr, None
        if ptr:
            self._destroy(ptr)


class NativeDecodeObject:
    """The native ``fx_decode`` handle with the ``torch.classes.flux.
    NativeSmolLM2Decode`` method surface (``native_decode_runtime_torch.cpp:38-79``)."""

    _PREFIX = "flux native full decode"

    def __init__(self, handle: int, device: torch.device, owner: _OwnedHandle):
        self._handle = handle
        self._device = device
        self._owner = owner
        lib = _native.load()
        buffers = _native.DecodeBuffers()
        _native.check(lib.fx_decode_get_buffers(handle, ctypes.byref(buffers)))
        info = self._info()
        cap, vocab = info.capacity, info.vocab
        self._buffers = buffers
        self._capacity = int(cap)
        self._vocab = int(vocab)
        self._kernels_per_step = int(info.kernels_per_step)
        f32, i64, o = torch.float32, torch.int64, owner
        self._input_token = _view(buffers.input_token, (1, 1), i64, o, device)
        self._logits = _view(buffers.logits, (1, 1, vocab), f32, o, device)
        self._generated = _view(buffers.generated_tokens, (cap,), i64, o, device)
        self._step = _view(buffers.generation_step, (), i64, o, device)
        self._key_cache = _view(buffers.key_cache, (LAYERS, 1, 3, cap, 64), f32, o, device)
        self._value_cache = _view(buffers.value_cache, (LAYERS, 1, 3, cap, 64), f32, o, device)
        self._position = _view(buffers.position, (), i64, o, device)
        self._length = _view(buffers.cache_length, (), i64, o, device)
        self._workspace = _view(buffers.workspace, (buffers.workspace_bytes,), torch.uint8, o, device)
        self._host_in, self._host_out = ctypes.c_int64(0), ctypes.c_int64(0)
        self._host_in_addr, self._host_out_addr = ctypes.addressof(self._host_in), ctypes.addressof(self._host_out)

    def _info(self) -> _native.DecodeInfo:
        info = _native.DecodeInfo()
        _native.check(_native.load().fx_decode_get_info(self._handle, ctypes.byref(info)))
        return info

    # methods of the reference custom class
    def replay(self, token: torch.Tensor | None = None) -> torch.Tensor:
        if token is not None:
            _check_tensor(token, self._device, torch.int64, (1, 1), "replay token", self._PREFIX)
        _native.check(_native.load().fx_decode_replay(self._handle, None if token is None else token.data_ptr(),
                                                      _stream(self._device)))
        return self._logits

    def replay_host(self, token: int | None = None) -> int:
        """One step with host buffers (``fx_decode_replay_host``): the host
        token in (None keeps the device's current token), the sampled token
        back as a Python int once it is on the host."""
        if token is not None:
            self._host_in.value = token
        _native.check(_native.load().fx_decode_replay_host(
            self._handle, None if token is None else self._host_in_addr, self._host_out_addr, _stream(self._device)))
        return self._host_out.value

    def generate_greedy(self, decode_steps: int, eos_token_id: int | None = None) -> torch.Tensor:
        """`decode_steps` chained greedy steps on device; with `eos_token_id`
        the steps after the one that samples it leave the state unchanged."""
        lib = _native.load()
        _native.check(lib.fx_decode_set_eos(self._handle, -1 if eos_token_id is None else int(eos_token_id)))
        _native.check(lib.fx_decode_generate(self._handle, int(decode_steps), _stream(self._device)))
        return self._generated

    def reset(self, token: torch.Tensor, key_caches: Sequence[torch.Tensor], value_caches: Sequence[torch.Tensor],
              position: int) -> None:
        _check_tensor(token, self._device, torch.int64, (1, 1), "token", self._PREFIX)
        if not 0 <= position < self._capacity:
            raise RuntimeError(f"{self._PREFIX}: reset position must be inside capacity")
        rows = _validate_sources(key_caches, value_caches, position, self._device, self._PREFIX)
        _native.check(_native.load().fx_decode_reset(
            self._handle, token.data_ptr(), _native.pointer_array(t.data_ptr() for t in key_caches),
            _native.pointer_array(t.data_ptr() for t in value_caches), rows, int(position), _stream(self._device)))

    def _read(self, which: int) -> int:
        value = ctypes.c_int64(0)
        _native.check(_native.load().fx_decode_read_state(self._handle, which, ctypes.byref(value)))
        return int(value.value)

    def logits(self) -> torch.Tensor: return self._logits
    def current_token(self) -> torch.Tensor: return self._input_token
    def generated_tokens(self) -> torch.Tensor: return self._generated
    def device_generation_step(self) -> torch.Tensor: return self._step
    def key_cache(self) -> torch.Tensor: return self._key_cache
    def value_cache(self) -> torch.Tensor: return self._value_cache
    def device_position(self) -> torch.Tensor: return self._position
    def device_cache_length(self) -> torch.Tensor: return self._length
    def workspace(self) -> torch.Tensor: return self._workspace
    def position(self) -> int: return self._read(_native.STATE_POSITION)
    def cache_length(self) -> int: return self._read(_native.STATE_CACHE_LENGTH)
    def generation_step(self) -> int: return self._read(_native.STATE_GENERATION_STEP)
    def capacity(self) -> int: return self._capacity
    def replay_count(self) -> int: return int(self._info().replay_count)
    def workspace_bytes(self) -> int: return int(self._buffers.workspace_bytes)
    def stable_buffer_bytes(self) -> int: return int(self._buffers.stable_buffer_bytes)
    def vocabulary_size(self) -> int: return self._vocab
    def layer_count(self) -> int: return LAYERS
    def kernels_per_step(self) -> int: return self._kernels_per_step

    def addresses(self) -> list[int]:
        b = self._buffers
        return [b.input_token, b.logits, b.generated_tokens, b.generation_step, b.key_cache, b.value_cache,
                b.position, b.cache_length, b.workspace, b.hidden_a, b.hidden_b, b.final_norm_output,
                b.attention_workspace]


def _validate_sources(keys, values, position: int, device, prefix: str) -> int:
    if len(keys) != LAYERS or len(values) != LAYERS:
        raise RuntimeError(f"{prefix}: reset requires one K/V tensor per layer")
    rows = None
    for k, v in zip(keys, values):
        ok = (k is not None and v is not None and k.device == device and v.device == device
              and k.dtype == torch.float32 and v.dtype == torch.float32 and k.is_contiguous() and v.is_contiguous()
              and k.dim() == 4 and v.shape == k.shape and k.shape[0] == 1 and k.shape[1] == 3
              and k.shape[2] >= position and k.shape[3] == 64)
        if not ok:
            raise RuntimeError(f"{prefix}: every K/V source must be contiguous float32 [1, 3, sequence>=position, 64]")
        if rows is not None and k.shape[2] != rows:
            raise RuntimeError(f"{prefix}: every K/V source must have the same sequence length")
        rows = int(k.shape[2])
    return rows or 0


class NativePrefillObject:
    """The native ``fx_prefill`` handle with the ``torch.classes.flux.
    NativeSmolLM2Prefill`` method surface (``native_prefill_runtime_torch.cpp:5-45``)."""

    _PREFIX = "flux native prefill"

    def __init__(self, handle: int, device: torch.device, owner: _OwnedHandle):
        self._handle = handle
        self._device = device
        self._owner = owner
        lib = _native.load()
        buffers = _native.PrefillBuffers()
        _native.check(lib.fx_prefill_get_buffers(handle, ctypes.byref(buffers)))
        self._buffers = buffers
        self._rows = int(lib.fx_prefill_prompt_length(handle))
        # The prefill owns its decode runtime: decode views keep the prefill handle alive.
        self._decode = NativeDecodeObject(lib.fx_prefill_decode(handle), device, owner)
        vocab = self._decode.vocabulary_size()
        self._logits = _view(buffers.prefill_logits, (1, 1, vocab), torch.float32, owner, device)
        self._final_hidden = _view(buffers.final_hidden, (1, 1, HIDDEN), torch.float32, owner, device)

    def prefill(self, input_ids: torch.Tensor) -> torch.Tensor:
        _check_tensor(input_ids, self._device, torch.int64, (1, self._rows), "input_ids", self._PREFIX)
        _native.check(_native.load().fx_prefill_run(self._handle, input_ids.data_ptr(), _stream(self._device)))
        return self._logits

    def replay(self, token: torch.Tensor | None = None) -> torch.Tensor:
        return self._decode.replay(token)

    def replay_host(self, token: int | None = None) -> int:
        return self._decode.replay_host(token)

    def generate_greedy(self, max_new_tokens: int, eos_token_id: int | None = None) -> torch.Tensor:
        if max_new_tokens < 1:
            raise RuntimeError(f"{self._PREFIX}: max_new_tokens must be positive")
        if max_new_tokens > self._decode.capacity() - self._rows + 1:
            raise RuntimeError(f"{self._PREFIX}: generation exceeds fixed cache capacity")
        if eos_token_id is None:
            storage = self._decode.generate_greedy(max_new_tokens - 1)
            return storage.narrow(0, 0, max_new_tokens).view(1, max_new_tokens)
        if not 0 <= int(eos_token_id) < self._decode.vocabulary_size():
            raise RuntimeError(f"{self._PREFIX}: eos_token_id must be a vocabulary id")
        # The prefill's own token may already be EOS; otherwise the device
        # loop stops itself and the step counter gives the length.
        if int(self._decode.generated_tokens()[0].item()) == int(eos_token_id):
            steps = 0
            self._decode.generate_greedy(0, eos_token_id)
        else:
            self._decode.generate_greedy(max_new_tokens - 1, eos_token_id)
            steps = self._decode.generation_step() - 1
        n = steps + 1
        return self._decode.generated_tokens().narrow(0, 0, n).view(1, n)

    def logits(self) -> torch.Tensor: return self._logits
    def final_hidden(self) -> torch.Tensor: return self._final_hidden
    def current_token(self) -> torch.Tensor: return self._decode.current_token()
    def generated_tokens(self) -> torch.Tensor: return self._decode.generated_tokens()
    def device_generation_step(self) -> torch.Tensor: return self._decode.device_generation_step()
    def key_cache(self) -> torch.Tensor: return self._decode.key_cache()
    def value_cache(self) -> torch.Tensor: return self._decode.value_cache()
    def device_position(self) -> torch.Tensor: return self._decode.device_position()
    def device_cache_length(self) -> torch.Tensor: return self._decode.device_cache_length()
    def position(self) -> int: return self._decode.position()
    def cache_length(self) -> int: return self._decode.cache_length()
    def prompt_length(self) -> int: return self._rows
    def capacity(self) -> int: return self._decode.capacity()
    def replay_count(self) -> int: return self._decode.replay_count()
    def generation_step(self) -> int: return self._decode.generation_step()
    def workspace_bytes(self) -> int: return int(self._buffers.workspace_bytes)
    def stable_buffer_bytes(self) -> int:
        return 8 + self._decode.vocabulary_size() * 4 + self._decode.stable_buffer_bytes()

    def cache_bytes(self) -> int:
        return 2 * self._decode.key_cache().numel() * 4

    def addresses(self) -> list[int]:
        b = self._buffers
        return [b.prefill_logits, b.workspace, b.attention_output, b.final_hidden] + self._decode.addresses()


# --------------------------------------------------------- Python owners


class NativeSmolLM2Prefill:
    """Native FP32 prompt prefill with direct native-decode continuation
    (``flux/runtime/native_smollm2.py:94-261``)."""

    def __init__(self) -> None:
        raise TypeError("use NativeSmolLM2Prefill.capture(...) to create a runtime")

    @classmethod
    def capture(cls, model: nn.Module, input_ids: torch.Tensor, *, max_decode_steps: int = 0) -> "NativeSmolLM2Prefill":
        if max_decode_steps < 0:
            raise ValueError("max_decode_steps must be non-negative")
        requested = input_ids.shape[1] + max_decode_steps if input_ids.ndim == 2 else 0
        NativeSmolLM2Decode._validate_capture_model_input(model, input_ids, requested)
        if int(input_ids.min().item()) < 0 or int(input_ids.max().item()) >= int(model.config.vocab_size):
            raise ValueError("input_ids contain a token outside the vocabulary")
        if not native_smollm2_prefill_is_available():
            raise RuntimeError(f"flux_b200 native prefill runtime is not available: {_native.load_error()}")
        device = input_ids.device
        cos, sin = _rope_tables(model, requested, device)
        weights = _model_weights(model)
        desc = _model_desc(weights, cos, sin, requested, "flux native prefill")
        handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            _native.check(_native.load().fx_prefill_create(ctypes.byref(desc), input_ids.data_ptr(),
                                                           input_ids.shape[1], _stream(device), ctypes.byref(handle)))
        self = object.__new__(cls)
        self.model = model
        self.input_ids = input_ids
        self._rope_cos, self._rope_sin = cos, sin
        owner = _OwnedHandle(handle.value, "fx_prefill_destroy", (weights, cos, sin))
        self._native = NativePrefillObject(handle.value, device, owner)
        self.prefill_logits = self._native.logits()
        return self

    def prefill(self, input_ids: torch.Tensor | None = None) -> torch.Tensor:
        ids = self.input_ids if input_ids is None else input_ids
        if ids.shape != self.input_ids.shape:
            raise ValueError("reused native prefill requires the captured prompt shape")
        if ids.dtype != torch.long or ids.device != self.input_ids.device:
            raise ValueError("reused input_ids must preserve CUDA device and long dtype")
        if not ids.is_contiguous():
            raise ValueError("reused input_ids must be contiguous")
        self.input_ids = ids
        return self._native.prefill(ids)

    def replay(self, token: torch.Tensor | None = None) -> torch.Tensor:
        return self._native.replay(token)

    def replay_host(self, token: int | None = None) -> int:
        """One synchronous step with host buffers: `token` in, the greedy
        token sampled by the step out (``fx_decode_replay_host``)."""
        return self._native.replay_host(token)

    def generate_greedy(self, max_new_tokens: int, *, eos_token_id: int | None = None) -> torch.Tensor:
        """Greedy tokens [1, n] starting with the prefill's token: n =
        max_new_tokens, or fewer when `eos_token_id` is given and sampled (the
        EOS token is included; the device loop stops on it)."""
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be positive")
        return self._native.generate_greedy(max_new_tokens, eos_token_id)

    logits = property(lambda self: self._native.logits())
    final_hidden = property(lambda self: self._native.final_hidden())
    key_cache = property(lambda self: self._native.key_cache())
    value_cache = property(lambda self: self._native.value_cache())
    device_position = property(lambda self: self._native.device_position())
    device_cache_length = property(lambda self: self._native.device_cache_length())
    current_token = property(lambda self: self._native.current_token())
    generated_tokens = property(lambda self: self._native.generated_tokens())
    device_generation_step = property(lambda self: self._native.device_generation_step())
    cache_position = property(lambda self: int(self._native.position()))
    cache_length = property(lambda self: int(self._native.cache_length()))
    prompt_length = property(lambda self: int(self._native.prompt_length()))
    capacity = property(lambda self: int(self._native.capacity()))
    replay_count = property(lambda self: int(self._native.replay_count()))
    generation_step = property(lambda self: int(self._native.generation_step()))

    @property
    def memory(self) -> NativePrefillRuntimeMemory:
        referenced = sum(t.numel() * t.element_size() for t in self.model.parameters())
        return NativePrefillRuntimeMemory(
            cache_bytes=int(self._native.cache_bytes()), prefill_workspace_bytes=int(self._native.workspace_bytes()),
            decode_workspace_bytes=int(self._native._decode.workspace_bytes()),
            stable_buffer_bytes=int(self._native.stable_buffer_bytes()), referenced_weight_bytes=referenced)

    def stable_addresses(self) -> dict[str, int]:
        return dict(zip(_PREFILL_ADDRESS_NAMES, self._native.addresses(), strict=True))

    def native_object(self) -> NativePrefillObject:
        return self._native


class NativeSmolLM2Decode:
    """Token-to-logits native decode graph owner (``native_smollm2.py:263-605``)."""

    def __init__(self) -> None:
        raise TypeError("use NativeSmolLM2Decode.capture(...) to create a runtime")

    @classmethod
    def capture(cls, model: nn.Module, input_ids: torch.Tensor, *, max_decode_steps: int,
                initial_token: torch.Tensor | None = None) -> "NativeSmolLM2Decode":
        """Prefill eagerly (Flux eager path), then capture native decode."""
        cls._validate_capture(model, input_ids, max_decode_steps)
        with torch.inference_mode():
            prefill = model(input_ids=input_ids, use_cache=True, logits_to_keep=1)
        if not isinstance(prefill.past_key_values, DynamicCache):
            raise TypeError("native SmolLM2 prefill expected Transformers DynamicCache, got "
                            f"{type(prefill.past_key_values).__name__}")
        token = prefill.logits.argmax(dim=-1) if initial_token is None else initial_token
        keys = [layer.keys for layer in prefill.past_key_values.layers]
        values = [layer.values for layer in prefill.past_key_values.layers]
        if any(t is None for t in keys + values):
            raise ValueError("prefill produced an uninitialized decoder cache")
        self = cls.capture_from_state(model, token, keys, values, cache_position=input_ids.shape[1],
                                      cache_capacity=input_ids.shape[1] + max_decode_steps)
        self.prefill_logits = prefill.logits.detach()
        self.prefill_input_ids = input_ids
        self._prefill_cache = prefill.past_key_values
        return self

    @classmethod
    def capture_from_state(cls, model: nn.Module, initial_token: torch.Tensor, key_caches: Sequence[torch.Tensor],
                           value_caches: Sequence[torch.Tensor], *, cache_position: int,
                           cache_capacity: int) -> "NativeSmolLM2Decode":
        """Capture from an already-prefilled compact cache."""
        cls._validate_model_and_state(model, initial_token, key_caches, value_caches, cache_position=cache_position,
                                      cache_capacity=cache_capacity)
        if not native_smollm2_runtime_is_available():
            raise RuntimeError(f"flux_b200 native decode runtime is not available: {_native.load_error()}")
        device = initial_token.device
        cos, sin = _rope_tables(model, cache_capacity, device)
        weights = _model_weights(model)
        desc = _model_desc(weights, cos, sin, cache_capacity, "flux native full decode")
        rows = _validate_sources(key_caches, value_caches, cache_position, device, "flux native full decode") \
            if cache_position > 0 else 0
        keys = _native.pointer_array(t.data_ptr() for t in key_caches) if cache_position > 0 else None
        values = _native.pointer_array(t.data_ptr() for t in value_caches) if cache_position > 0 else None
        handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            _native.check(_native.load().fx_decode_create(ctypes.byref(desc), initial_token.data_ptr(), keys, values,
                                                          rows, cache_position, _stream(device), ctypes.byref(handle)))
        self = object.__new__(cls)
        self.model = model
        self._rope_cos, self._rope_sin = cos, sin
        self._source_key_caches = tuple(key_caches)
        self._source_value_caches = tuple(value_caches)
        owner = _OwnedHandle(handle.value, "fx_decode_destroy", (weights, cos, sin))
        self._native = NativeDecodeObject(handle.value, device, owner)
        self.prefill_logits = None
        self.prefill_input_ids = None
        self._prefill_cache = None
        return self

    @staticmethod
    def _validate_capture(model, input_ids, max_decode_steps) -> None:
        if input_ids.dtype != torch.long or input_ids.ndim != 2:
            raise ValueError("input_ids must be a rank-2 torch.long tensor")
        if input_ids.shape[0] != 1 or input_ids.shape[1] < 1:
            raise ValueError("native full decode requires a non-empty batch of one")
        if input_ids.device != next(model.parameters()).device:
            raise ValueError("input_ids must be on the model device")
        if max_decode_steps < 1:
            raise ValueError("max_decode_steps must be positive")
        NativeSmolLM2Decode._validate_capture_model_input(model, input_ids, input_ids.shape[1] + max_decode_steps)

    @staticmethod
    def _validate_capture_model_input(model, input_ids, requested: int) -> None:
        if input_ids.dtype != torch.long or input_ids.ndim != 2:
            raise ValueError("input_ids must be a rank-2 torch.long tensor")
        if input_ids.shape[0] != 1 or input_ids.shape[1] < 1:
            raise ValueError("native SmolLM2 runtime requires a non-empty batch of one")
        if not input_ids.is_contiguous():
            raise ValueError("input_ids must be contiguous")
        if input_ids.device != next(model.parameters()).device:
            raise ValueError("input_ids must be on the model device")
        if requested < input_ids.shape[1]:
            raise ValueError("requested capacity must include the complete prompt")
        if requested > int(model.config.max_position_embeddings):
            raise ValueError("requested native cache exceeds the model position limit")
        empty = torch.empty((1, 3, 0, 64), dtype=torch.float32, device=input_ids.device)
        NativeSmolLM2Decode._validate_model_and_state(model, input_ids[:, :1], [empty] * LAYERS, [empty] * LAYERS,
                                                      cache_position=0, cache_capacity=max(requested, 1))

    @staticmethod
    def _decode_workspace_bytes(capacity: int) -> int:
        """Reference accounting of its decode workspace (``native_smollm2.py:
        387-403``); the native object reports its own via ``workspace_bytes``."""
        chunks = (capacity + 127) // 128
        return 4 * (4 * 576 + 960 + 2 * 9 * 64 + 576 + 1536 + 576 + 2 * 64 + 9 * chunks * 66)

    @staticmethod
    def _validate_model_and_state(model, initial_token, key_caches, value_caches, *, cache_position: int,
                                  cache_capacity: int) -> None:
        """``native_smollm2.py:405-500`` with the capacity limit raised to 131072."""
        from flux_b200.integration import FINAL_FLUX_OPERATOR_CATEGORIES, FluxLlamaDecoderLayer, FluxPackedLlamaMLP

        if not torch.cuda.is_available():
            raise RuntimeError("Flux native full decode requires CUDA")
        if model.training:
            raise ValueError("Flux native full decode requires model.eval()")
        if set(getattr(model, "_flux_operator_categories", ())) != set(FINAL_FLUX_OPERATOR_CATEGORIES):
            raise ValueError("native full decode requires the retained Flux configuration")
        config = model.config
        geometry = (int(config.num_hidden_layers), int(config.hidden_size), int(config.intermediate_size),
                    int(config.num_attention_heads), int(config.num_key_value_heads), int(config.head_dim))
        if geometry != (30, 576, 1536, 9, 3, 64):
            raise ValueError("native full decode requires SmolLM2-135M geometry (30, 576, 1536, 9, 3, 64)")
        if len(model.model.layers) != LAYERS or not all(
                isinstance(layer, FluxLlamaDecoderLayer) and isinstance(layer.mlp, FluxPackedLlamaMLP)
                for layer in model.model.layers):
            raise TypeError("model does not contain 30 fully enabled Flux layers")
        if next(model.parameters()).dtype != torch.float32:
            raise TypeError("native full decode currently requires FP32 weights")
        eps = {float(model.model.norm.variance_epsilon)}
        for layer in model.model.layers:
            eps.add(float(layer.input_layernorm.variance_epsilon))
            eps.add(float(layer.post_attention_layernorm.variance_epsilon))
        if len(eps) != 1:
            raise ValueError("native full decode requires one shared RMSNorm epsilon")
        if cache_capacity < 1 or cache_capacity > MAX_CAPACITY:
            raise ValueError(f"cache_capacity must be in [1, {MAX_CAPACITY}]")
        if cache_capacity > int(config.max_position_embeddings):
            raise ValueError("cache_capacity exceeds the model position limit")
        if cache_position < 0 or cache_position >= cache_capacity:
            raise ValueError("cache_position must be inside cache_capacity")
        device = next(model.parameters()).device
        if (initial_token.shape != (1, 1) or initial_token.dtype != torch.long or initial_token.device != device
                or not initial_token.is_contiguous()):
            raise ValueError("initial_token must be contiguous CUDA long [1, 1]")
        if len(key_caches) != LAYERS or len(value_caches) != LAYERS:
            raise ValueError("one K/V source is required for each of 30 layers")
        for name, tensors in (("key", key_caches), ("value", value_caches)):
            for index, t in enumerate(tensors):
                if (t.shape[:2] != (1, 3) or t.ndim != 4 or t.shape[2] < cache_position or t.shape[3] != 64
                        or t.dtype != torch.float32 or t.device != device or not t.is_contiguous()):
                    raise ValueError(f"{name} cache layer {index} is unsupported")
        if any(k.shape != v.shape for k, v in zip(key_caches, value_caches)):
            raise ValueError("each layer's K and V source shapes must match")

    def replay(self, token: torch.Tensor | None = None) -> torch.Tensor:
        """Asynchronously enqueue an optional token copy and one graph launch."""
        return self._native.replay(token)

    def replay_host(self, token: int | None = None) -> int:
        """One synchronous step with host buffers: `token` in, the greedy
        token sampled by the step out (``fx_decode_replay_host``)."""
        return self._native.replay_host(token)

    def reset(self, token: torch.Tensor, key_caches, value_caches, *, cache_position: int) -> None:
        """Synchronously restore prefilled state outside steady replay."""
        self._native.reset(token, list(key_caches), list(value_caches), cache_position)

    logits = property(lambda self: self._native.logits())
    key_cache = property(lambda self: self._native.key_cache())
    value_cache = property(lambda self: self._native.value_cache())
    device_position = property(lambda self: self._native.device_position())
    device_cache_length = property(lambda self: self._native.device_cache_length())
    cache_position = property(lambda self: int(self._native.position()))
    cache_length = property(lambda self: int(self._native.cache_length()))
    capacity = property(lambda self: int(self._native.capacity()))
    replay_count = property(lambda self: int(self._native.replay_count()))

    @property
    def memory(self) -> NativeDecodeRuntimeMemory:
        referenced = sum(t.numel() * t.element_size() for t in self.model.parameters())
        return NativeDecodeRuntimeMemory(
            cache_bytes=(self.key_cache.numel() + self.value_cache.numel()) * self.key_cache.element_size(),
            workspace_bytes=int(self._native.workspace_bytes()),
            stable_buffer_bytes=int(self._native.stable_buffer_bytes()), referenced_weight_bytes=referenced)

    def stable_addresses(self) -> dict[str, int]:
        return dict(zip(_ADDRESS_NAMES, self._native.addresses(), strict=True))

    def native_object(self) -> NativeDecodeObject:
        return self._native


def native_smollm2_greedy_generate(model: nn.Module, input_ids: torch.Tensor, *, max_new_tokens: int,
                                   eos_token_id: int | None = None) -> torch.Tensor:
    """Generate greedily with native prefill and native decode replay (stopping
    on device after `eos_token_id` when given)."""
    if max_new_tokens < 1:
        raise ValueError("max_new_tokens must be positive")
    runtime = NativeSmolLM2Prefill.capture(model, input_ids, max_decode_steps=max_new_tokens - 1)
    generated = runtime.generate_greedy(max_new_tokens, eos_token_id=eos_token_id)
    return torch.cat((input_ids, generated), dim=-1)


class NativeSmolLM2BatchedDecode:
    """Greedy decode of ``batch`` (1..64) independent sequences advanced
    together, one CUDA-graph replay per step (``fx_batch_*``).

    No counterpart in the reference, whose runtime is batch 1 only; the
    sequence-sharded batched configuration runs one of these per GPU with its
    own sequences and nothing shared between GPUs.  Sequence ``i`` is installed
    with :meth:`load` from a compact per-layer cache ``[1, 3, rows, 64]`` (or
    ``[3, rows, 64]``) and its next input token; :meth:`step` then advances
    every sequence by greedy steps, each at its own position."""

    _PREFIX = "flux native batched decode"

    def __init__(self, model: nn.Module, batch: int, cache_capacity: int, generated_capacity: int | None = None):
        if not 1 <= batch <= 64:
            raise ValueError("batched decode supports 1 to 64 sequences per runtime")
        if cache_capacity < 1 or cache_capacity > int(model.config.max_position_embeddings):
            raise ValueError("requested native cache exceeds the model position limit")
        if not native_smollm2_runtime_is_available():
            raise RuntimeError(f"flux_b200 native runtime is not available: {_native.load_error()}")
        device = next(model.parameters()).device
        cos, sin = _rope_tables(model, cache_capacity, device)
        weights = _model_weights(model)
        desc = _model_desc(weights, cos, sin, cache_capacity, self._PREFIX)
        generated_capacity = cache_capacity if generated_capacity is None else int(generated_capacity)
        handle = ctypes.c_void_p()
        lib = _native.load()
        with torch.cuda.device(device):
            _native.check(lib.fx_batch_create(ctypes.byref(desc), batch, generated_capacity, _stream(device),
                                              ctypes.byref(handle)))
        self._owner = _OwnedHandle(handle.value, "fx_batch_destroy", (weights, cos, sin, desc))
        self._handle = handle.value
        self._device = device
        self.batch = batch
        self.capacity = cache_capacity
        b = _native.BatchBuffers()
        _native.check(lib.fx_batch_get_buffers(self._handle, ctypes.byref(b)))
        vocab = int(weights["embedding"].shape[0])
        self._tokens = _view(b.tokens, (batch,), torch.long, self._owner, device)
        self._positions = _view(b.positions, (batch,), torch.long, self._owner, device)
        self._logits = _view(b.logits, (batch, vocab), torch.float32, self._owner, device)
        self._generated = _view(b.generated, (batch, b.generated_capacity), torch.long, self._owner, device)
        self._step = _view(b.step, (1,), torch.long, self._owner, device)
        shape = (LAYERS, batch, 3, cache_capacity, 64)
        self._key_cache = _view(b.key_cache, shape, torch.float32, self._owner, device)
        self._value_cache = _view(b.value_cache, shape, torch.float32, self._owner, device)
        self.kernels_per_step = int(b.kernels_per_step)

    def load(self, index: int, token: torch.Tensor | int, key_caches: Sequence[torch.Tensor],
             value_caches: Sequence[torch.Tensor], length: int) -> None:
        """Install sequence ``index``: ``length`` cached rows per layer and its next input token."""
        if not 0 <= index < self.batch:
            raise ValueError("sequence index out of range")
        if not 0 <= length < self.capacity:
            raise RuntimeError(f"{self._PREFIX}: length must be within cache capacity")
        if not isinstance(token, torch.Tensor):
            token = torch.tensor([int(token)], dtype=torch.long, device=self._device)
        token = token.reshape(1).to(device=self._device, dtype=torch.long).contiguous()
        rows, keys, values = 0, None, None
        if length > 0:
            if len(key_caches) != LAYERS or len(value_caches) != LAYERS:
                raise RuntimeError(f"{self._PREFIX}: one K/V tensor per layer is required")
            srcs = []
            for t in list(key_caches) + list(value_caches):
                t3 = t.reshape(3, t.shape[-2], 64) if t.dim() in (3, 4) else t
                if t3.device != self._device or t3.dtype != torch.float32 or not t3.is_contiguous():
                    raise RuntimeError(f"{self._PREFIX}: K/V sources must be contiguous float32 on the runtime device")
                srcs.append(t3)
            rows = int(srcs[0].shape[1])
            if rows < length or any(int(t.shape[1]) != rows for t in srcs):
                raise RuntimeError(f"{self._PREFIX}: K/V sources must hold `length` rows")
            keys = _native.pointer_array(t.data_ptr() for t in srcs[:LAYERS])
            values = _native.pointer_array(t.data_ptr() for t in srcs[LAYERS:])
            self._keepalive = (srcs, token)
        with torch.cuda.device(self._device):
            _native.check(_native.load().fx_batch_load(self._handle, index, token.data_ptr(), keys, values, rows,
                                                       length, _stream(self._device)))

    def step(self, steps: int = 1) -> torch.Tensor:
        """Enqueue ``steps`` greedy steps; returns the (stable) logits ``[B, vocab]`` of the last."""
        with torch.cuda.device(self._device):
            _native.check(_native.load().fx_batch_step(self._handle, steps, _stream(self._device)))
        return self._logits

    def check(self) -> None:
        """Wait for enqueued steps; raise if a kernel reported an error."""
        _native.check(_native.load().fx_batch_check(self._handle))

    def logits(self) -> torch.Tensor: return self._logits
    def tokens(self) -> torch.Tensor: return self._tokens
    def positions(self) -> torch.Tensor: return self._positions
    def generated_tokens(self) -> torch.Tensor: return self._generated
    def device_generation_step(self) -> torch.Tensor: return self._step
    def key_cache(self) -> torch.Tensor: return self._key_cache
    def value_cache(self) -> torch.Tensor: return self._value_cache


__all__ = [
    "NativeDecodeRuntimeMemory", "NativePrefillRuntimeMemory", "NativeSmolLM2BatchedDecode", "NativeSmolLM2Decode",
    "NativeSmolLM2Prefill", "native_smollm2_greedy_generate", "native_smollm2_prefill_is_available",
    "native_smollm2_runtime_is_available",
]
