"""ctypes binding of ``libfluxb200.so`` (the C ABI declared in ``include/flux_b200.h``).

The library is the only compute path.  If it has not been built, every entry
point raises :class:`NativeLibraryUnavailable` -- there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "_lib" / "libfluxb200.so"
LAYERS = 30

FX_OK = 0
FX_ERR_INVALID = 1
FX_ERR_CUDA = 2
FX_ERR_EXHAUSTED = 3
FX_ERR_STATE = 4
FX_ERR_DEVICE = 5

STATE_POSITION = 0
STATE_CACHE_LENGTH = 1
STATE_GENERATION_STEP = 2

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float
_st = ctypes.c_int32


class NativeLibraryUnavailable(RuntimeError):
    """``libfluxb200.so`` is missing or failed to load."""


class ModelDesc(ctypes.Structure):
    """``fx_model_desc``."""

    _fields_ = [
        ("device", _i32),
        ("vocab", _i64),
        ("capacity", _i64),
        ("epsilon", _f32),
        ("embedding", _p),
        ("final_norm", _p),
        ("lm_head", _p),
        ("rope_cos", _p),
        ("rope_sin", _p),
        ("input_norm", _p * LAYERS),
        ("packed_qkv", _p * LAYERS),
        ("o_proj", _p * LAYERS),
        ("post_norm", _p * LAYERS),
        ("gate_up", _p * LAYERS),
        ("down", _p * LAYERS),
        ("attention_scale", _f32 * LAYERS),
    ]


class DecodeBuffers(ctypes.Structure):
    """``fx_decode_buffers``."""

    _fields_ = [
        ("input_token", _p),
        ("logits", _p),
        ("generated_tokens", _p),
        ("generation_step", _p),
        ("key_cache", _p),
        ("value_cache", _p),
        ("position", _p),
        ("cache_length", _p),
        ("workspace", _p),
        ("workspace_bytes", _i64),
        ("hidden_a", _p),
        ("hidden_b", _p),
        ("final_norm_output", _p),
        ("attention_workspace", _p),
        ("stable_buffer_bytes", _i64),
        ("timeline", _p),
        ("timeline_ctas", _i64),
        ("timeline_events", _i64),
    ]


class DecodeInfo(ctypes.Structure):
    """``fx_decode_info``."""

    _fields_ = [
        ("capacity", _i64),
        ("vocab", _i64),
        ("start_position", _i64),
        ("replay_count", _i64),
        ("kernels_per_step", _i64),
    ]


class PrefillBuffers(ctypes.Structure):
    """``fx_prefill_buffers``."""

    _fields_ = [
        ("prefill_logits", _p),
        ("workspace", _p),
        ("workspace_bytes", _i64),
        ("attention_output", _p),
        ("final_hidden", _p),
        ("initial_token", _p),
    ]


class BatchBuffers(ctypes.Structure):
    """``fx_batch_buffers``."""

    _fields_ = [
        ("tokens", _p),
        ("positions", _p),
        ("logits", _p),
        ("generated", _p),
        ("step", _p),
        ("key_cache", _p),
        ("value_cache", _p),
        ("batch", _i64),
        ("capacity", _i64),
        ("generated_capacity", _i64),
        ("kernels_per_step", _i64),
    ]


# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "fx_last_error": (ctypes.c_char_p, []),
    "fx_version": (ctypes.c_char_p, []),
    "fx_rmsnorm_f32": (_st, [_p, _p, _p, _i64, _i64, _f32, _p]),
    "fx_residual_rmsnorm_f32": (_st, [_p, _p, _p, _p, _p, _i64, _i64, _f32, _p]),
    "fx_packed_swiglu_f32": (_st, [_p, _p, _i64, _i64, _p]),
    "fx_softmax_f32": (_st, [_p, _p, _i64, _i64, _p]),
    "fx_attention_score_softmax_f32": (_st, [_p, _p, _p, _p, _p, _f32, _p, _p]),
    "fx_rope_f32": (_st, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p]),
    "fx_packed_qkv_rope_cache_f32": (_st, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p]),
    "fx_gqa_decode_attention_workspace_floats": (_i64, [_i64, _i64, _i64, _i64]),
    "fx_gqa_decode_attention_f32": (_st, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _f32,
                                          _i64, _i64, _i64, _i64, _i64, _p]),
    "fx_gqa_decode_attention_static_scratch_floats": (_i64, []),
    "fx_gqa_decode_attention_static_scratch_f32": (_st, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f32,
                                                         _i64, _i64, _i64, _i64, _i64, _p]),
    "fx_packed_gate_up_swiglu_f32": (_st, [_p, _p, _p, _i64, _i64, _p]),
    "fx_linear_f32": (_st, [_p, _p, _p, _i64, _i64, _i64, _p]),
    "fx_tf32_split_f32": (_st, [_p, _p, _p, _i64, _p]),
    "fx_linear_3xtf32_f32": (_st, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p]),
    "fx_greedy_argmax_f32": (_st, [_p, _i64, _p, _p]),
    "fx_greedy_argmax_update_f32": (_st, [_p, _i64, _p, _p, _i64, _p, _p, _p, _p]),
    "fx_decode_create": (_st, [ctypes.POINTER(ModelDesc), _p, _p, _p, _i64, _i64, _p, ctypes.POINTER(_p)]),
    "fx_decode_replay": (_st, [_p, _p, _p]),
    "fx_decode_replay_host": (_st, [_p, _p, _p, _p]),
    "fx_decode_generate": (_st, [_p, _i64, _p]),
    "fx_decode_reset": (_st, [_p, _p, _p, _p, _i64, _i64, _p]),
    "fx_decode_inject_failure": (_st, [_p, ctypes.c_int32]),
    "fx_decode_set_eos": (_st, [_p, _i64]),
    "fx_decode_install_prefill": (_st, [_p, _p, _i64, _p]),
    "fx_decode_wait": (_st, [_p, _p]),
    "fx_decode_get_buffers": (_st, [_p, ctypes.POINTER(DecodeBuffers)]),
    "fx_decode_read_state": (_st, [_p, _i32, ctypes.POINTER(_i64)]),
    "fx_decode_get_info": (_st, [_p, ctypes.POINTER(DecodeInfo)]),
    "fx_decode_destroy": (None, [_p]),
    "fx_batch_create": (_st, [ctypes.POINTER(ModelDesc), _i64, _i64, _p, ctypes.POINTER(_p)]),
    "fx_batch_load": (_st, [_p, _i64, _p, _p, _p, _i64, _i64, _p]),
    "fx_batch_step": (_st, [_p, _i64, _p]),
    "fx_batch_wait": (_st, [_p, _p]),
    "fx_batch_check": (_st, [_p]),
    "fx_batch_get_buffers": (_st, [_p, ctypes.POINTER(BatchBuffers)]),
    "fx_batch_destroy": (None, [_p]),
    "fx_prefill_create": (_st, [ctypes.POINTER(ModelDesc), _p, _i64, _p, ctypes.POINTER(_p)]),
    "fx_prefill_run": (_st, [_p, _p, _p]),
    "fx_prefill_decode": (_p, [_p]),
    "fx_prefill_get_buffers": (_st, [_p, ctypes.POINTER(PrefillBuffers)]),
    "fx_prefill_prompt_length": (_i64, [_p]),
    "fx_prefill_destroy": (None, [_p]),
}

_LIB: ctypes.CDLL | None = None
_LOAD_ERROR: Exception | None = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with every signature declared."""
    global _LIB, _LOAD_ERROR
    if _LIB is not None:
        return _LIB
    target = Path(path) if path is not None else LIBRARY_PATH
    if not target.exists():
        _LOAD_ERROR = NativeLibraryUnavailable(
            f"flux_b200 native library is not built ({target} is missing); "
            "run `python -m flux_b200.build`")
        raise _LOAD_ERROR
    try:
        lib = ctypes.CDLL(str(target))
    except OSError as error:
        _LOAD_ERROR = NativeLibraryUnavailable(f"failed to load {target}: {error}")
        raise _LOAD_ERROR from error
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    _LOAD_ERROR = None
    return lib


TORCH_CLASSES_PATH = LIBRARY_PATH.with_name("libfluxb200_torch.so")
_TORCH_CLASSES: bool | None = None


def load_torch_classes() -> bool:
    """Register ``torch.classes.flux.NativeSmolLM2Decode`` / ``NativeSmolLM2Prefill``
    (``libfluxb200_torch.so``, the reference's custom-class surface over this
    library); False when that library is not built or does not load.  The C
    library loads first so both share one copy of it."""
    global _TORCH_CLASSES
    if _TORCH_CLASSES is None:
        _TORCH_CLASSES = False
        if TORCH_CLASSES_PATH.exists():
            try:
                load()
                import torch
                torch.classes.load_library(str(TORCH_CLASSES_PATH))
                _TORCH_CLASSES = True
            except (OSError, RuntimeError, NativeLibraryUnavailable):
                _TORCH_CLASSES = False
    return _TORCH_CLASSES


def is_available() -> bool:
    try:
        load()
    except NativeLibraryUnavailable:
        return False
    return True


def load_error() -> Exception | None:
    try:
        load()
    except NativeLibraryUnavailable:
        pass
    return _LOAD_ERROR


class NativeError(RuntimeError):
    """A non-zero ``fx_status``; ``status`` keeps the code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def check(status: int) -> None:
    if status != FX_OK:
        message = load().fx_last_error().decode("utf-8", "replace")
        raise NativeError(status, message or f"flux_b200 call failed with status {status}")


def int64_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    return (_i64 * len(values))(*values)


def pointer_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    return (_p * len(values))(*values)
