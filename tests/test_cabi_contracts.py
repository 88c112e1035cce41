"""CPU checks of the C ABI's argument contracts (``include/flux_b200.h``): the
entry points refuse bad arguments with a status code and an ``fx_last_error``
message before they touch the GPU, so an FFI caller (ctypes, cgo, JNI) can rely
on them on any host.  No call here reaches CUDA."""

from __future__ import annotations

import ctypes

import pytest

from flux_b200 import _native

FAKE = 0x100000  # a non-null, 16-byte aligned address that is never dereferenced


def _desc(**overrides) -> _native.ModelDesc:
    d = _native.ModelDesc()
    d.device, d.vocab, d.capacity, d.epsilon = 0, 49152, 256, 1e-5
    d.embedding = d.final_norm = d.lm_head = d.rope_cos = d.rope_sin = FAKE
    for l in range(_native.LAYERS):
        d.input_norm[l] = d.packed_qkv[l] = d.o_proj[l] = FAKE
        d.post_norm[l] = d.gate_up[l] = d.down[l] = FAKE
        d.attention_scale[l] = 0.125
    for key, value in overrides.items():
        if key.endswith("_layer0"):
            getattr(d, key[: -len("_layer0")])[0] = value
        else:
            setattr(d, key, value)
    return d


def _refused(status: int, status_expected: int, message: str) -> None:
    assert status == status_expected
    assert message in _native.load().fx_last_error().decode()


@pytest.mark.parametrize("overrides,message", [
    ({"capacity": 0}, "cache capacity must be in [1, 131072]"),
    ({"capacity": 131073}, "cache capacity must be in [1, 131072]"),
    ({"vocab": 0}, "vocabulary must be non-empty"),
    ({"epsilon": 0.0}, "epsilon must be positive"),
    ({"lm_head": None}, "a model tensor pointer is null"),
    ({"down_layer0": None}, "exactly 30 complete layer descriptors"),
    ({"packed_qkv_layer0": FAKE + 4}, "16-byte aligned"),
    ({"attention_scale_layer0": float("inf")}, "attention scale must be finite"),
])
def test_decode_create_validates_the_model(overrides, message):
    lib = _native.load()
    desc = _desc(**overrides)
    token = ctypes.c_int64(1)
    out = ctypes.c_void_p(FAKE)
    status = lib.fx_decode_create(ctypes.byref(desc), ctypes.addressof(token), None, None, 0, 0, None,
                                  ctypes.byref(out))
    _refused(status, _native.FX_ERR_INVALID, message)
    assert out.value is None  # the output handle is cleared on refusal


def test_decode_create_checks_token_and_position():
    lib = _native.load()
    desc = _desc()
    out = ctypes.c_void_p()
    _refused(lib.fx_decode_create(ctypes.byref(desc), None, None, None, 0, 0, None, ctypes.byref(out)),
             _native.FX_ERR_INVALID, "initial token is null")
    token = ctypes.c_int64(1)
    _refused(lib.fx_decode_create(ctypes.byref(desc), ctypes.addressof(token), None, None, 0, 256, None,
                                  ctypes.byref(out)),
             _native.FX_ERR_INVALID, "initial position must be inside capacity")
    _refused(lib.fx_decode_create(ctypes.byref(desc), ctypes.addressof(token), None, None, 0, 5, None,
                                  ctypes.byref(out)),
             _native.FX_ERR_INVALID, "every K/V source must be contiguous")


def test_null_runtime_handles_are_refused():
    lib = _native.load()
    _refused(lib.fx_decode_replay(None, None, None), _native.FX_ERR_INVALID, "runtime is null")
    nxt = ctypes.c_int64()
    _refused(lib.fx_decode_replay_host(None, None, ctypes.addressof(nxt), None), _native.FX_ERR_INVALID,
             "null pointer")
    _refused(lib.fx_decode_generate(None, 1, None), _native.FX_ERR_INVALID, "runtime is null")


@pytest.mark.parametrize("batch,generated,message", [
    (0, 8, "batch must be in [1, 64]"),
    (65, 8, "batch must be in [1, 64]"),
    (4, 0, "generated capacity must be in [1, 131072]"),
])
def test_batch_create_validates_sizes(batch, generated, message):
    lib = _native.load()
    desc = _desc()
    out = ctypes.c_void_p()
    _refused(lib.fx_batch_create(ctypes.byref(desc), batch, generated, None, ctypes.byref(out)),
             _native.FX_ERR_INVALID, message)


def test_tensor_core_projection_validates_shapes():
    lib = _native.load()
    err = ctypes.c_int32()
    args = (FAKE, FAKE, FAKE, None, FAKE)
    _refused(lib.fx_linear_3xtf32_f32(*args, 4, 33, 64, ctypes.addressof(err), None), _native.FX_ERR_INVALID,
             "K a positive multiple of 32")
    _refused(lib.fx_linear_3xtf32_f32(*args, 0, 64, 64, ctypes.addressof(err), None), _native.FX_ERR_INVALID,
             "K a positive multiple of 32")
    _refused(lib.fx_linear_3xtf32_f32(None, FAKE, FAKE, None, FAKE, 4, 64, 64, ctypes.addressof(err), None),
             _native.FX_ERR_INVALID, "null pointer")


def test_static_scratch_attention_refuses_oversized_problems_before_the_gpu():
    lib = _native.load()
    limit = lib.fx_gqa_decode_attention_static_scratch_floats()
    capacity = 128 * (limit // (9 * 66) + 1)
    assert lib.fx_gqa_decode_attention_workspace_floats(1, 9, capacity, 64) > limit
    strides = _native.int64_array([1, 1, 1, 1])
    status = lib.fx_gqa_decode_attention_static_scratch_f32(
        FAKE, strides, FAKE, strides, FAKE, strides, None, None, None, None, FAKE, 0.125, 1, 9, 3, capacity, 64,
        None)
    _refused(status, _native.FX_ERR_INVALID, "static array")


def test_attention_workspace_size_refuses_overflowing_products():
    """A product that does not fit int64 reports INT64_MAX (no workspace is
    large enough) instead of wrapping to a small size that would pass the
    static-array and workspace checks."""
    lib = _native.load()
    int64_max = (1 << 63) - 1
    assert lib.fx_gqa_decode_attention_workspace_floats(1 << 20, 1 << 20, 1 << 40, 64) == int64_max
    assert lib.fx_gqa_decode_attention_workspace_floats(1, 9, int64_max, 64) == int64_max
    assert lib.fx_gqa_decode_attention_workspace_floats(0, 9, 1024, 64) == 0
    strides = _native.int64_array([1, 1, 1, 1])
    # query heads up to 16 x KV heads and head_dim <= 256 are checked before any size product
    for hq, hkv, d in ((1 << 40, 1 << 10, 64), (9, 3, 1 << 20), ((1 << 20) * 16, 1 << 20, 64)):
        status = lib.fx_gqa_decode_attention_static_scratch_f32(
            FAKE, strides, FAKE, strides, FAKE, strides, None, None, None, None, FAKE, 0.125, 1, hq, hkv, 1024, d,
            None)
        _refused(status, _native.FX_ERR_INVALID, "head_dim <= 256")


C_CALLER = r"""
#include "flux_b200.h"
#include <stdio.h>
#include <string.h>
int main(void) {
    fx_model_desc m = {0};
    fx_decode* d = 0;
    int64_t token = 1;
    fx_status st = fx_decode_create(&m, &token, 0, 0, 0, 0, 0, &d);
    puts(fx_last_error());
    return st == FX_ERR_INVALID && d == 0 && strstr(fx_last_error(), "vocabulary") != 0 ? 0 : 1;
}
"""


def test_header_is_plain_c_and_links(tmp_path):
    """A C99 caller (what cgo or any C FFI generator sees) compiles against
    include/flux_b200.h with -pedantic, links against the library, and reads
    a refusal through fx_last_error."""
    import shutil
    import subprocess
    from pathlib import Path
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    root = Path(__file__).resolve().parent.parent
    lib_dir = _native.LIBRARY_PATH.parent
    src, exe = tmp_path / "caller.c", tmp_path / "caller"
    src.write_text(C_CALLER)
    build = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", f"-I{root / 'include'}",
                            str(src), f"-L{lib_dir}", "-lfluxb200", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "vocabulary must be non-empty" in run.stdout
