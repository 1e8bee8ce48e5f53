"""Drop-in conformance of libhyperion_mlx.so at the C boundary (CPU only).

* the reference's own ABI contract test (native/hyperion_mlx/tests/abi_contract_test.cc),
  compiled unchanged against this repository's header and library;
* the header compiles as strict C11 (as abi_c_header_test.c requires);
* every function declared in include/*.h is exported, and exactly 14 hyp_* functions;
* struct layouts (HypCanaryInfo is 224 bytes with the reference's offsets).
"""
import ctypes
import os
import re
import subprocess

import pytest

import hyperion_b200 as hb

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(REPO, "include")


def declared(header):
    src = open(os.path.join(INC, header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b((?:hyp|hyb)_[a-z0-9_]+)\s*\(", src)))


def test_header_compiles_as_strict_c11(tmp_path):
    c = tmp_path / "t.c"
    c.write_text('#include "hyperion_mlx.h"\n#include "hyperion_b200.h"\nint main(void){return (int)sizeof(HypCanaryInfo) - 224;}\n')
    exe = tmp_path / "t"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Wpedantic", "-Werror", "-I", INC, str(c), "-o", str(exe)],
                   check=True)
    assert subprocess.run([str(exe)]).returncode == 0


def test_all_declared_symbols_exported(built_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", hb.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\s[TW]\s+(\S+)", out))
    abi = declared("hyperion_mlx.h")
    ext = declared("hyperion_b200.h")
    assert abi == sorted(hb.ABI_FUNCTIONS)
    assert len(abi) == 14
    for name in abi + ext:
        assert name in exported, name
    assert set(ext) == set(hb.EXT_FUNCTIONS)
    assert sorted(n for n in exported if n.startswith("hyp_")) == sorted(abi)


def test_struct_layouts():
    assert ctypes.sizeof(hb.HypCanaryInfo) == 224
    assert hb.HypCanaryInfo.recommended_working_set_bytes.offset == 32
    assert hb.HypCanaryInfo.mlx_runtime_version.offset == 64
    assert hb.HypCanaryInfo.gpu_name.offset == 96


def test_reference_abi_contract_test_passes(built_lib):
    from oracle.build_oracle import build_ref, reference_present
    if not reference_present():
        pytest.skip("reference tree not mounted")
    exe = build_ref(hb.LIB_PATH)["abi_contract_test"]
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr


def test_handle_lifecycle_and_errors_without_gpu(built_lib):
    L = built_lib
    assert L.hyp_runtime_canary(None) == hb.INVALID_ARGUMENT
    assert "non-null output pointer" in hb.last_error()
    one = ctypes.create_string_buffer(1)
    assert L.hyp_last_error(one, 1) == hb.OK and one.raw == b"\x00"
    assert L.hyp_last_error(None, 0) == hb.INVALID_ARGUMENT
    m = ctypes.c_void_p()
    assert L.hyp_model_create(ctypes.byref(m)) == hb.OK
    kv = ctypes.c_void_p()
    assert L.hyp_kvstate_create(m, ctypes.byref(kv)) == hb.INVALID_ARGUMENT and not kv.value
    r = ctypes.c_void_p()
    assert L.hyp_step_result_create(ctypes.byref(r)) == hb.OK
    # a step-result handle passed as a model is rejected by its magic tag
    g = hb.geometry_params(__import__("hyperion_b200.synth", fromlist=["config0"]).config0())
    assert L.hyp_model_load(r, ctypes.byref(g), b"x") == hb.INVALID_ARGUMENT
    f = hb.HypStepResultFields()
    assert L.hyp_step_result_fields(r, ctypes.byref(f)) == hb.OK
    assert L.hyp_step_result_fields(r, None) == hb.INVALID_ARGUMENT
    assert L.hyp_decode_block(m, None, 1, r) == hb.INVALID_ARGUMENT
    # batched decode, clone and speculative verify validate before any device work
    tok = (ctypes.c_uint32 * 9)()
    acc = ctypes.c_uint32()
    assert L.hyb_verify(m, None, tok, 2, tok, None, ctypes.byref(acc)) == hb.INVALID_ARGUMENT
    assert L.hyb_verify(None, None, tok, 2, tok, None, ctypes.byref(acc)) == hb.INVALID_ARGUMENT
    assert L.hyb_decode_batch(m, None, 1, tok, None) == hb.INVALID_ARGUMENT
    assert "not loaded" in hb.last_error()
    out = ctypes.c_void_p()
    assert L.hyb_kvstate_clone(m, None, 0, ctypes.byref(out)) == hb.INVALID_ARGUMENT and not out.value
    assert L.hyp_step_result_free(ctypes.byref(r)) == hb.OK and not r.value
    assert L.hyp_step_result_free(ctypes.byref(r)) == hb.OK
    assert L.hyp_model_free(ctypes.byref(m)) == hb.OK and not m.value
    assert L.hyp_model_free(None) == hb.INVALID_ARGUMENT
    # op-level argument validation happens before any device work
    assert L.hyb_quantized_matmul(None, None, None, None, None, 1, 64, 8, 64, 4, None) == hb.INVALID_ARGUMENT
    assert L.hyb_quantized_matmul(None, None, None, None, None, 1, 64, 8, 32, 4, None) == hb.UNSUPPORTED
