"""CPU-side checks of libkvc.so: it loads, exports every symbol include/*.h
declares, its host codecs and parameter defaults match the reference, and
without a GPU its compaction entry points fail loudly (-10), never falling
back to a CPU path."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import REPO, golden_path, has_gpu, load_case
from kvc_b200 import abi, lib as kvclib


def declared_functions(header):
    """Names of the non-inline function declarations of a public header."""
    src = open(os.path.join(REPO, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    src = re.sub(r"^\s*#[^\n]*", "", src, flags=re.M)
    src = src.replace('extern "C" {', "")
    # drop bodies of inline helpers and struct/enum definitions
    while "{" in src:
        src = re.sub(r"\{[^{}]*\}", ";", src)
    names = set()
    for stmt in src.split(";"):
        stmt = " ".join(stmt.split())
        if "(" not in stmt or stmt.startswith("typedef") or "static inline" in stmt or 'extern "C"' in stmt:
            continue
        m = re.search(r"([A-Za-z_]\w*)\s*\(", stmt)
        if m:
            names.add(m.group(1))
    return sorted(names)


@pytest.mark.parametrize("header", ["kv-compact-api.h", "kv-compact-accel-cuda.h", "kvc-batched.h", "kvc-peer.h"])
def test_every_declared_symbol_is_exported(kvc, header):
    names = declared_functions(header)
    assert names, header
    for n in names:
        assert hasattr(kvc["_lib"], n), f"{n} declared in {header} but not exported"


def test_symbol_lists_cover_headers():
    declared = set()
    for h in ("kv-compact-api.h", "kv-compact-accel-cuda.h", "kvc-batched.h", "kvc-peer.h"):
        declared |= set(declared_functions(h))
    listed = set(kvclib.DROPIN_SYMBOLS + kvclib.SEAM_SYMBOLS + kvclib.BATCHED_SYMBOLS + kvclib.PEER_SYMBOLS)
    assert declared == listed


def test_params_default_matches_reference(kvc, oracle):
    a, b = kvc["params_default"](), oracle["params_default"]()
    for f in abi.PARAM_FIELDS:
        va, vb = getattr(a, f), getattr(b, f)
        if f in ("layer_filter", "reasoning"):
            assert not va and not vb
        else:
            assert va == vb, f


def test_struct_layout_sizes():
    """kv_compact_params: 22 fields, 3 trailing pointers (reference
    include/kv-compact-api.h:133-215); result and quant result layouts."""
    assert len(abi.Params._fields_) == 22
    assert ctypes.sizeof(abi.Params) == 19 * 4 + 4 + 3 * 8  # 19 ints/floats, pad, 3 pointers
    assert ctypes.sizeof(abi.Stats) == 3 * 4 + 4 + 3 * 8
    assert ctypes.sizeof(abi.Result) == 2 * 4 + 3 * 8 + ctypes.sizeof(abi.Stats)


def test_host_codecs_bitexact_vs_reference_fixture(kvc):
    case = load_case(golden_path("codecs"))
    X = case["X"]
    for typ, tag in ((0, "f32"), (1, "f16"), (2, "q4_0"), (3, "q4_1"), (8, "q8_0")):
        B = abi.quantize_rows(kvc, X, typ)
        np.testing.assert_array_equal(B, case["enc_" + tag])
        D = abi.dequantize_rows(kvc, B, typ, X.shape[1])
        np.testing.assert_array_equal(D, case["dec_" + tag])
    rb = [kvc["quant_row_bytes"](t, 128) for t in (0, 1, 2, 3, 8)]
    np.testing.assert_array_equal(rb, case["row_bytes"])


def test_host_codecs_random_vs_oracle(kvc, oracle):
    rng = np.random.default_rng(3)
    X = (rng.standard_normal((64, 256)) * rng.choice([1e-4, 1.0, 1e3], size=(64, 1))).astype(np.float32)
    X[5, :] = 0.0
    X[6, ::7] = -0.0
    for typ in (0, 1, 2, 3, 8):
        np.testing.assert_array_equal(abi.quantize_rows(kvc, X, typ), abi.quantize_rows(oracle, X, typ))


@pytest.mark.skipif(has_gpu(), reason="checks the no-device behaviour")
def test_no_device_fails_loudly(kvc):
    K = np.ones((16, 8), np.float32)
    r = abi.Result()
    rc = kvc["kv_compact"](abi.fptr(K), abi.fptr(K), abi.fptr(K[:4]), 16, 4, 1, 8, 8, None, ctypes.byref(r))
    assert rc == -10
    assert kvc["_lib"].kv_compact_cuda_available() == 0


def test_error_codes_before_device(kvc):
    """Argument errors are reported before any device is touched."""
    K = np.ones((8, 4), np.float32)
    Q = np.ones((2, 4), np.float32)
    r = abi.Result()
    f = kvc["kv_compact"]
    assert f(None, abi.fptr(K), abi.fptr(Q), 8, 2, 1, 4, 4, None, r) == -1
    assert f(abi.fptr(K), abi.fptr(K), abi.fptr(Q), 0, 2, 1, 4, 4, None, r) == -2
    assert f(abi.fptr(K), abi.fptr(K), abi.fptr(Q), 8, 0, 1, 4, 4, None, r) == -2
    mr = kvc["kv_compact_multi_round"]
    assert mr(abi.fptr(K), abi.fptr(K), abi.fptr(Q), 8, 2, 1, 4, 4, None, 0, r, None) == -3
    assert mr(abi.fptr(K), abi.fptr(K), None, 8, 2, 1, 4, 4, None, 1, r, None) == -1
    Kq = np.zeros((8, 34), np.uint8)
    qr = abi.QuantResult()
    qf = kvc["kv_compact_quantized"]
    assert qf(abi.u8ptr(Kq), abi.u8ptr(Kq), abi.fptr(Q), 8, 8, 34, 34, 8, 2, 1, 16, 16, None, qr) == -4


def test_free_is_double_free_safe(kvc):
    r = abi.Result()
    kvc["result_free"](ctypes.byref(r))
    kvc["result_free"](ctypes.byref(r))
    q = abi.QuantResult()
    kvc["quant_result_free"](ctypes.byref(q))
    kvc["quant_result_free"](ctypes.byref(q))
