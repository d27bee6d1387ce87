"""Pin the CPU oracle: the C restatement in oracle/ must reproduce, bit for
bit, the outputs the reference library produced for every golden fixture
(fixtures: tests/golden/make_golden.py, which runs the reference itself)."""
import ctypes

import numpy as np
import pytest

from caserun import run_case
from conftest import golden_cases, golden_path, load_case
from kvc_b200 import abi

CASES = [c for c in golden_cases() if c != "codecs"]


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_bitexact(oracle, name):
    case = load_case(golden_path(name))
    rc, out = run_case(oracle, case)
    assert rc == 0
    assert out["t"] == int(case["t"])
    np.testing.assert_array_equal(out["indices"], case["indices"])
    np.testing.assert_array_equal(out["beta"], case["beta"])
    np.testing.assert_array_equal(out["C_v"], case["C_v"])
    np.testing.assert_array_equal(out["stats_arr"], case["stats"])
    if "K_out" in case:
        np.testing.assert_array_equal(out["K_out"], case["K_out"])
        np.testing.assert_array_equal(out["V_out"], case["V_out"])
    if "per_round" in case:
        pr = np.array([[s["avg_cosine_sim"], s["avg_mse"], s["avg_agreement"]] for s in out["per_round"]], np.float32)
        np.testing.assert_array_equal(pr, case["per_round"])


def test_oracle_codecs_bitexact(oracle):
    case = load_case(golden_path("codecs"))
    X = case["X"]
    for typ, tag in ((0, "f32"), (1, "f16"), (2, "q4_0"), (3, "q4_1"), (8, "q8_0")):
        B = abi.quantize_rows(oracle, X, typ)
        np.testing.assert_array_equal(B, case["enc_" + tag])
        D = abi.dequantize_rows(oracle, B, typ, X.shape[1])
        np.testing.assert_array_equal(D, case["dec_" + tag])
    rb = [oracle["quant_row_bytes"](t, 128) for t in (0, 1, 2, 3, 8)]
    np.testing.assert_array_equal(rb, case["row_bytes"])
    re = [oracle["quant_row_elements"](t, b) for t, b in ((0, 512), (1, 256), (2, 72), (3, 80), (8, 136))]
    np.testing.assert_array_equal(re, case["row_elems"])


def test_oracle_error_codes(oracle):
    """Return codes of the reference (src/kv-compact-api.cpp:369-392,990-997,1201)."""
    K = np.ones((8, 4), np.float32)
    V = np.ones((8, 4), np.float32)
    Q = np.ones((2, 4), np.float32)
    r = abi.Result()
    f = oracle["kv_compact"]
    assert f(None, abi.fptr(V), abi.fptr(Q), 8, 2, 1, 4, 4, None, r) == -1
    assert f(abi.fptr(K), abi.fptr(V), abi.fptr(Q), 0, 2, 1, 4, 4, None, r) == -2
    assert f(abi.fptr(K), abi.fptr(V), abi.fptr(Q), 8, 0, 1, 4, 4, None, r) == -2
    assert f(abi.fptr(K), abi.fptr(V), abi.fptr(Q), 8, 2, 1, 4, 4, None, None) == -1
    mr = oracle["kv_compact_multi_round"]
    assert mr(abi.fptr(K), abi.fptr(V), abi.fptr(Q), 8, 2, 1, 4, 4, None, 0, r, None) == -3
    assert mr(abi.fptr(K), abi.fptr(V), None, 8, 2, 1, 4, 4, None, 1, r, None) == -1
    qf = oracle["kv_compact_quantized"]
    Kq = np.zeros((8, 34), np.uint8)
    qr = abi.QuantResult()
    assert qf(abi.u8ptr(Kq), abi.u8ptr(Kq), abi.fptr(Q), 8, 8, 34, 34, 8, 2, 1, 16, 16, None, qr) == -4
    assert qf(None, abi.u8ptr(Kq), abi.fptr(Q), 8, 8, 34, 34, 8, 2, 1, 32, 32, None, qr) == -1


def test_oracle_nnls_known_answers(oracle):
    """Known-answer NNLS cases of the reference's math tests
    (tests/test-kv-compact-math.cpp:194-231): identity system with a positive
    solution, a solution that must clamp at zero, and a mean fit."""
    lib = oracle["_lib"]
    lib.oracle_nnls_lh.restype = ctypes.c_int
    A = np.eye(2, dtype=np.float32)
    b = np.array([3, 5], np.float32)
    w = np.zeros(2, np.float32)
    lib.oracle_nnls_lh(abi.fptr(A), abi.fptr(b), abi.fptr(w), 2, 2, 100)
    np.testing.assert_allclose(w, [3, 5], atol=1e-5)
    b = np.array([3, -2], np.float32)
    lib.oracle_nnls_lh(abi.fptr(A), abi.fptr(b), abi.fptr(w), 2, 2, 100)
    assert abs(w[0] - 3) < 1e-5 and w[1] <= 1e-6
    A = np.ones((4, 1), np.float32)
    b = np.array([1, 2, 3, 4], np.float32)
    w1 = np.zeros(1, np.float32)
    lib.oracle_nnls_lh(abi.fptr(A), abi.fptr(b), abi.fptr(w1), 4, 1, 100)
    assert abs(w1[0] - 2.5) < 1e-4


def test_oracle_least_squares_known_answer(oracle):
    """A consistent 4x3 system with two right-hand sides recovers x_true
    (the reference's LS known answer, tests/test-kv-compact-math.cpp:365-609)."""
    lib = oracle["_lib"]
    A = np.array([[1, 2, 0], [0, 1, 1], [1, 0, 1], [2, 1, 1]], np.float32)
    x_true = np.array([[1, -1], [2, 0.5], [-1, 3]], np.float32)
    b = (A @ x_true).astype(np.float32)
    x = np.zeros((3, 2), np.float32)
    lib.oracle_least_squares(abi.fptr(A), abi.fptr(b), abi.fptr(x), 4, 3, 2, ctypes.c_float(1e-8))
    np.testing.assert_allclose(x, x_true, atol=1e-3)
