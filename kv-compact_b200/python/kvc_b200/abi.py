"""ctypes mirror of include/kv-compact-api.h and include/kvc-batched.h.

The struct layouts are the reference's (fabiantax/kv-compact
include/kv-compact-api.h:98-241,318-326; its own ctypes mirror is
python/kv_compact/_bindings.py:28-74). The same classes bind three libraries
that export the same entry points: this repository's libkvc.so, the
reference library built from source for parity checks, and the CPU oracle
(whose symbols carry an ``oracle_`` prefix).
"""
import ctypes
from ctypes import (POINTER, Structure, c_double, c_float, c_int, c_size_t,
                    c_uint8, c_void_p)

import numpy as np

KV_TYPE_F32, KV_TYPE_F16, KV_TYPE_Q4_0, KV_TYPE_Q4_1, KV_TYPE_Q8_0 = 0, 1, 2, 3, 8
KV_TOKEN_ANSWER, KV_TOKEN_THINKING, KV_TOKEN_TRANSITION = 0, 1, 2

LAYER_FILTER_FN = ctypes.CFUNCTYPE(c_int, c_int, c_int, c_void_p)
CLASSIFIER_FN = ctypes.CFUNCTYPE(c_int, c_int, c_void_p)


class Reasoning(Structure):
    _fields_ = [
        ("classifier", CLASSIFIER_FN),
        ("classifier_data", c_void_p),
        ("thinking_weight", c_float),
        ("transition_weight", c_float),
        ("token_offset", c_int),
    ]


class Params(Structure):
    _fields_ = [
        ("target_ratio", c_float),
        ("target_count", c_int),
        ("use_sensitivity", c_int),
        ("ridge", c_float),
        ("nnls_max_iter", c_int),
        ("refine_rounds", c_int),
        ("use_diversity", c_int),
        ("diversity_strength", c_float),
        ("n_shared_prefix", c_int),
        ("use_cheap_qref", c_int),
        ("skip_beta", c_int),
        ("score_method", c_int),
        ("use_omp", c_int),
        ("omp_k_choice", c_int),
        ("omp_refit_interval", c_int),
        ("nnls_method", c_int),
        ("nnls_pgd_iters", c_int),
        ("chunk_size", c_int),
        ("n_threads", c_int),
        ("layer_filter", LAYER_FILTER_FN),
        ("layer_filter_data", c_void_p),
        ("reasoning", POINTER(Reasoning)),
    ]


class Stats(Structure):
    _fields_ = [
        ("avg_cosine_sim", c_float),
        ("avg_mse", c_float),
        ("avg_agreement", c_float),
        ("elapsed_ms", c_double),
        ("scoring_ms", c_double),
        ("nnls_ms", c_double),
    ]


class Result(Structure):
    _fields_ = [
        ("t", c_int),
        ("n_head_kv", c_int),
        ("selected_indices", POINTER(c_int)),
        ("beta", POINTER(POINTER(c_float))),
        ("C_v", POINTER(POINTER(c_float))),
        ("stats", Stats),
    ]


class QuantResult(Structure):
    _fields_ = [
        ("base", Result),
        ("k_type", c_int),
        ("v_type", c_int),
        ("K_out", POINTER(c_uint8)),
        ("V_out", POINTER(c_uint8)),
        ("k_row_bytes", c_size_t),
        ("v_row_bytes", c_size_t),
    ]


PARAM_FIELDS = [f for f, _ in Params._fields_]

_FP = POINTER(c_float)
_U8P = POINTER(c_uint8)


def bind(lib, prefix=""):
    """Declare argtypes/restype of the drop-in entry points on ``lib``.

    ``prefix`` is "" for libkvc.so and the reference, "oracle_" for the CPU
    oracle. Returns a dict name -> ctypes function (names without prefix).
    """
    names = {
        "params_default": "kv_compact_params_default" if not prefix else prefix + "params_default",
        "kv_compact": prefix + "kv_compact",
        "kv_compact_multi_round": prefix + "kv_compact_multi_round",
        "result_free": "kv_compact_result_free" if not prefix else prefix + "result_free",
        "kv_compact_quantized": prefix + "kv_compact_quantized",
        "quant_result_free": "kv_compact_quant_result_free" if not prefix else prefix + "quant_result_free",
        "dequantize_row": "kv_dequantize_row" if not prefix else prefix + "dequantize_row",
        "quantize_row": "kv_quantize_row" if not prefix else prefix + "quantize_row",
        "quant_row_elements": "kv_quant_row_elements" if not prefix else prefix + "quant_row_elements",
        "quant_row_bytes": "kv_quant_row_bytes" if not prefix else prefix + "quant_row_bytes",
    }
    f = {k: getattr(lib, v) for k, v in names.items()}
    f["params_default"].restype = Params
    f["params_default"].argtypes = []
    f["kv_compact"].restype = c_int
    f["kv_compact"].argtypes = [_FP, _FP, _FP, c_int, c_int, c_int, c_int, c_int,
                                POINTER(Params), POINTER(Result)]
    f["kv_compact_multi_round"].restype = c_int
    f["kv_compact_multi_round"].argtypes = [_FP, _FP, _FP, c_int, c_int, c_int, c_int, c_int,
                                            POINTER(Params), c_int, POINTER(Result),
                                            POINTER(Stats)]
    f["result_free"].restype = None
    f["result_free"].argtypes = [POINTER(Result)]
    f["kv_compact_quantized"].restype = c_int
    f["kv_compact_quantized"].argtypes = [_U8P, _U8P, _FP, c_int, c_int, c_size_t, c_size_t,
                                          c_int, c_int, c_int, c_int, c_int,
                                          POINTER(Params), POINTER(QuantResult)]
    f["quant_result_free"].restype = None
    f["quant_result_free"].argtypes = [POINTER(QuantResult)]
    f["dequantize_row"].restype = c_int
    f["dequantize_row"].argtypes = [_U8P, c_int, c_size_t, _FP, c_int]
    f["quantize_row"].restype = c_size_t
    f["quantize_row"].argtypes = [_FP, c_int, c_int, _U8P]
    f["quant_row_elements"].restype = c_int
    f["quant_row_elements"].argtypes = [c_int, c_size_t]
    f["quant_row_bytes"].restype = c_size_t
    f["quant_row_bytes"].argtypes = [c_int, c_int]
    return f


def fptr(a):
    """float32 numpy array (or None) -> POINTER(c_float)."""
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_FP)


def u8ptr(a):
    if a is None:
        return None
    assert a.dtype == np.uint8 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_U8P)


def make_params(fns, **kw):
    """Default params from the library, with keyword overrides."""
    p = fns["params_default"]()
    for k, v in kw.items():
        if k not in PARAM_FIELDS:
            raise KeyError(k)
        setattr(p, k, v)
    return p


def result_to_numpy(r, d_v):
    """Copy a filled Result into numpy arrays."""
    t, H = r.t, r.n_head_kv
    out = {
        "t": t,
        "indices": np.ctypeslib.as_array(r.selected_indices, (t,)).copy() if t > 0 else np.zeros(0, np.int32),
        "beta": np.stack([np.ctypeslib.as_array(r.beta[h], (t,)).copy() for h in range(H)]) if t > 0 else np.zeros((H, 0), np.float32),
        "C_v": np.stack([np.ctypeslib.as_array(r.C_v[h], (t * d_v,)).reshape(t, d_v).copy() for h in range(H)]) if t > 0 else np.zeros((H, 0, d_v), np.float32),
        "stats": {k: getattr(r.stats, k) for k, _ in Stats._fields_},
    }
    return out


class Reasoner:
    """Keeps a classifier callback and its struct alive for one call."""

    def __init__(self, fn, thinking_weight=0.3, transition_weight=0.7, token_offset=0):
        self._cb = CLASSIFIER_FN(lambda pos, _data: int(fn(pos)))
        self.struct = Reasoning(self._cb, None, thinking_weight, transition_weight, token_offset)

    def attach(self, params):
        params.reasoning = ctypes.pointer(self.struct)
        return params


def run_compact(fns, K, V, Q, n_q, H, dk, dv, params):
    T = K.shape[0]
    r = Result()
    rc = fns["kv_compact"](fptr(K), fptr(V), fptr(Q), T, n_q, H, dk, dv,
                           ctypes.byref(params) if params is not None else None, ctypes.byref(r))
    if rc != 0:
        return rc, None
    out = result_to_numpy(r, dv)
    fns["result_free"](ctypes.byref(r))
    return 0, out


def run_multi_round(fns, K, V, Q, n_q, H, dk, dv, params, n_rounds):
    T = K.shape[0]
    r = Result()
    per = (Stats * max(n_rounds, 1))()
    rc = fns["kv_compact_multi_round"](fptr(K), fptr(V), fptr(Q), T, n_q, H, dk, dv,
                                       ctypes.byref(params) if params is not None else None,
                                       n_rounds, ctypes.byref(r), per)
    if rc != 0:
        return rc, None
    out = result_to_numpy(r, dv)
    out["per_round"] = [{k: getattr(per[i], k) for k, _ in Stats._fields_} for i in range(n_rounds)]
    fns["result_free"](ctypes.byref(r))
    return 0, out


def run_quantized(fns, Kq, Vq, Q, k_type, v_type, krb, vrb, T, n_q, H, dk, dv, params):
    r = QuantResult()
    rc = fns["kv_compact_quantized"](u8ptr(Kq), u8ptr(Vq), fptr(Q), k_type, v_type, krb, vrb,
                                     T, n_q, H, dk, dv,
                                     ctypes.byref(params) if params is not None else None,
                                     ctypes.byref(r))
    if rc != 0:
        return rc, None
    out = result_to_numpy(r.base, dv)
    t = r.base.t
    out["K_out"] = np.ctypeslib.as_array(r.K_out, (t * krb,)).copy().reshape(t, krb) if t > 0 else np.zeros((0, krb), np.uint8)
    out["V_out"] = np.ctypeslib.as_array(r.V_out, (t * vrb,)).copy().reshape(t, vrb) if t > 0 else np.zeros((0, vrb), np.uint8)
    fns["quant_result_free"](ctypes.byref(r))
    return 0, out


def quantize_rows(fns, X, typ):
    """[rows x n] float32 -> [rows x row_bytes] uint8 with the library's encoder."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    rows, n = X.shape
    rb = fns["quant_row_bytes"](typ, n)
    out = np.zeros((rows, rb), np.uint8)
    for i in range(rows):
        fns["quantize_row"](fptr(X[i]), typ, n, u8ptr(out[i]))
    return out


def dequantize_rows(fns, B, typ, n):
    B = np.ascontiguousarray(B, dtype=np.uint8)
    rows, rb = B.shape
    out = np.zeros((rows, n), np.float32)
    for i in range(rows):
        fns["dequantize_row"](u8ptr(B[i]), typ, rb, fptr(out[i]), n)
    return out
