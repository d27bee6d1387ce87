"""ctypes bindings of include/kvc-state.h: compaction of a saved llama.cpp
sequence state (llama_state_seq_get_data) in one call, plus a layout
inspection that needs no device."""
import ctypes
from ctypes import POINTER, Structure, c_float, c_int, c_size_t, c_uint8, c_uint32, c_void_p

import numpy as np

from . import abi



class StateParams(Structure):
    _fields_ = [("n_head_kv", c_int), ("n_pos_per_embd", c_uint32), ("target_ratio", c_float),
                ("n_ref_queries", c_int), ("score_method", c_int), ("use_sensitivity", c_int),
                ("fold_beta", c_int), ("ridge", c_float), ("layer_filter", abi.LAYER_FILTER_FN),
                ("layer_filter_data", c_void_p)]


class StateInfo(Structure):
    _fields_ = [("n_stream", c_uint32), ("cell_count", c_uint32), ("v_trans", c_uint32), ("n_layer", c_uint32),
                ("n_compacted", c_int), ("t", c_int), ("n_ref_queries", c_int), ("trailing_bytes", c_size_t)]


def bind(lib):
    lib.kvc_state_params_default.restype = StateParams
    lib.kvc_state_params_default.argtypes = []
    lib.kvc_state_inspect.restype = c_int
    lib.kvc_state_inspect.argtypes = [POINTER(c_uint8), c_size_t, c_uint32, POINTER(StateInfo)]
    lib.kvc_state_compact.restype = c_int
    lib.kvc_state_compact.argtypes = [POINTER(c_uint8), c_size_t, POINTER(StateParams),
                                      POINTER(POINTER(c_uint8)), POINTER(c_size_t), POINTER(POINTER(c_int)),
                                      POINTER(StateInfo)]
    lib.kvc_state_free.restype = None
    lib.kvc_state_free.argtypes = [c_void_p]
    return lib


def params(lib, **kw):
    p = lib.kvc_state_params_default()
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def inspect(lib, buf, n_pos_per_embd=1):
    buf = np.ascontiguousarray(np.frombuffer(buf, np.uint8) if isinstance(buf, (bytes, bytearray)) else buf, np.uint8)
    info = StateInfo()
    rc = lib.kvc_state_inspect(buf.ctypes.data_as(POINTER(c_uint8)), buf.size, n_pos_per_embd, ctypes.byref(info))
    return rc, info


def compact(lib, buf, p):
    """Returns (rc, compacted state bytes, kept cell indices, StateInfo)."""
    buf = np.ascontiguousarray(np.frombuffer(buf, np.uint8) if isinstance(buf, (bytes, bytearray)) else buf, np.uint8)
    out = POINTER(c_uint8)()
    sel = POINTER(c_int)()
    n = c_size_t(0)
    info = StateInfo()
    rc = lib.kvc_state_compact(buf.ctypes.data_as(POINTER(c_uint8)), buf.size, ctypes.byref(p), ctypes.byref(out),
                               ctypes.byref(n), ctypes.byref(sel), ctypes.byref(info))
    if rc != 0:
        return rc, None, None, info
    data = bytes(np.ctypeslib.as_array(out, (n.value,))) if n.value else b""
    idx = np.ctypeslib.as_array(sel, (info.t,)).copy() if info.t else np.zeros(0, np.int32)
    lib.kvc_state_free(ctypes.cast(out, c_void_p))
    lib.kvc_state_free(ctypes.cast(sel, c_void_p))
    return rc, data, idx, info
