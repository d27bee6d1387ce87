"""Loader and wrappers for libkvc.so.

There is no CPU fallback: if the CUDA library is missing the loader raises,
and every compaction entry point returns -10 when no sm_100 device exists.
"""
import ctypes
import os
from ctypes import POINTER, Structure, c_float, c_int, c_size_t, c_uint64, c_void_p

from . import LIB_PATH, abi

# names the library exports (include/*.h); tests check every one resolves
DROPIN_SYMBOLS = [
    "kv_compact_params_default", "kv_compact", "kv_compact_multi_round", "kv_compact_result_free",
    "kv_compact_quantized", "kv_compact_quant_result_free", "kv_dequantize_row", "kv_quantize_row",
    "kv_quant_row_elements", "kv_quant_row_bytes",
]
SEAM_SYMBOLS = [
    "kv_compact_cuda_available", "kv_compact_cuda_mat_mul_ABt_scaled", "kv_compact_cuda_score_all_heads",
    "kv_compact_cuda_refit_target_all_heads", "kv_compact_cuda_pool_free",
    "kv_compact_cuda_score_all_heads_noalloc",
]
BATCHED_SYMBOLS = ["kvc_plan_layers", "kvc_compact_layers_dev", "kvc_launch_count", "kvc_profile",
                   "kvc_quantize_rows_dev", "kvc_dequantize_rows_dev"]
PEER_SYMBOLS = ["kvc_peer_alloc", "kvc_peer_free", "kvc_peer_open", "kvc_peer_close", "kvc_copy_async",
                "kvc_copy2d_async", "kvc_place_slice"]
STAGES = ["decode", "score", "softmax_importance", "select", "refit_target", "beta", "x_build", "ls_gram",
          "refine", "metrics", "requant", "ls_factor", "ls_out"]


class ModelDesc(Structure):
    _fields_ = [("n_layers", c_int), ("T", c_int), ("n_head_kv", c_int), ("d_k", c_int), ("d_v", c_int),
                ("k_type", c_int), ("v_type", c_int), ("k_row_bytes", c_size_t), ("v_row_bytes", c_size_t)]


class LayerDesc(Structure):
    _fields_ = [("K", c_void_p), ("V", c_void_p), ("Q_ref", c_void_p), ("n_q", c_int), ("n_tokens", c_int)]


class LayerResult(Structure):
    _fields_ = [("t", c_int), ("selected_indices", c_void_p), ("beta", c_void_p), ("C_v", c_void_p),
                ("K_out", c_void_p), ("V_out", c_void_p), ("stats", abi.Stats)]


_LIB = None


def load(path=None):
    """Load libkvc.so once and declare every entry point's signature."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    path = path or os.environ.get("KVC_LIB", LIB_PATH)
    if not os.path.exists(path):
        raise OSError(f"libkvc.so not found at {path}: build it with `make -C kv-compact_b200`")
    lib = ctypes.CDLL(path, mode=ctypes.RTLD_LOCAL)
    fns = abi.bind(lib)
    FP = POINTER(c_float)
    lib.kv_compact_cuda_available.restype = c_int
    lib.kv_compact_cuda_available.argtypes = []
    lib.kv_compact_cuda_mat_mul_ABt_scaled.restype = c_int
    lib.kv_compact_cuda_mat_mul_ABt_scaled.argtypes = [FP, FP, FP, c_int, c_int, c_int, c_float]
    lib.kv_compact_cuda_score_all_heads.restype = c_int
    lib.kv_compact_cuda_score_all_heads.argtypes = [FP, FP, POINTER(FP), c_int, c_int, c_int, c_int, c_float]
    lib.kv_compact_cuda_refit_target_all_heads.restype = c_int
    lib.kv_compact_cuda_refit_target_all_heads.argtypes = [POINTER(FP), FP, POINTER(FP), c_int, c_int, c_int, c_int]
    lib.kv_compact_cuda_score_all_heads_noalloc.restype = c_int
    lib.kv_compact_cuda_score_all_heads_noalloc.argtypes = [FP, FP, POINTER(FP), c_int, c_int, c_int, c_int,
                                                            c_float]
    lib.kv_compact_cuda_pool_free.restype = None
    lib.kv_compact_cuda_pool_free.argtypes = []
    lib.kvc_plan_layers.restype = c_int
    lib.kvc_plan_layers.argtypes = [POINTER(ModelDesc), POINTER(LayerDesc), POINTER(abi.Params), POINTER(c_int)]
    lib.kvc_compact_layers_dev.restype = c_int
    lib.kvc_compact_layers_dev.argtypes = [POINTER(ModelDesc), POINTER(LayerDesc), POINTER(abi.Params),
                                           POINTER(LayerResult), c_int]
    lib.kvc_launch_count.restype = c_uint64
    lib.kvc_launch_count.argtypes = []
    lib.kvc_quantize_rows_dev.restype = c_int
    lib.kvc_quantize_rows_dev.argtypes = [c_void_p, c_size_t, c_int, c_int, c_int, c_void_p, c_size_t]
    lib.kvc_dequantize_rows_dev.restype = c_int
    lib.kvc_dequantize_rows_dev.argtypes = [c_void_p, c_size_t, c_int, c_int, c_int, c_void_p]
    lib.kvc_profile.restype = c_int
    lib.kvc_profile.argtypes = [c_int, POINTER(ctypes.c_double), POINTER(c_uint64), c_int]
    lib.kvc_peer_alloc.restype = c_int
    lib.kvc_peer_alloc.argtypes = [c_size_t, POINTER(c_void_p), c_void_p]
    lib.kvc_peer_free.restype = c_int
    lib.kvc_peer_free.argtypes = [c_void_p]
    lib.kvc_peer_open.restype = c_int
    lib.kvc_peer_open.argtypes = [c_void_p, POINTER(c_void_p)]
    lib.kvc_peer_close.restype = c_int
    lib.kvc_peer_close.argtypes = [c_void_p]
    lib.kvc_copy_async.restype = c_int
    lib.kvc_copy_async.argtypes = [c_void_p, c_void_p, c_size_t, c_void_p]
    lib.kvc_copy2d_async.restype = c_int
    lib.kvc_copy2d_async.argtypes = [c_void_p, c_size_t, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p]
    lib.kvc_place_slice.restype = c_int
    lib.kvc_place_slice.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p]
    fns["_lib"] = lib
    fns["_path"] = path
    if path == LIB_PATH or _LIB is None:
        _LIB = fns
    return fns


def quantize_dev(fns, x, typ):
    """float32 CUDA tensor [rows, n] -> uint8 CUDA tensor [rows, row_bytes]."""
    import torch
    rows, n = x.shape
    rb = fns["quant_row_bytes"](typ, n)
    out = torch.empty((rows, rb), dtype=torch.uint8, device=x.device)
    rc = fns["_lib"].kvc_quantize_rows_dev(x.data_ptr(), x.stride(0), typ, rows, n, out.data_ptr(), rb)
    if rc != 0:
        raise RuntimeError(f"kvc_quantize_rows_dev failed: {rc}")
    return out


def dequantize_dev(fns, b, typ, n):
    import torch
    rows, rb = b.shape
    out = torch.empty((rows, n), dtype=torch.float32, device=b.device)
    rc = fns["_lib"].kvc_dequantize_rows_dev(b.data_ptr(), rb, typ, rows, n, out.data_ptr())
    if rc != 0:
        raise RuntimeError(f"kvc_dequantize_rows_dev failed: {rc}")
    return out


def profile(fns, enable):
    """Read and reset per-stage device times; enable/disable event timing."""
    n = len(STAGES)
    ms = (ctypes.c_double * n)()
    cnt = (c_uint64 * n)()
    rc = fns["_lib"].kvc_profile(1 if enable else 0, ms, cnt, n)
    if rc < 0:
        raise RuntimeError(f"kvc_profile failed: {rc}")
    return {STAGES[i]: (ms[i], int(cnt[i])) for i in range(n)}


class BatchedModel:
    """Whole-model device-resident compaction over torch tensors.

    K[l], V[l]: uint8 (or float32) CUDA tensors [T_l, row_bytes]; Q[l]: float32
    CUDA tensors [n_q, H*d_k] or None. tokens: per-layer T_l (default: T for
    every layer). Output buffers are allocated once from kvc_plan_layers()
    and reused by every run(); out_ptrs[l] = (K_out, V_out) device pointers
    makes layer l's requantised rows go there instead (self.kout[l] and
    self.vout[l] are then None).
    """

    def __init__(self, fns, K, V, Q, T, H, dk, dv, k_type, v_type, params, requant=True, tokens=None,
                 out_ptrs=None):
        import torch
        self.fns, self.lib = fns, fns["_lib"]
        self.params = params
        n = len(K)
        self.md = ModelDesc(n, T, H, dk, dv, k_type, v_type, K[0].shape[1] * K[0].element_size(),
                            V[0].shape[1] * V[0].element_size())
        self.layers = (LayerDesc * n)()
        self._keep = (K, V, Q)
        for l in range(n):
            q = Q[l] if Q is not None else None
            self.layers[l] = LayerDesc(K[l].data_ptr(), V[l].data_ptr(), q.data_ptr() if q is not None else None,
                                       q.shape[0] if q is not None else 0, 0 if tokens is None else tokens[l])
        ts = (c_int * n)()
        rc = self.lib.kvc_plan_layers(ctypes.byref(self.md), self.layers, ctypes.byref(params), ts)
        if rc != 0:
            raise RuntimeError(f"kvc_plan_layers failed: {rc}")
        self.t = list(ts)
        dev = K[0].device
        self.sel, self.beta, self.cv, self.kout, self.vout = [], [], [], [], []
        self.results = (LayerResult * n)()
        for l in range(n):
            t = max(self.t[l], 1)
            self.sel.append(torch.empty(t, dtype=torch.int32, device=dev))
            self.beta.append(torch.empty(H * t, dtype=torch.float32, device=dev))
            self.cv.append(torch.empty(H * t * dv, dtype=torch.float32, device=dev))
            ext = out_ptrs is not None and out_ptrs[l] is not None
            own = requant and not ext
            self.kout.append(torch.empty(t * self.md.k_row_bytes, dtype=torch.uint8, device=dev) if own else None)
            self.vout.append(torch.empty(t * self.md.v_row_bytes, dtype=torch.uint8, device=dev) if own else None)
            kp = out_ptrs[l][0] if ext else (self.kout[l].data_ptr() if own else None)
            vp = out_ptrs[l][1] if ext else (self.vout[l].data_ptr() if own else None)
            self.results[l] = LayerResult(0, self.sel[l].data_ptr(), self.beta[l].data_ptr(), self.cv[l].data_ptr(),
                                          kp, vp, abi.Stats())

    def run(self, want_stats=True):
        rc = self.lib.kvc_compact_layers_dev(ctypes.byref(self.md), self.layers, ctypes.byref(self.params),
                                             self.results, 1 if want_stats else 0)
        if rc != 0:
            raise RuntimeError(f"kvc_compact_layers_dev failed: {rc}")
        return rc

    def stats(self, l):
        s = self.results[l].stats
        return {k: getattr(s, k) for k, _ in abi.Stats._fields_}
