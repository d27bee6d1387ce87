"""Synthetic llama.cpp sequence-state buffers for the state-path tests.

Layout (llama_state_seq_get_data, as the reference parses and writes it,
include/kv-compact-state.h:1-15,104-222,645-810):
  [n_stream:u32] per stream: [cell_count:u32] per cell [pos:i32][n_seq_id:u32]
  ([x:i32][y:i32] when n_pos_per_embd > 1)[seq_id:i32 * n_seq_id]
  [v_trans:u32][n_layer:u32] per layer [k_type:i32][k_size_row:u64][rows]
  per layer [v_type:i32][v_size_row:u64][rows]   (non-transposed)
            [v_type:i32][v_size_el:u32][n_embd_v:u32][n_embd_v x cells] (transposed)
  [trailing bytes]
"""
import struct

import numpy as np

from kvc_b200 import abi, workloads


def encode(fns, X, typ):
    """[rows x n] fp32 -> [rows x row_bytes] in type `typ` with the library's host codec."""
    if typ == 0:
        return np.ascontiguousarray(X, np.float32).view(np.uint8).reshape(X.shape[0], -1)
    return abi.quantize_rows(fns, X, typ)


def make_state(fns, seed, T, n_layer, H, d, k_type, v_type, v_trans=False, n_pos_per_embd=1, trailing=b"",
               extra_empty_streams=0):
    """Returns (state bytes, K fp32 per layer, V fp32 per layer) with RoPE'd
    low-rank keys and N(0,1) values (the cfg2 distributions)."""
    rng = np.random.default_rng(seed)
    out = [struct.pack("<I", 1 + extra_empty_streams), struct.pack("<I", T)]
    for i in range(T):
        seqs = [0] if i % 5 else [0, 1]
        rec = struct.pack("<iI", i, len(seqs))
        if n_pos_per_embd > 1:
            rec += struct.pack("<ii", i % 7, i // 7)
        rec += struct.pack("<%di" % len(seqs), *seqs)
        out.append(rec)
    out.append(struct.pack("<II", 1 if v_trans else 0, n_layer))
    Ks, Vs = [], []
    for _ in range(n_layer):
        K = workloads.rope_keys(rng, T, H, d).astype(np.float32)
        Ks.append(K)
        kb = encode(fns, K, k_type)
        out.append(struct.pack("<iQ", k_type, kb.shape[1]))
        out.append(kb.tobytes())
    for _ in range(n_layer):
        V = rng.standard_normal((T, H * d)).astype(np.float32)
        Vs.append(V)
        if not v_trans:
            vb = encode(fns, V, v_type)
            out.append(struct.pack("<iQ", v_type, vb.shape[1]))
            out.append(vb.tobytes())
        else:
            el = 4 if v_type == 0 else 2
            vb = encode(fns, np.ascontiguousarray(V.T), v_type)          # n_embd rows of T values
            out.append(struct.pack("<iII", v_type, el, H * d))
            out.append(vb.tobytes())
    for _ in range(extra_empty_streams):
        out.append(struct.pack("<I", 0))
    out.append(trailing)
    return b"".join(out), Ks, Vs


def sections(buf, n_pos_per_embd=1):
    """Split a state into its pieces: n_stream, cell records (bytes each),
    v_trans, and per layer (k header, K bytes) and (v header, V bytes), the
    bytes after stream 0 (empty streams and trailing data)."""
    pos = 0

    def take(n):
        nonlocal pos
        b = buf[pos:pos + n]
        assert len(b) == n, "truncated state"
        pos += n
        return b
    n_stream = struct.unpack("<I", take(4))[0]
    cc = struct.unpack("<I", take(4))[0]
    cells = []
    for _ in range(cc):
        start = pos
        _, n_seq = struct.unpack("<iI", take(8))
        if n_pos_per_embd > 1:
            take(8)
        take(4 * n_seq)
        cells.append(buf[start:pos])
    v_trans, n_layer = struct.unpack("<II", take(8))
    ks, vs = [], []
    for _ in range(n_layer):
        kt, kr = struct.unpack("<iQ", take(12))
        ks.append(((kt, kr), take(cc * kr)))
    for _ in range(n_layer):
        if not v_trans:
            vt, vr = struct.unpack("<iQ", take(12))
            vs.append(((vt, vr), take(cc * vr)))
        else:
            vt, el, ne = struct.unpack("<iII", take(12))
            vs.append(((vt, el, ne), take(ne * cc * el)))
    return dict(n_stream=n_stream, cells=cells, v_trans=v_trans, k=ks, v=vs, rest=buf[pos:])


def bind_ref(lib):
    """Signatures of the checker oracle/_ref/libstate_ref.so (oracle/state_ref.cpp)."""
    import ctypes
    U8P = ctypes.POINTER(ctypes.c_uint8)
    lib.state_ref_compact.restype = ctypes.c_int
    lib.state_ref_compact.argtypes = [U8P, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32, ctypes.c_float, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                      ctypes.c_float, ctypes.POINTER(U8P), ctypes.POINTER(ctypes.c_size_t),
                                      ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                      ctypes.POINTER(ctypes.c_float)]
    lib.state_ref_free.restype = None
    lib.state_ref_free.argtypes = [ctypes.c_void_p]
    return lib


def ref_compact(lib, buf, n_head_kv, ratio=0.2, n_pos_per_embd=1, n_ref=0, score_method=0, sensitivity=0,
                layer_mask=None, fold_beta=0, ridge=1e-6, want_importance=False):
    """The checker's compacted state and kept cells: (rc, bytes, indices), plus
    the global importance it ranked when want_importance."""
    import ctypes
    U8P = ctypes.POINTER(ctypes.c_uint8)
    a = np.frombuffer(buf, np.uint8)
    out = U8P()
    n = ctypes.c_size_t(0)
    T = struct.unpack_from("<I", buf, 4)[0]
    sel = np.zeros(max(1, T), np.int32)
    gimp = np.zeros(max(1, T), np.float32)
    t = ctypes.c_int(0)
    mask = None
    if layer_mask is not None:
        mask = (ctypes.c_int * len(layer_mask))(*[int(x) for x in layer_mask])
    rc = lib.state_ref_compact(a.ctypes.data_as(U8P), a.size, n_head_kv, n_pos_per_embd, ratio, n_ref, score_method,
                               sensitivity, mask, fold_beta, ridge, ctypes.byref(out), ctypes.byref(n),
                               sel.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), ctypes.byref(t),
                               gimp.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    if rc != 0:
        return (rc, None, None, None) if want_importance else (rc, None, None)
    data = bytes(np.ctypeslib.as_array(out, (n.value,)))
    lib.state_ref_free(ctypes.cast(out, ctypes.c_void_p))
    if want_importance:
        return rc, data, sel[:t.value].copy(), gimp[:T]
    return rc, data, sel[:t.value].copy()
