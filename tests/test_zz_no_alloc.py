"""The scoring entry point that allocates no device memory.

Callers such as serving engines that hand all of HBM to their own allocator
cannot let a library call cudaMalloc; kv_compact_cuda_score_all_heads_noalloc
serves them from a fixed array compiled into libkvc.so. Its scores must equal
those of kv_compact_cuda_score_all_heads bit for bit (the scoring tolerance of
the other tests), on consecutive calls that reuse the shared array, and sizes
beyond the array must be refused. Collected last so a failure here does not
hide the rest of the suite; it also passes when run alone.
"""
import ctypes

import numpy as np
import pytest

from kvc_b200 import abi

pytestmark = pytest.mark.gpu

FP = ctypes.POINTER(ctypes.c_float)


def _scores(fn, Q, K, nq, T, H, d, scale):
    outs = [np.full(nq * T, np.nan, np.float32) for _ in range(H)]
    arr = (FP * H)(*[o.ctypes.data_as(FP) for o in outs])
    rc = fn(abi.fptr(Q), abi.fptr(K), arr, nq, T, H, d, ctypes.c_float(scale))
    return rc, [o.reshape(nq, T) for o in outs]


def test_noalloc_scores_match_allocating_entry_point_twice(kvc):
    lib = kvc["_lib"]
    rng = np.random.default_rng(2024)
    # calls in a row on different shapes; n_q > 64 takes the scoring kernel's
    # 128-query tile, n_q <= 64 its 64-query tile
    shapes = [(64, 1000, 4, 128), (37, 777, 3, 48), (128, 1000, 4, 128)]
    for nq, T, H, d in shapes:
        Q = rng.standard_normal((nq, H * d)).astype(np.float32)
        K = rng.standard_normal((T, H * d)).astype(np.float32)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
        rc_a, ref = _scores(lib.kv_compact_cuda_score_all_heads, Q, K, nq, T, H, d, scale)
        rc_b, got = _scores(lib.kv_compact_cuda_score_all_heads_noalloc, Q, K, nq, T, H, d, scale)
        assert rc_a == 0 and rc_b == 0
        for h in range(H):
            np.testing.assert_array_equal(got[h], ref[h])


def test_noalloc_rejects_sizes_beyond_its_array(kvc):
    lib = kvc["_lib"]
    nq, T, H, d = 128, 8192, 8, 128          # needs far more than 4,194,304 floats
    Q = np.zeros((nq, H * d), np.float32)
    K = np.zeros((T, H * d), np.float32)
    rc, outs = _scores(lib.kv_compact_cuda_score_all_heads_noalloc, Q, K, nq, T, H, d, 1.0)
    assert rc == -13
    assert all(np.isnan(o).all() for o in outs)
