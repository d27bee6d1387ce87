"""GPU parity at the metric configuration and the reference's own API suite.

cfg4 is the workload the throughput metric is quoted on: one filtered layer
holds T = 100,000 tokens x 8 KV heads x d = 128, stored Q8_0 (or Q4_0), with
a SnapKV window of 32 queries x GQA 4 (n_q = 128) and 20% retention
(79 auto chunks of 1280 keys, 20,000 kept). One full layer of each variant
goes through kv_compact_quantized on libkvc.so and on the reference library
built from its sources (oracle/_ref, all host threads), and the results are
held to the parity bar:

  * selected indices equal, except swaps of keys whose oracle importances
    differ by less than parity.NEAR_TIE_REL (counted and printed); the
    importances come from the C oracle run on the chunks that differ (a
    chunk's selection depends only on its own tokens and the queries,
    src/kv-compact-api.cpp:466-498);
  * K_out bit-exact on every row whose index matches;
  * V_out equal to the requantised C_v (V_out row j = encode(C_v[0][j] ...
    C_v[H-1][j])), the requantisation checked against the host encoder;
  * C_v within parity.CV_REL_TOL of the fp64 solve of the same ridge problem
    for the chunks whose indices match, or no farther from it than the
    reference's C_v;
  * stats.avg_cosine_sim >= parity.COS_RATIO x the reference's.

The reference's own test program (tests/test-kv-compact-api.cpp, compiled
against include/kv-compact-api.h and linked to libkvc.so by
oracle/Makefile's reftest target) must exit 0 on the GPU.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import parity
from conftest import REPO
from kvc_b200 import ORACLE_PATH, REF_PATH, abi, workloads

pytestmark = pytest.mark.gpu

REFTEST = os.path.join(REPO, "oracle", "_ref", "test-kv-compact-api-on-kvc")


@pytest.fixture(scope="module")
def reference():
    if not os.path.exists(REF_PATH):
        pytest.skip("oracle/_ref/libkv-compact.so not built here")
    return abi.bind(ctypes.CDLL(REF_PATH, mode=ctypes.RTLD_LOCAL))


@pytest.fixture(scope="module")
def oracle_traced():
    so = ctypes.CDLL(ORACLE_PATH, mode=ctypes.RTLD_LOCAL)
    fns = abi.bind(so, prefix="oracle_")
    so.oracle_trace_importance.restype = None
    so.oracle_trace_importance.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int]
    fns["_trace"] = so.oracle_trace_importance
    return fns


def _cfg4_layer(kvc, typ, seed):
    """One cfg4 layer generated on the device, quantised by the device
    encoder (bit-identical to the host encoder), returned as host arrays."""
    import torch
    from kvc_b200 import lib
    T, H, d = 100_000, 8, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    K = workloads.torch_rope_keys(T, H, d, g, "cuda")
    V = torch.randn((T, H * d), generator=g, device="cuda")
    Q = workloads.torch_snapkv_queries(H, d, g, "cuda").contiguous()
    Kq = lib.quantize_dev(kvc, K, typ).cpu().numpy()
    Vq = lib.quantize_dev(kvc, V, typ).cpu().numpy()
    Qh = Q.cpu().numpy()
    del K, V, Q
    torch.cuda.empty_cache()
    return Kq, Vq, Qh


def _chunk_importance(oracle, Kf, Vf, Q, st, C, H, d, pk):
    """Oracle importances of the keys of one chunk (computed as the chunk's
    own unchunked sub-call), indexed by chunk-local position."""
    n_q = Q.shape[0]
    imp = np.zeros(C, np.float32)
    sub = dict(pk, chunk_size=-1)
    oracle["_trace"](imp.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), C)
    rc, _ = abi.run_compact(oracle, np.ascontiguousarray(Kf[st:st + C]), np.ascontiguousarray(Vf[st:st + C]), Q,
                            n_q, H, d, d, abi.make_params(oracle, **sub))
    oracle["_trace"](None, 0)
    assert rc == 0
    return imp


@pytest.mark.parametrize("typ", [abi.KV_TYPE_Q8_0, abi.KV_TYPE_Q4_0], ids=["q8_0", "q4_0"])
def test_cfg4_full_layer_matches_reference(kvc, reference, oracle_traced, typ):
    T, H, d = 100_000, 8, 128
    Kq, Vq, Q = _cfg4_layer(kvc, typ, 4000 + typ)
    krb, vrb, nq = Kq.shape[1], Vq.shape[1], Q.shape[0]
    pk = dict(target_ratio=0.2)
    args = (Kq, Vq, Q, typ, typ, krb, vrb, T, nq, H, d, d)
    rc, ours = abi.run_quantized(kvc, *args, abi.make_params(kvc, **pk))
    assert rc == 0
    rc, theirs = abi.run_quantized(reference, *args,
                                   abi.make_params(reference, n_threads=len(os.sched_getaffinity(0)), **pk))
    assert rc == 0
    units = parity.plan_units(T, pk)
    assert len(units) == 79
    assert ours["t"] == theirs["t"] == 20000

    # indices, chunk by chunk; importances from the oracle only where they differ
    Kf = abi.dequantize_rows(kvc, Kq, typ, H * d)
    Vf = abi.dequantize_rows(kvc, Vq, typ, H * d)
    mism = ties = 0
    worst = 0.0
    equal_chunks = []
    off = 0
    for ci, (st, C, tc, pre, cheap) in enumerate(units):
        a, b = ours["indices"][off:off + tc], theirs["indices"][off:off + tc]
        if np.array_equal(a, b):
            equal_chunks.append(ci)
        else:
            imp = np.zeros(T, np.float32)
            imp[st:st + C] = _chunk_importance(oracle_traced, Kf, Vf, Q, st, C, H, d, pk)
            m, t_, w = parity.classify_indices(a, b, imp, [(st, C, tc, pre, cheap)])
            mism, ties, worst = mism + m, ties + t_, max(worst, w)
        off += tc
    print(f"\ncfg4 {abi_name(typ)} layer: {mism} index differences of {ours['t']}, {ties} near-tie swaps, "
          f"{len(equal_chunks)} of {len(units)} chunks identical")
    assert mism == ties, f"{mism} index mismatches, {ties} near-ties, worst gap {worst:.3e}"

    # K_out: the kept K rows re-encoded, bit-exact where the index matches
    same = ours["indices"] == theirs["indices"]
    np.testing.assert_array_equal(ours["K_out"][same], theirs["K_out"][same])
    # V_out: our C_v requantised (host encoder) row by row
    cv_rows = np.ascontiguousarray(ours["C_v"].transpose(1, 0, 2).reshape(ours["t"], H * d))
    np.testing.assert_array_equal(ours["V_out"], abi.quantize_rows(kvc, cv_rows, typ))

    # C_v against the fp64 ridge solve, on every chunk whose indices match
    e_ours_n = e_ref_n = e_den = 0.0
    offs = np.cumsum([0] + [u[2] for u in units])
    for ci in equal_chunks:
        st, C, tc, pre, cheap = units[ci]
        o0, o1 = offs[ci], offs[ci + 1]
        sel = ours["indices"][o0:o1] - st
        ex = parity.exact_cv(Kf[st:st + C], Vf[st:st + C], Q, H, d, sel, theirs["beta"][:, o0:o1],
                             [(0, C, tc, pre, cheap)], pk, False)
        e_ours_n += float(np.sum((ours["C_v"][:, o0:o1].astype(np.float64) - ex) ** 2))
        e_ref_n += float(np.sum((theirs["C_v"][:, o0:o1].astype(np.float64) - ex) ** 2))
        e_den += float(np.sum(ex ** 2))
    e_ours, e_ref = np.sqrt(e_ours_n / e_den), np.sqrt(e_ref_n / e_den)
    print(f"cfg4 {abi_name(typ)} layer: C_v rel-L2 vs fp64 ours {e_ours:.2e} reference {e_ref:.2e}; "
          f"cosine ours {ours['stats']['avg_cosine_sim']:.6f} reference {theirs['stats']['avg_cosine_sim']:.6f}")
    assert e_ours <= max(parity.CV_REL_TOL, e_ref)
    assert ours["stats"]["avg_cosine_sim"] >= parity.COS_RATIO * theirs["stats"]["avg_cosine_sim"] - 1e-6


def abi_name(typ):
    return {abi.KV_TYPE_Q8_0: "Q8_0", abi.KV_TYPE_Q4_0: "Q4_0", abi.KV_TYPE_F16: "F16"}.get(typ, str(typ))


def test_reference_api_suite_on_libkvc():
    """The reference's own tests/test-kv-compact-api.cpp, linked unchanged
    against libkvc.so, passes on the GPU."""
    if not os.path.exists(REFTEST):
        pytest.skip("oracle/_ref/test-kv-compact-api-on-kvc not built here")
    p = subprocess.run([REFTEST], capture_output=True, text=True, timeout=1200)
    tail = "\n".join(p.stdout.splitlines()[-15:])
    print(f"\n{tail}")
    assert p.returncode == 0, f"rc {p.returncode}\n{tail}\n{p.stderr[-2000:]}"
    assert "All tests passed!" in p.stdout


@pytest.mark.parametrize("typ,fused", [(abi.KV_TYPE_Q8_0, False), (abi.KV_TYPE_Q4_0, False), (abi.KV_TYPE_F16, False),
                                       (abi.KV_TYPE_Q8_0, True), (abi.KV_TYPE_Q4_0, True)],
                         ids=["q8_0", "q4_0", "f16", "q8_0_fused", "q4_0_fused"])
def test_tensor_core_scores_match_exact_mode(kvc, reference, oracle_traced, monkeypatch, typ, fused):
    """Scores from K's block bytes on the tensor cores (the default) against
    the bit-exact SIMT scoring (KVC_EXACT_SCORES=1): the exact mode still
    selects the reference's keys bit for bit, and the tensor-core mode selects
    them too, except near-ties (< parity.NEAR_TIE_REL relative importance gap).
    `fused`: the opt-in kernel that also forms the refit target Y = A V in the
    scoring pass (KVC_FUSED_PV=1)."""
    if fused:
        monkeypatch.setenv("KVC_FUSED_PV", "1")
    T, H, d, nq = 12_800, 8, 128, 128
    K, V, Q = workloads.small_case(300 + typ, T, nq, H, d, "rope")
    Kq, Vq = abi.quantize_rows(kvc, K, typ), abi.quantize_rows(kvc, V, typ)
    pk = dict(target_ratio=0.2)
    args = (Kq, Vq, Q, typ, typ, Kq.shape[1], Vq.shape[1], T, nq, H, d, d)
    rc, theirs = abi.run_quantized(reference, *args, abi.make_params(reference, **pk))
    assert rc == 0
    rc, tc = abi.run_quantized(kvc, *args, abi.make_params(kvc, **pk))
    assert rc == 0
    monkeypatch.setenv("KVC_EXACT_SCORES", "1")
    rc, exact = abi.run_quantized(kvc, *args, abi.make_params(kvc, **pk))
    assert rc == 0
    monkeypatch.delenv("KVC_EXACT_SCORES")
    if fused:                                   # the refit targets of the two paths agree (C_v through them)
        assert parity.rel_l2(tc["C_v"], exact["C_v"]) < 1e-4
    np.testing.assert_array_equal(exact["indices"], theirs["indices"])
    np.testing.assert_array_equal(exact["K_out"], theirs["K_out"])
    units = parity.plan_units(T, pk)
    Kf = abi.dequantize_rows(kvc, Kq, typ, H * d)
    Vf = abi.dequantize_rows(kvc, Vq, typ, H * d)
    imp = np.zeros(T, np.float32)
    oracle_traced["_trace"](imp.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), T)
    rc, _ = abi.run_compact(oracle_traced, Kf, Vf, Q, nq, H, d, d, abi.make_params(oracle_traced, **pk))
    oracle_traced["_trace"](None, 0)
    assert rc == 0
    mism, ties, worst = parity.classify_indices(tc["indices"], theirs["indices"], imp, units)
    print(f"\n{abi_name(typ)}: tensor-core scoring {mism} index differences ({ties} near-ties) of {tc['t']}; "
          f"C_v tensor-core vs exact mode rel-L2 {parity.rel_l2(tc['C_v'], exact['C_v']):.2e}")
    assert mism == ties, f"{mism} index mismatches, {ties} near-ties, worst gap {worst:.3e}"
    assert tc["stats"]["avg_cosine_sim"] >= parity.COS_RATIO * theirs["stats"]["avg_cosine_sim"] - 1e-6
