"""Failure detection and error propagation, without faulting the GPU.

The reference propagates a failed chunk's error code after its parallel
region and frees the partial results (src/kv-compact-api.cpp:502-507). Here:

  * host-side injection (KVC_FAULT_INJECT): an allocation that fails as on an
    exhausted device returns -11, a missing device -10, through
    kv_compact_quantized, with the result left empty;
  * a bounded device wait that runs out (KVC_TC_STALL_TEST: the scoring
    kernel's first pipeline wait targets an mbarrier phase nothing completes)
    returns -12 through the same call;

and after each, with the hook removed, the next call on the same context
succeeds and equals a clean run bit for bit (nothing leaked or left in
flight). No test traps, faults or hangs the GPU: the waits are bounded and
the kernel frees its TMEM and waits for its own copies before returning."""
import numpy as np
import pytest

from kvc_b200 import abi, workloads

pytestmark = pytest.mark.gpu


def _case(kvc, typ=abi.KV_TYPE_Q8_0):
    T, H, d, nq = 6000, 4, 128, 128
    K, V, Q = workloads.small_case(77, T, nq, H, d, "rope")
    Kq, Vq = abi.quantize_rows(kvc, K, typ), abi.quantize_rows(kvc, V, typ)
    return (Kq, Vq, Q, typ, typ, Kq.shape[1], Vq.shape[1], T, nq, H, d, d)


def _run(kvc, args):
    return abi.run_quantized(kvc, *args, abi.make_params(kvc, target_ratio=0.2))


def _same(a, b):
    for k in ("indices", "beta", "C_v", "K_out", "V_out"):
        np.testing.assert_array_equal(a[k], b[k])


@pytest.mark.parametrize("what,code", [("alloc", -11), ("nodev", -10)])
def test_injected_host_failure_propagates(kvc, monkeypatch, what, code):
    args = _case(kvc)
    rc, clean = _run(kvc, args)
    assert rc == 0
    monkeypatch.setenv("KVC_FAULT_INJECT", what)
    rc, out = _run(kvc, args)
    assert rc == code and out is None
    monkeypatch.delenv("KVC_FAULT_INJECT")
    rc, again = _run(kvc, args)
    assert rc == 0
    _same(again, clean)


@pytest.mark.parametrize("fused", [True, False], ids=["score_pv_tc", "score_tc"])
def test_bounded_device_wait_runs_out(kvc, monkeypatch, fused):
    """Both tensor-core scoring kernels (fused with the refit target, and
    alone) take their error path when a wait runs out."""
    if fused:
        monkeypatch.setenv("KVC_FUSED_PV", "1")
    args = _case(kvc)
    rc, clean = _run(kvc, args)
    assert rc == 0
    monkeypatch.setenv("KVC_TC_STALL_TEST", "1")
    rc, out = _run(kvc, args)
    assert rc == -12 and out is None
    monkeypatch.delenv("KVC_TC_STALL_TEST")
    rc, again = _run(kvc, args)
    assert rc == 0
    _same(again, clean)
