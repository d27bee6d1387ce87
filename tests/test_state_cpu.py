"""State path without a device: kvc_state_inspect's walk of the llama.cpp
state layout against the reference's own parser (parsed_kv_state::parse,
compiled from the reference headers into oracle/_ref/libstate_ref.so) on the
layouts the format allows — row and transposed V, F32/F16/Q8_0/Q4_0 rows,
M-RoPE cell extensions, empty extra streams, trailing bytes — and on
truncated buffers; and the checker's own output re-parsed."""
import ctypes
import os

import numpy as np
import pytest

import statefmt
from conftest import REPO
from kvc_b200 import state as kst

STATE_REF = os.path.join(REPO, "oracle", "_ref", "libstate_ref.so")
U8P = ctypes.POINTER(ctypes.c_uint8)


@pytest.fixture(scope="module")
def sref():
    if not os.path.exists(STATE_REF):
        pytest.skip("oracle/_ref/libstate_ref.so not built here")
    lib = ctypes.CDLL(STATE_REF, mode=ctypes.RTLD_LOCAL)
    lib.state_ref_inspect.restype = ctypes.c_int
    lib.state_ref_inspect.argtypes = [U8P, ctypes.c_size_t, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32),
                                      ctypes.POINTER(ctypes.c_size_t)]
    return statefmt.bind_ref(lib)


@pytest.fixture(scope="module")
def klib(kvc):
    return kst.bind(kvc["_lib"])


def ref_inspect(sref, buf, n_pos):
    a = np.frombuffer(buf, np.uint8)
    out = (ctypes.c_uint32 * 4)()
    tr = ctypes.c_size_t(0)
    rc = sref.state_ref_inspect(a.ctypes.data_as(U8P), a.size, n_pos, out, ctypes.byref(tr))
    return rc, tuple(out), tr.value


LAYOUTS = [
    dict(k_type=1, v_type=1),
    dict(k_type=8, v_type=8),
    dict(k_type=2, v_type=0),
    dict(k_type=0, v_type=1, v_trans=True),
    dict(k_type=1, v_type=0, v_trans=True, n_pos_per_embd=4, trailing=b"recurrent-state" * 3),
    dict(k_type=1, v_type=1, extra_empty_streams=2, trailing=b"\x01\x02\x03"),
]


@pytest.mark.parametrize("lay", LAYOUTS, ids=lambda x: "-".join(f"{k}={v}" for k, v in x.items() if k != "trailing"))
def test_inspect_matches_reference_parser(kvc, klib, sref, lay):
    n_pos = lay.get("n_pos_per_embd", 1)
    buf, _, _ = statefmt.make_state(kvc, 3, 96, 3, 2, 64, **lay)
    rc, info = kst.inspect(klib, buf, n_pos)
    rrc, (n_stream, cells, v_trans, n_layer), trailing = ref_inspect(sref, buf, n_pos)
    assert rc == 0 and rrc == 0
    assert (info.n_stream, info.cell_count, info.v_trans, info.n_layer) == (n_stream, cells, v_trans, n_layer)
    assert info.trailing_bytes == trailing == len(lay.get("trailing", b""))


def test_truncated_states_are_rejected(kvc, klib, sref):
    buf, _, _ = statefmt.make_state(kvc, 4, 40, 2, 2, 32, 8, 1)
    rng = np.random.default_rng(0)
    for cut in sorted(set(rng.integers(1, len(buf) - 1, 24).tolist()) | {3, 7, len(buf) - 1}):
        rc, _ = kst.inspect(klib, buf[:cut])
        rrc, _, _ = ref_inspect(sref, buf[:cut], 1)
        assert rrc == -20, cut
        assert rc == -20, (cut, rc)


def test_quantised_transposed_v_is_refused(kvc, klib):
    buf, _, _ = statefmt.make_state(kvc, 5, 64, 1, 2, 32, 1, 1, v_trans=True)
    b = bytearray(buf)
    secs = statefmt.sections(buf)
    # rewrite layer 0's transposed V type from F16 to Q8_0
    off = len(buf) - len(secs["rest"]) - len(secs["v"][0][1]) - 12
    b[off:off + 4] = (8).to_bytes(4, "little")
    rc, _ = kst.inspect(klib, bytes(b))
    assert rc == -21


def test_checker_output_reparses(kvc, sref):
    """The checker's compacted state is a state again: t cells, the same
    layers and trailing bytes, K rows = the kept cells' rows (no beta)."""
    trailing = b"tail" * 5
    buf, _, _ = statefmt.make_state(kvc, 6, 200, 2, 2, 32, 1, 0, trailing=trailing)
    rc, out, sel = statefmt.ref_compact(sref, buf, 2, ratio=0.25)
    assert rc == 0 and len(sel) == 50 and np.all(np.diff(sel) > 0)
    rrc, (n_stream, cells, _, n_layer), tr = ref_inspect(sref, out, 1)
    assert rrc == 0 and (n_stream, cells, n_layer, tr) == (1, 50, 2, len(trailing))
    a, b = statefmt.sections(buf), statefmt.sections(out)
    assert b["cells"] == [a["cells"][i] for i in sel]
    for l in range(2):
        rb = a["k"][l][0][1]
        rows = np.frombuffer(a["k"][l][1], np.uint8).reshape(200, rb)
        assert b["k"][l][1] == rows[sel].tobytes()
    assert b["rest"] == trailing
