"""State path on the GPU: kvc_state_compact against the checker built from
the reference's own state and math headers (oracle/_ref/libstate_ref.so,
the steps of the reference CLI's state path) on synthetic llama.cpp states.

Per case: the kept cells equal the checker's (any difference must be a near
tie of the global importance the checker ranked, below 1e-6 relative); the
headers, cell records, empty streams and trailing bytes are byte-identical;
K rows are byte-identical (without beta) or within 1e-3 of the checker's
folded rows (with beta, whose direction the checker solves in fp32); layers
left out keep V rows byte-identical; refitted F32 values are within 1e-3 of
the fp64 solution of the same ridge problem, or no farther from it than the
checker's; quantised values no farther from it than the checker's + 1e-3."""
import ctypes
import os

import numpy as np
import pytest

import parity
import statefmt
from conftest import REPO
from kvc_b200 import abi
from kvc_b200 import state as kst

pytestmark = pytest.mark.gpu

STATE_REF = os.path.join(REPO, "oracle", "_ref", "libstate_ref.so")
T, L, H, D = 2048, 4, 2, 64

CASES = {
    "f16k_f32v": (dict(k_type=1, v_type=0), dict()),
    "q8_kv": (dict(k_type=8, v_type=8), dict()),
    "f16_transposed_v": (dict(k_type=1, v_type=1, v_trans=True), dict()),
    "mrope_cells_trailing_sensitivity": (dict(k_type=0, v_type=0, n_pos_per_embd=4, extra_empty_streams=1,
                                              trailing=b"recurrent" * 11), dict(sensitivity=1)),
    "layer_filter_rms": (dict(k_type=1, v_type=0), dict(layer_mask=[1, 0, 1, 0], score_method=1)),
    "fold_beta": (dict(k_type=0, v_type=0), dict(fold_beta=1)),
}


@pytest.fixture(scope="module")
def sref():
    if not os.path.exists(STATE_REF):
        pytest.fail("oracle/_ref/libstate_ref.so missing: run `make -C oracle ref` where the reference exists")
    return statefmt.bind_ref(ctypes.CDLL(STATE_REF, mode=ctypes.RTLD_LOCAL))


def decode_v(kvc, sec, t, ev, v_trans):
    hdr, data = sec
    if v_trans:
        vt, el, ne = hdr
        vals = np.frombuffer(data, np.float32 if vt == 0 else np.float16).astype(np.float32).reshape(ne, t)
        return np.ascontiguousarray(vals.T)
    vt, vr = hdr
    return abi.dequantize_rows(kvc, np.frombuffer(data, np.uint8).reshape(t, vr), vt, ev)


@pytest.mark.parametrize("case", sorted(CASES))
def test_state_compact_matches_checker(kvc, sref, case):
    lay, ck = CASES[case]
    lib = kst.bind(kvc["_lib"])
    n_pos = lay.get("n_pos_per_embd", 1)
    buf, _, _ = statefmt.make_state(kvc, 21, T, L, H, D, **lay)
    mask = ck.get("layer_mask")
    keep = (lambda l, n, data: int(mask[l])) if mask is not None else None
    cb = abi.LAYER_FILTER_FN(keep) if keep else abi.LAYER_FILTER_FN()
    p = kst.params(lib, n_head_kv=H, n_pos_per_embd=n_pos, target_ratio=0.2, score_method=ck.get("score_method", 0),
                   use_sensitivity=ck.get("sensitivity", 0), fold_beta=ck.get("fold_beta", 0), layer_filter=cb)
    rc, out, sel, info = kst.compact(lib, buf, p)
    assert rc == 0
    rrc, rout, rsel, gimp = statefmt.ref_compact(sref, buf, H, ratio=0.2, n_pos_per_embd=n_pos,
                                                 score_method=ck.get("score_method", 0),
                                                 sensitivity=ck.get("sensitivity", 0), layer_mask=mask,
                                                 fold_beta=ck.get("fold_beta", 0), want_importance=True)
    assert rrc == 0
    t = info.t
    assert t == len(rsel) == int(np.float32(T) * np.float32(0.2))
    assert info.n_compacted == (sum(mask) if mask is not None else L)
    mism, ties, worst = parity.classify_indices(sel, rsel, gimp, [(0, T, t, 0, False)])
    print(f"\n{case}: {mism} cell mismatches ({ties} near ties) of {t}")
    assert mism == ties, f"{mism} mismatches, worst gap {worst:.3e}"
    a, o, r = statefmt.sections(buf, n_pos), statefmt.sections(out, n_pos), statefmt.sections(rout, n_pos)
    assert o["n_stream"] == r["n_stream"] and o["v_trans"] == r["v_trans"] and o["rest"] == r["rest"]
    assert o["cells"] == [a["cells"][i] for i in sel]
    same = np.array_equal(sel, rsel)
    if same:
        assert o["cells"] == r["cells"]
    ek = ev = H * D
    on = mask if mask is not None else [1] * L
    for l in range(L):
        assert o["k"][l][0] == r["k"][l][0] and o["v"][l][0] == r["v"][l][0]
        if not same:
            continue
        if ck.get("fold_beta") and on[l]:
            kt, kr = o["k"][l][0]
            ko = abi.dequantize_rows(kvc, np.frombuffer(o["k"][l][1], np.uint8).reshape(t, kr), kt, ek)
            kr_ = abi.dequantize_rows(kvc, np.frombuffer(r["k"][l][1], np.uint8).reshape(t, kr), kt, ek)
            e = parity.rel_l2(ko, kr_)
            print(f"  layer {l}: folded K rel-L2 vs checker {e:.2e}")
            assert e <= 1e-3
        else:
            assert o["k"][l][1] == r["k"][l][1], f"layer {l} K rows differ"
        if not on[l]:
            assert o["v"][l][1] == r["v"][l][1], f"layer {l} passthrough V rows differ"
            continue
        if ck.get("fold_beta"):
            vo = decode_v(kvc, o["v"][l], t, ev, o["v_trans"])
            vr = decode_v(kvc, r["v"][l], t, ev, r["v_trans"])
            e = parity.rel_l2(vo, vr)
            print(f"  layer {l}: C_v (fitted with own beta) rel-L2 vs checker {e:.2e}")
            assert e <= 5e-2
            continue
        kt, kr = a["k"][l][0]
        Kf = abi.dequantize_rows(kvc, np.frombuffer(a["k"][l][1], np.uint8).reshape(T, kr), kt, ek)
        Vf = decode_v(kvc, a["v"][l], T, ev, a["v_trans"])
        n_ref = max(16, T // 4)
        ex = parity.exact_cv(Kf, Vf, Kf[T - n_ref:], H, D, sel, np.zeros((H, t), np.float32), [(0, T, t, 0, False)],
                             dict(ridge=1e-6), False)
        ex_rows = np.concatenate([ex[h] for h in range(H)], axis=1)          # [t x H*dv]
        vo = decode_v(kvc, o["v"][l], t, ev, o["v_trans"])
        vr = decode_v(kvc, r["v"][l], t, ev, r["v_trans"])
        e_o, e_r = parity.rel_l2(vo, ex_rows), parity.rel_l2(vr, ex_rows)
        print(f"  layer {l}: values rel-L2 vs fp64 ours {e_o:.2e} checker {e_r:.2e}")
        if o["v"][l][0][0] == 0:
            assert e_o <= max(parity.CV_REL_TOL, e_r)
        else:
            assert e_o <= e_r + 1e-3
