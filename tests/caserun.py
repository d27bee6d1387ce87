"""Replay a golden case (tests/golden/cases/*.npz) through a bound library."""
import numpy as np

from kvc_b200 import abi


def mock_classifier(T):
    """70% thinking, 5% transition, rest answer (reference test-kv-compact-api.cpp:1581-1588)."""
    think_end = (T * 70) // 100
    trans_end = think_end + (T * 5) // 100

    def f(pos):
        if pos < think_end:
            return abi.KV_TOKEN_THINKING
        if pos < trans_end:
            return abi.KV_TOKEN_TRANSITION
        return abi.KV_TOKEN_ANSWER
    return f


def run_case(fns, case):
    """Returns (rc, out) with the same keys the fixture stores."""
    meta = case["meta"]
    kind = meta["kind"]
    dk, pk, extra = meta["data"], meta["params"], meta.get("extra", {})
    params = abi.make_params(fns, **pk) if pk is not None else None
    keep = None
    if extra.get("reasoning") and params is not None:
        keep = abi.Reasoner(mock_classifier(dk["T"]), *extra["reasoning"])
        keep.attach(params)
    if kind == "compact":
        Q = case["Q"] if case["Q"].size else None
        rc, out = abi.run_compact(fns, case["K"], case["V"], Q, dk["n_q"], dk["H"], dk["d"], dk["d"], params)
    elif kind == "quantized":
        Kq, Vq = case["Kq"], case["Vq"]
        rc, out = abi.run_quantized(fns, Kq, Vq, case["Q"], dk["k_type"], dk["v_type"], Kq.shape[1],
                                    Vq.shape[1], dk["T"], dk["n_q"], dk["H"], dk["d"], dk["d"], params)
    elif kind == "multi_round":
        rc, out = abi.run_multi_round(fns, case["K"], case["V"], case["Q"], dk["n_q"], dk["H"], dk["d"],
                                      dk["d"], params, extra["n_rounds"])
    else:
        raise ValueError(kind)
    del keep
    if rc == 0:
        st = out["stats"]
        out["stats_arr"] = np.array([st["avg_cosine_sim"], st["avg_mse"], st["avg_agreement"]], np.float32)
    return rc, out
