"""Generate golden fixtures by running the reference library itself.

Loads oracle/_ref/libkv-compact.so — fabiantax/kv-compact's
src/kv-compact-api.cpp compiled from its own source by oracle/Makefile
(target ``ref``) — and records, for seeded inputs, every output the drop-in
API returns. The fixtures pin:
  * the C restatement in oracle/ (bit-exact; tests/test_oracle_golden.py), and
  * libkvc.so on a GPU (parity; tests/test_parity_gpu.py).

Run from the repository root, in a container where the reference sources
exist:  make -C oracle ref && python tests/golden/make_golden.py
Each case is one compressed .npz in tests/golden/cases/ holding its inputs,
its parameters (JSON) and the reference's outputs.
"""
import ctypes
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, os.path.join(REPO, "kv-compact_b200", "python"))

from kvc_b200 import REF_PATH, abi, workloads  # noqa: E402

OUT = os.path.join(HERE, "cases")


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


def compact_cases():
    """(name, data kwargs, params kwargs, extras)."""
    C = []
    # basic shapes and the three aggregation methods
    for sm in (0, 1, 2):
        C.append((f"basic_sm{sm}", dict(seed=1, T=64, n_q=32, H=4, d=32, kind="gauss"),
                  dict(target_ratio=0.5, score_method=sm), {}))
    C.append(("target_count", dict(seed=2, T=64, n_q=16, H=2, d=16, kind="gauss"),
              dict(target_count=10), {}))
    C.append(("no_compression", dict(seed=3, T=32, n_q=8, H=2, d=16, kind="gauss"),
              dict(target_ratio=1.0), {}))
    C.append(("null_params", dict(seed=4, T=48, n_q=8, H=2, d=16, kind="gauss"), None, {}))
    # chunking: explicit uneven chunks (200+200+100), auto chunks, prefix
    C.append(("chunk_uneven", dict(seed=5, T=500, n_q=16, H=2, d=16, kind="gauss"),
              dict(target_ratio=0.5, chunk_size=200), {}))
    C.append(("chunk_auto_rope", dict(seed=6, T=1400, n_q=128, H=1, d=128, kind="rope"),
              dict(target_ratio=0.2), {}))
    C.append(("chunk_auto_tail", dict(seed=7, T=2900, n_q=32, H=1, d=32, kind="rope"),
              dict(target_ratio=0.2), {}))
    C.append(("prefix", dict(seed=8, T=256, n_q=16, H=2, d=32, kind="gauss"),
              dict(target_ratio=0.25, n_shared_prefix=16), {}))
    C.append(("prefix_chunked", dict(seed=9, T=1500, n_q=16, H=1, d=32, kind="rope"),
              dict(target_ratio=0.2, n_shared_prefix=300), {}))
    C.append(("prefix_gt_t", dict(seed=10, T=128, n_q=8, H=1, d=16, kind="gauss"),
              dict(target_ratio=0.1, n_shared_prefix=40), {}))
    # cheap reference queries (K-as-Q), unchunked and chunked, Q pointer NULL
    C.append(("cheapq_lowrank", dict(seed=11, T=512, n_q=0, H=1, d=128, kind="lowrank"),
              dict(target_ratio=0.5, use_cheap_qref=1, chunk_size=-1), {"q_null": True}))
    C.append(("cheapq_chunked", dict(seed=12, T=1200, n_q=0, H=1, d=32, kind="gauss"),
              dict(target_ratio=0.5, use_cheap_qref=1, chunk_size=300), {"q_null": True}))
    C.append(("qnull_no_flag", dict(seed=13, T=200, n_q=0, H=2, d=16, kind="gauss"),
              dict(target_ratio=0.5), {"q_null": True}))
    # diversity, beta (LH, PGD), refinement, sensitivity, OMP, reasoning
    C.append(("diversity", dict(seed=14, T=256, n_q=16, H=2, d=32, kind="rope"),
              dict(target_ratio=0.25, use_diversity=1, diversity_strength=0.5), {}))
    C.append(("diversity_prefix", dict(seed=15, T=256, n_q=16, H=2, d=32, kind="rope"),
              dict(target_ratio=0.25, use_diversity=1, diversity_strength=0.1, n_shared_prefix=8), {}))
    C.append(("beta_lh", dict(seed=16, T=128, n_q=32, H=2, d=32, kind="gauss"),
              dict(target_ratio=0.25, skip_beta=0, nnls_method=0), {}))
    C.append(("beta_pgd", dict(seed=17, T=128, n_q=32, H=2, d=32, kind="gauss"),
              dict(target_ratio=0.25, skip_beta=0, nnls_method=1), {}))
    C.append(("beta_pgd_iters", dict(seed=18, T=128, n_q=48, H=2, d=32, kind="gauss"),
              dict(target_ratio=0.25, skip_beta=0, nnls_method=1, nnls_pgd_iters=10), {}))
    C.append(("refine_nobeta", dict(seed=19, T=160, n_q=16, H=2, d=32, kind="rope"),
              dict(target_ratio=0.25, refine_rounds=2), {}))
    C.append(("refine_lh", dict(seed=20, T=160, n_q=32, H=2, d=32, kind="gauss"),
              dict(target_ratio=0.2, refine_rounds=2, skip_beta=0, nnls_method=0), {}))
    C.append(("cfg5_small", dict(seed=21, T=640, n_q=64, H=2, d=64, kind="lowrank"),
              dict(target_ratio=0.1, skip_beta=0, nnls_method=0, use_diversity=1,
                   diversity_strength=0.1, refine_rounds=2), {}))
    C.append(("sensitivity", dict(seed=22, T=200, n_q=16, H=3, d=16, kind="gauss"),
              dict(target_ratio=0.3, use_sensitivity=1), {}))
    C.append(("omp", dict(seed=23, T=96, n_q=16, H=2, d=16, kind="gauss"),
              dict(target_ratio=0.25, use_omp=1), {}))
    C.append(("omp_fast_beta", dict(seed=24, T=96, n_q=16, H=2, d=16, kind="gauss"),
              dict(target_ratio=0.25, use_omp=1, omp_k_choice=4, omp_refit_interval=2,
                   skip_beta=0), {}))
    C.append(("reasoning", dict(seed=25, T=300, n_q=16, H=2, d=16, kind="rope"),
              dict(target_ratio=0.3), {"reasoning": (0.3, 0.7)}))
    C.append(("reasoning_chunked", dict(seed=26, T=900, n_q=16, H=2, d=16, kind="rope"),
              dict(target_ratio=0.3, chunk_size=256), {"reasoning": (0.0, 0.5)}))
    C.append(("ridge_zero", dict(seed=27, T=64, n_q=64, H=1, d=16, kind="gauss"),
              dict(target_ratio=0.5, ridge=0.0), {}))
    return C


def spiky(T, n_q, H, d, seed):
    """The reference's clustered-keys-with-sinks generator
    (tests/test-kv-compact-api.cpp:1360-1418), restated in numpy float32."""
    f32 = np.float32
    V = workloads.sincos_data(T * H * d, seed + 500).reshape(T, H * d)
    dd = np.arange(d)
    base = np.sin((dd * 7 + seed).astype(f32) * f32(0.31)).astype(f32)
    K = np.empty((T, H, d), f32)
    for t in range(T):
        for h in range(H):
            if t == 0:
                K[t, h] = f32(3.0) * np.cos((dd * 13 + seed).astype(f32) * f32(0.17)).astype(f32)
            elif t in (1, T // 4, T // 2):
                K[t, h] = f32(2.5) * np.sin((dd * 11 + t * 37 + seed).astype(f32) * f32(0.23)).astype(f32)
            else:
                amp = f32(0.1) if t > T - T // 10 else f32(0.05)
                noise = amp * np.sin((t * 31 + dd * 7 + h * 53 + seed).astype(f32) * f32(0.41)).astype(f32)
                k = base + noise
                K[t, h] = (f32(1.5) * k) if t > T - T // 10 else k
    Q = np.empty((n_q, H, d), f32)
    for q in range(n_q):
        for h in range(H):
            sw = f32(0.7) + f32(0.3) * np.sin(f32((q * 13 + h * 7 + seed)) * f32(0.29))
            sink = np.cos((dd * 13 + seed).astype(f32) * f32(0.17)).astype(f32)
            row = sw * sink + (f32(1.0) - sw) * base
            row = row + f32(0.2) * np.sin((q * 41 + dd * 3 + h * 19 + seed).astype(f32) * f32(0.37)).astype(f32)
            Q[q, h] = row
    return (np.ascontiguousarray(K.reshape(T, H * d)), np.ascontiguousarray(V.astype(f32)),
            np.ascontiguousarray(Q.reshape(n_q, H * d)))


def h16(*arrs):
    """Round inputs to fp16-representable values (as the fp16 caches of the
    benchmark configurations are) so fixtures store them as float16."""
    return tuple(np.ascontiguousarray(a.astype(np.float16).astype(np.float32)) for a in arrs)


def save(name, **arrays):
    os.makedirs(OUT, exist_ok=True)
    for k in ("K", "V", "Q"):
        if k in arrays and arrays[k].dtype == np.float32 and arrays[k].size:
            a16 = arrays[k].astype(np.float16)
            if np.array_equal(a16.astype(np.float32), arrays[k]):
                arrays[k] = a16
    np.savez_compressed(os.path.join(OUT, name + ".npz"), **arrays)


def pack_out(prefix, out):
    d = {prefix + "t": np.int32(out["t"]), prefix + "indices": out["indices"].astype(np.int32),
         prefix + "beta": out["beta"], prefix + "C_v": out["C_v"]}
    st = out["stats"]
    d[prefix + "stats"] = np.array([st["avg_cosine_sim"], st["avg_mse"], st["avg_agreement"]], np.float32)
    if "K_out" in out:
        d[prefix + "K_out"] = out["K_out"]
        d[prefix + "V_out"] = out["V_out"]
    return d


def main():
    if not os.path.exists(REF_PATH):
        sys.exit("reference library not built: run `make -C oracle ref` first")
    ref = abi.bind(ctypes.CDLL(REF_PATH))
    n = 0
    for name, dk, pk, extra in compact_cases():
        K, V, Q = h16(*workloads.small_case(dk["seed"], dk["T"], max(dk["n_q"], 1), dk["H"], dk["d"], dk["kind"]))
        Qp = None if extra.get("q_null") else Q
        params = abi.make_params(ref, **pk) if pk is not None else None
        keep = None
        if "reasoning" in extra and params is not None:
            keep = abi.Reasoner(mock_classifier(dk["T"]), *extra["reasoning"])
            keep.attach(params)
        rc, out = abi.run_compact(ref, K, V, Qp, dk["n_q"], dk["H"], dk["d"], dk["d"], params)
        assert rc == 0, (name, rc)
        meta = dict(kind="compact", data=dk, params=pk, extra={k: v for k, v in extra.items()})
        save(name, meta=json.dumps(meta), K=K, V=V, Q=Q if Qp is not None else np.zeros((0,), np.float32),
             **pack_out("", out))
        n += 1

    # spiky data with extreme ratios: exact importance ties (exp underflow)
    for ratio, tag in ((0.02, "50x"), (0.1, "10x")):
        K, V, Q = spiky(200, 16, 2, 16, 42)
        params = abi.make_params(ref, target_ratio=ratio)
        rc, out = abi.run_compact(ref, K, V, Q, 16, 2, 16, 16, params)
        assert rc == 0
        meta = dict(kind="compact", data=dict(T=200, n_q=16, H=2, d=16), params=dict(target_ratio=ratio), extra={})
        save("spiky_" + tag, meta=json.dumps(meta), K=K, V=V, Q=Q, **pack_out("", out))
        n += 1

    # quantised path: Q8_0, Q4_0, Q4_1, F16, F32 and a mixed K/V pair
    for kt, vt, tag in ((8, 8, "q8_0"), (2, 2, "q4_0"), (3, 3, "q4_1"), (1, 1, "f16"),
                        (0, 0, "f32"), (8, 2, "mixed")):
        T, n_q, H, d = 320, 32, 2, 64
        K, V, Q = h16(*workloads.small_case(100 + kt * 10 + vt, T, n_q, H, d, "rope"))
        Kq, Vq = abi.quantize_rows(ref, K, kt), abi.quantize_rows(ref, V, vt)
        params = abi.make_params(ref, target_ratio=0.2, chunk_size=160)
        rc, out = abi.run_quantized(ref, Kq, Vq, Q, kt, vt, Kq.shape[1], Vq.shape[1], T, n_q, H, d, d, params)
        assert rc == 0
        meta = dict(kind="quantized", data=dict(T=T, n_q=n_q, H=H, d=d, k_type=kt, v_type=vt),
                    params=dict(target_ratio=0.2, chunk_size=160), extra={})
        save("quant_" + tag, meta=json.dumps(meta), Kq=Kq, Vq=Vq, Q=Q, **pack_out("", out))
        n += 1

    # multi-round
    for cheap, tag in ((0, "q"), (1, "cheap")):
        K, V, Q = h16(*workloads.small_case(300 + cheap, 256, 16, 2, 32, "rope"))
        params = abi.make_params(ref, target_ratio=0.5, use_cheap_qref=cheap)
        rc, out = abi.run_multi_round(ref, K, V, Q, 16, 2, 32, 32, params, 2)
        assert rc == 0
        meta = dict(kind="multi_round", data=dict(T=256, n_q=16, H=2, d=32), params=dict(target_ratio=0.5, use_cheap_qref=cheap),
                    extra=dict(n_rounds=2))
        pr = np.array([[s["avg_cosine_sim"], s["avg_mse"], s["avg_agreement"]] for s in out["per_round"]], np.float32)
        save("multi_round_" + tag, meta=json.dumps(meta), K=K, V=V, Q=Q, per_round=pr, **pack_out("", out))
        n += 1

    # codecs on rows with edge values: zeros, constants, tiny (f16 subnormal
    # scales), large, negative-only, and random rows
    rng = np.random.default_rng(7)
    rows = [np.zeros(64, np.float32), np.full(64, 3.25, np.float32), np.full(64, -1e-6, np.float32),
            (rng.standard_normal(64) * 1e-5).astype(np.float32),
            (rng.standard_normal(64) * 3e4).astype(np.float32),
            -np.abs(rng.standard_normal(64)).astype(np.float32),
            np.linspace(-1, 1, 64).astype(np.float32)]
    rows += [rng.standard_normal(64).astype(np.float32) * s for s in (0.01, 1.0, 50.0)]
    X = np.stack(rows)
    codec = {"X": X}
    for typ, tag in ((0, "f32"), (1, "f16"), (2, "q4_0"), (3, "q4_1"), (8, "q8_0")):
        B = abi.quantize_rows(ref, X, typ)
        codec["enc_" + tag] = B
        codec["dec_" + tag] = abi.dequantize_rows(ref, B, typ, X.shape[1])
    codec["row_bytes"] = np.array([ref["quant_row_bytes"](t, 128) for t in (0, 1, 2, 3, 8)], np.int64)
    codec["row_elems"] = np.array([ref["quant_row_elements"](t, b) for t, b in ((0, 512), (1, 256), (2, 72), (3, 80), (8, 136))], np.int64)
    save("codecs", meta=json.dumps(dict(kind="codec")), **codec)
    n += 1
    print(f"wrote {n} cases to {OUT}")


if __name__ == "__main__":
    main()
