"""Parity helpers: chunk geometry, near-tie classification of index
mismatches, and an fp64 solve of the ridge least-squares problem.

Tolerances (the bar the parity tests hold libkvc.so to):
  * selected indices: bit-exact, except keys whose oracle importances differ
    from the key they displaced by less than NEAR_TIE_REL (relative gap);
    every such swap is reported;
  * C_v: within CV_REL_TOL relative L2 of the fp64 solution of the same
    ridge problem, or no farther from it than the reference's own C_v
    (the reference's fp32 Gaussian elimination carries ~1e-2 null-space noise
    when n_q < t);
  * compacted-attention cosine (stats.avg_cosine_sim) >= 0.9999 x the
    reference's;
  * quantised rows: bit-exact for every row whose index matches.
"""
import math

import numpy as np

NEAR_TIE_REL = 1e-6
CV_REL_TOL = 1e-3
COS_RATIO = 0.9999


def cheap_nq(T):
    n = T // 2
    n = min(n, 64)
    n = max(n, 4)
    return min(n, T)


def t_for(T, p):
    f32 = np.float32
    if p.get("target_count", 0) > 0:
        t = min(p["target_count"], T)
    else:
        t = int(f32(T) * f32(p.get("target_ratio", 0.5)))
        t = max(1, min(t, T))
    pre = p.get("n_shared_prefix", 0)
    if pre > t:
        t = min(pre, T)
    return t


def plan_units(T, p):
    """[(start, C, t, prefix, cheap_chunk)] as the reference's kv_compact chunks."""
    f32 = np.float32
    cs = p.get("chunk_size", 0)
    if cs == 0:
        tc = p.get("target_count", 0)
        re = f32(tc) / f32(T) if tc > 0 else f32(p.get("target_ratio", 0.5))
        if re <= 0:
            re = f32(0.5)
        if re > 1:
            re = f32(1.0)
        et = int(f32(T) * re)
        if et > 256:
            cs = int(f32(256.0) / re)
            cs = max(cs, 64)
            if cs >= T:
                cs = T
        else:
            cs = T
    elif cs < 0:
        cs = T
    pre_top = p.get("n_shared_prefix", 0)
    if cs >= T:
        t = t_for(T, p)
        return [(0, T, t, max(0, min(pre_top, t)), False)]
    out = []
    for c in range((T + cs - 1) // cs):
        st = c * cs
        C = min(cs, T - st)
        pre = pre_top if c == 0 else 0
        pre = min(pre, C)
        cp = dict(p)
        cp["n_shared_prefix"] = pre
        t = t_for(C, cp)
        out.append((st, C, t, max(0, min(pre, t)), bool(p.get("use_cheap_qref", 0))))
    return out


def classify_indices(ours, ref, imp, units):
    """Returns (n_mismatch, n_near_tie, worst_rel_gap_of_non_ties)."""
    ours, ref = set(int(x) for x in ours), set(int(x) for x in ref)
    mism = ties = 0
    worst = 0.0
    for (st, C, t, pre, _) in units:
        o = {j for j in ours if st <= j < st + C}
        r = {j for j in ref if st <= j < st + C}
        a = sorted(o - r, key=lambda j: -imp[j])
        b = sorted(r - o, key=lambda j: -imp[j])
        if len(a) != len(b):
            mism += max(len(a), len(b))
            worst = max(worst, 1.0)
            continue
        for x, y in zip(a, b):
            mism += 1
            va, vb = float(imp[x]), float(imp[y])
            den = max(abs(va), abs(vb))
            gap = 0.0 if den < 1e-30 else abs(va - vb) / den
            if gap < NEAR_TIE_REL:
                ties += 1
            else:
                worst = max(worst, gap)
    return mism, ties, worst


def _softmax(x):
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)


def cheap_rows(n, T):
    out = []
    for qi in range(n):
        fr = np.float32(qi + 1) / np.float32(n + 1)
        fr = np.float32(fr * fr)
        pos = int(np.float32(fr * np.float32(T - 1)))
        out.append(min(max(pos, 0), T - 1))
    return out


def exact_cv(K, V, Q, H, d, sel, beta, units, p, q_null):
    """fp64 ridge solution for the given selection and beta, per head [t x d]."""
    ridge = float(np.float32(p.get("ridge", 1e-6)))
    K64, V64 = K.astype(np.float64), V.astype(np.float64)
    T = K.shape[0]
    if q_null or p.get("use_cheap_qref", 0):
        Qtop = K64[cheap_rows(cheap_nq(T), T)]
    else:
        Qtop = Q.astype(np.float64)
    sel = np.asarray(sel)
    out = np.zeros((H, len(sel), d))
    off = 0
    for (st, C, t, pre, cheap_chunk) in units:
        s_loc = sel[off:off + t] - st
        Kc, Vc = K64[st:st + C], V64[st:st + C]
        Qc = Kc[cheap_rows(cheap_nq(C), C)] if cheap_chunk else Qtop
        for h in range(H):
            q = Qc[:, h * d:(h + 1) * d]
            k = Kc[:, h * d:(h + 1) * d]
            v = Vc[:, h * d:(h + 1) * d]
            S = q @ k.T / math.sqrt(d)
            Y = _softmax(S) @ v
            X = _softmax(S[:, s_loc] + beta[h, off:off + t][None, :].astype(np.float64))
            nq = X.shape[0]
            if nq < t:
                Z = np.linalg.solve(X @ X.T + ridge * np.eye(nq), Y)
                Cv = X.T @ Z
            else:
                Cv = np.linalg.solve(X.T @ X + ridge * np.eye(t), X.T @ Y)
            out[h, off:off + t] = Cv
        off += t
    return out


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def nnls_residuals(K, Q, H, d, sel, beta, units):
    """Per (chunk, head): the residual ||M w - b|| of the bias fit in fp64,
    with M[q, j] = exp(S[q, sel_j] - max_q), b[q] = sum_j exp(S[q, j] - max_q)
    over the chunk's keys and w = exp(beta) (the problem the reference's
    Lawson-Hanson fit solves, src/kv-compact-api.cpp:812-831)."""
    K64, Q64 = K.astype(np.float64), Q.astype(np.float64)
    sel = np.asarray(sel)
    out = []
    off = 0
    for (st, C, t, pre, cheap_chunk) in units:
        s_loc = sel[off:off + t] - st
        for h in range(H):
            S = Q64[:, h * d:(h + 1) * d] @ K64[st:st + C, h * d:(h + 1) * d].T / math.sqrt(d)
            E = np.exp(S - S.max(axis=1, keepdims=True))
            w = np.exp(beta[h, off:off + t].astype(np.float64))
            out.append(float(np.linalg.norm(E[:, s_loc] @ w - E.sum(axis=1))))
        off += t
    return np.array(out)

