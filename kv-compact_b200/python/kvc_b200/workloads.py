"""Seeded synthetic caches with the shapes and value distributions of the
benchmark configurations (no public dataset is involved; every input is
generated from a seed).

  cfg1  1 layer, 1 KV head, d=128, T=4096, fp32. K = U[Tx16] W[16x128] + N(0,0.1),
        U, W ~ N(0,1), channels 0-3 scaled x8; V ~ N(0,1); K-as-Q (cheap Q).
  cfg2  32 layers x 8 KV heads x d=128, T=16384, fp16 K/V. K = RoPE(theta=5e5)
        applied (rotate-half, positions 0..T-1) to a rank-32 Gaussian base
        (U W / sqrt(32), so entries ~N(0,1)) plus N(0,0.05); V ~ N(0,1).
        Q: SnapKV window W=32 of N(0,1) queries over 32 q-heads, GQA group 4,
        flattened to n_q=128 rows: row w*4+g of KV head h holds q-head h*4+g.
  cfg3  cfg2 at T=1,048,576 with a 1024-token shared prefix.
  cfg4  48 layers x 8 x 128, T=100,000, every 4th layer compacted (12),
        K/V from the cfg2 distributions stored as Q8_0 (or Q4_0).
  cfg5  16 layers x 4 x 128, T=32768, fp32 cfg1 distributions, 256 N(0,1)
        queries, beta by Lawson-Hanson, diversity 0.1, 2 refinement rounds.

numpy versions serve small test cases; torch versions generate full-size
caches directly in device memory for bench.py.
"""
import math

import numpy as np

ROPE_THETA = 500000.0


def rope_rotate_half(x, positions, theta=ROPE_THETA):
    """Rotate-half RoPE on the last axis of x [..., T, d] (numpy, float64 math)."""
    d = x.shape[-1]
    half = d // 2
    inv = theta ** (-np.arange(half, dtype=np.float64) * 2.0 / d)
    ang = positions[:, None].astype(np.float64) * inv[None, :]
    c, s = np.cos(ang), np.sin(ang)
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def lowrank_keys(rng, T, H, d, rank=16, noise=0.1, outliers=4, outlier_scale=8.0):
    """cfg1 keys: [T x H*d] float32."""
    out = np.empty((T, H, d), np.float32)
    for h in range(H):
        U = rng.standard_normal((T, rank)).astype(np.float32)
        W = rng.standard_normal((rank, d)).astype(np.float32)
        k = U @ W + noise * rng.standard_normal((T, d)).astype(np.float32)
        k[:, :outliers] *= outlier_scale
        out[:, h, :] = k
    return out.reshape(T, H * d)


def rope_keys(rng, T, H, d, rank=32, noise=0.05, start=0):
    """cfg2 keys: [T x H*d] float32."""
    out = np.empty((T, H, d), np.float32)
    pos = np.arange(start, start + T)
    for h in range(H):
        U = rng.standard_normal((T, rank))
        W = rng.standard_normal((rank, d))
        base = (U @ W) / math.sqrt(rank)
        out[:, h, :] = rope_rotate_half(base, pos) + noise * rng.standard_normal((T, d))
    return out.reshape(T, H * d)


def snapkv_queries(rng, H, d, window=32, group=4):
    """[window*group x H*d]: row w*group+g of KV head h = q-head h*group+g."""
    q = rng.standard_normal((window, H * group, d)).astype(np.float32)
    out = np.empty((window * group, H, d), np.float32)
    for h in range(H):
        for g in range(group):
            out[g::group, h, :] = q[:, h * group + g, :]
    return out.reshape(window * group, H * d)


def small_case(seed, T, n_q, H, d, kind="rope"):
    """(K, V, Q) float32 for parity tests."""
    rng = np.random.default_rng(seed)
    if kind == "rope":
        K = rope_keys(rng, T, H, d)
    elif kind == "lowrank":
        K = lowrank_keys(rng, T, H, d)
    elif kind == "gauss":
        K = rng.standard_normal((T, H * d)).astype(np.float32)
    else:
        raise ValueError(kind)
    V = rng.standard_normal((T, H * d)).astype(np.float32)
    if kind == "rope" and n_q % 4 == 0:
        Q = snapkv_queries(rng, H, d, window=n_q // 4, group=4)
    else:
        Q = rng.standard_normal((n_q, H * d)).astype(np.float32)
    return np.ascontiguousarray(K), np.ascontiguousarray(V), np.ascontiguousarray(Q)


def sincos_data(n, seed):
    """The reference tests' deterministic generator (tests/test-kv-compact-api.cpp:16-21)."""
    i = np.arange(n, dtype=np.float64)
    a = np.sin(((i * 7 + seed).astype(np.float32) * np.float32(0.31)).astype(np.float32))
    b = np.cos(((i * 3 + seed + 17).astype(np.float32) * np.float32(0.53)).astype(np.float32))
    return (a.astype(np.float32) + np.float32(0.3) * b.astype(np.float32)).astype(np.float32)


# ---------------------------------------------------------------------------
# torch generators (device-resident, for the full-size benchmark)
# ---------------------------------------------------------------------------

def torch_rope_keys(T, H, d, gen, device, rank=32, noise=0.05, dtype=None):
    """cfg2 keys for one layer on `device`: [T, H*d] float32."""
    import torch
    half = d // 2
    inv = torch.pow(torch.tensor(ROPE_THETA, dtype=torch.float64, device=device),
                    -torch.arange(half, dtype=torch.float64, device=device) * 2.0 / d)
    pos = torch.arange(T, dtype=torch.float64, device=device)
    ang = pos[:, None] * inv[None, :]
    c = torch.cos(ang).float()
    s = torch.sin(ang).float()
    out = torch.empty((T, H, d), dtype=torch.float32, device=device)
    for h in range(H):
        U = torch.randn((T, rank), generator=gen, device=device)
        W = torch.randn((rank, d), generator=gen, device=device)
        base = (U @ W) * (1.0 / math.sqrt(rank))
        x1, x2 = base[:, :half], base[:, half:]
        out[:, h, :half] = x1 * c - x2 * s
        out[:, h, half:] = x2 * c + x1 * s
        out[:, h, :] += noise * torch.randn((T, d), generator=gen, device=device)
    return out.reshape(T, H * d)


def torch_snapkv_queries(H, d, gen, device, window=32, group=4):
    import torch
    q = torch.randn((window, H * group, d), generator=gen, device=device)
    out = torch.empty((window * group, H, d), dtype=torch.float32, device=device)
    for h in range(H):
        for g in range(group):
            out[g::group, h, :] = q[:, h * group + g, :]
    return out.reshape(window * group, H * d)
