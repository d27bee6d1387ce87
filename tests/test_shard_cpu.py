"""Partition of one model across ranks and the merge of the slice results on
rank 0 (kvc_b200.shard), on CPU: the partition covers every (layer, chunk)
unit exactly once in order, balanced by tokens; the slices' output rows are
the chunks' kept counts as the reference plans them; and the gather over two
and three gloo ranks rebuilds the whole-model arrays exactly as one rank
holding every slice would."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import parity
from kvc_b200 import shard


def test_partition_covers_every_unit_once_in_order():
    for n_layers, T, ratio, world in [(12, 100_000, 0.2, 8), (12, 100_000, 0.2, 3), (32, 16_384, 0.2, 4),
                                      (1, 4096, 0.5, 2), (2, 3000, 0.2, 8), (12, 100_000, 0.2, 1)]:
        plan = shard.partition(n_layers, T, ratio, world)
        assert len(plan) == world
        chunks = shard.chunk_table(T, ratio)
        ref_units = parity.plan_units(T, dict(target_ratio=ratio))
        assert [(c[0], c[1], c[2]) for c in chunks] == [(u[0], u[1], u[2]) for u in ref_units]
        seen = []
        for sl in plan:
            for s in sl:
                assert s.tok0 == chunks[s.c0][0] and s.tok1 == chunks[s.c1 - 1][0] + chunks[s.c1 - 1][1]
                assert s.kept == sum(c[2] for c in chunks[s.c0:s.c1])
                seen += [(s.layer, c) for c in range(s.c0, s.c1)]
        assert seen == [(l, c) for l in range(n_layers) for c in range(len(chunks))]
        loads = [sum(s.tokens for s in sl) for sl in plan]
        assert sum(loads) == n_layers * T
        if n_layers * len(chunks) >= world:
            assert max(loads) - min(loads) <= 2 * max(c[1] for c in chunks)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _whole(n_layers, T, ratio, H, kb, vb):
    """Deterministic stand-ins of whole-layer results (indices in layer positions)."""
    out = []
    for l in range(n_layers):
        chunks = shard.chunk_table(T, ratio)
        sel = np.concatenate([st + np.arange(t) * 3 % C for st, C, t in chunks]).astype(np.int32)
        t = len(sel)
        rng = np.random.default_rng(l)
        out.append({"sel": sel, "beta": rng.standard_normal(H * t).astype(np.float32),
                    "kout": rng.integers(0, 255, t * kb, dtype=np.uint8),
                    "vout": rng.integers(0, 255, t * vb, dtype=np.uint8)})
    return out


def _worker(rank, world, port, q, n_layers, T, ratio, H, kb, vb, overlapped=False):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import torch
    import torch.distributed as dist
    from kvc_b200 import dist as kdist
    try:
        kdist.init("gloo", timeout_s=60)
        plan = shard.partition(n_layers, T, ratio, world)
        whole = _whole(n_layers, T, ratio, H, kb, vb)
        local = []
        for s in plan[rank]:                       # this rank's slice outputs, indices slice-relative
            w = whole[s.layer]
            t = len(w["sel"])
            local.append({"sel": torch.from_numpy(w["sel"][s.out0:s.out1] - s.tok0),
                          "beta": torch.from_numpy(w["beta"].reshape(H, t)[:, s.out0:s.out1].copy()).reshape(-1),
                          "kout": torch.from_numpy(w["kout"][s.out0 * kb:s.out1 * kb].copy()),
                          "vout": torch.from_numpy(w["vout"][s.out0 * vb:s.out1 * vb].copy())})
        finals = None
        if rank == 0:
            t = shard.layer_kept(T, ratio)
            finals = [{"sel": torch.full((t,), -1, dtype=torch.int32), "beta": torch.full((H * t,), np.nan),
                       "kout": torch.zeros(t * kb, dtype=torch.uint8), "vout": torch.zeros(t * vb, dtype=torch.uint8)}
                      for _ in range(n_layers)]
        if overlapped:                             # receives first, each slice sent as it is "computed"
            g = shard.Gather(dist, rank, world, plan, finals, H)
            g.begin()
            for i in reversed(range(len(local))):  # computed out of plan order: sends must still match
                g.send([i], local)
            g.finish(local)
        else:
            shard.gather_to_root(dist, rank, world, plan, local, finals, H)
        ok = True
        if rank == 0:
            for l in range(n_layers):
                for k in ("sel", "beta", "kout", "vout"):
                    ok = ok and np.array_equal(finals[l][k].numpy(), whole[l][k])
        kdist.finish(world)
        q.put((rank, ok, None))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("world,overlapped", [(2, False), (3, False), (2, True), (3, True)])
def test_gather_rebuilds_whole_model_arrays(world, overlapped):
    args = (3, 5000, 0.2, 2, 34, 18, overlapped)   # 3 layers x 4 chunks, 2 heads, row bytes 34 / 18
    # world 2: each rank holds two slices, sent below in reverse order when overlapped
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, ok, err = q.get(timeout=120)
        assert err is None, err
        res[rank] = ok
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0]


@pytest.mark.parametrize("world,extra", [(2, 0.0), (2, 0.05), (3, 0.05), (8, 0.05), (5, 0.3)])
def test_weighted_partition_and_peer_copy_plan(world, extra):
    """Rank 0's larger share (root_weights) keeps the partition exact, and the
    peer copies of every rank's slices (put_ops, applied here to one host
    buffer as rank 0's result buffer) rebuild the whole-model arrays."""
    n_layers, T, ratio, H, kb, vb = 3, 5000, 0.2, 2, 34, 18
    w = shard.root_weights(world, extra)
    plan = shard.partition(n_layers, T, ratio, world, w)
    chunks = shard.chunk_table(T, ratio)
    seen = [(s.layer, c) for sl in plan for s in sl for c in range(s.c0, s.c1)]
    assert seen == [(l, c) for l in range(n_layers) for c in range(len(chunks))]
    loads = np.array([sum(s.tokens for s in sl) for sl in plan], dtype=float)
    want = np.array(w) / sum(w) * n_layers * T
    assert np.all(np.abs(loads - want) <= max(c[1] for c in chunks))
    whole = _whole(n_layers, T, ratio, H, kb, vb)
    layout, nbytes = shard.result_layout(n_layers, T, ratio, H, kb, vb)
    buf = np.zeros(nbytes, dtype=np.uint8)
    for r in range(world):
        for s in plan[r]:
            wl = whole[s.layer]
            t = len(wl["sel"])
            out = {"sel": (wl["sel"][s.out0:s.out1]).astype(np.int32).view(np.uint8),
                   "beta": np.ascontiguousarray(wl["beta"].reshape(H, t)[:, s.out0:s.out1]).view(np.uint8).ravel(),
                   "kout": wl["kout"][s.out0 * kb:s.out1 * kb], "vout": wl["vout"][s.out0 * vb:s.out1 * vb]}
            for op in shard.put_ops(s, layout, T, ratio, H, kb, vb):
                src = out[op[1]]
                if op[0] == "1d":
                    _, _, dst, so, n = op
                    buf[dst:dst + n] = src[so:so + n]
                else:
                    _, _, dst, dp, sp, width, height = op
                    for i in range(height):
                        buf[dst + i * dp:dst + i * dp + width] = src[i * sp:i * sp + width]
    for l in range(n_layers):
        L = layout[l]
        got = {k: buf[L[k][0]:L[k][0] + L[k][1]] for k in L}
        assert np.array_equal(got["sel"].view(np.int32), whole[l]["sel"])
        assert np.array_equal(got["beta"].view(np.float32), whole[l]["beta"])
        assert np.array_equal(got["kout"], whole[l]["kout"])
        assert np.array_equal(got["vout"], whole[l]["vout"])
        offs = sorted(v[0] for v in L.values())
        assert all(o % 256 == 0 for o in offs)
