"""One model's compaction partitioned across ranks (one process per GPU).

The reference compacts a layer chunk by chunk, each chunk independently of
the others (src/kv-compact-api.cpp:463-499), and merges the chunk results by
concatenating them in chunk order with the indices offset by the chunk start
(src/kv-compact-api.cpp:514-539). A work unit here is one (layer, chunk) with
all KV heads (selection is shared across the heads of a call,
src/kv-compact-api.cpp:651-744, so heads stay together). The flattened
(layer, chunk) list of the filtered layers is cut into `world` contiguous
ranges of about equal token count; consecutive units of one layer form a
slice. A rank compacts its slices with the chunk size fixed to the layer's
own (auto) chunk size, so every chunk is planned exactly as in the whole
layer, and the merge is the reference's: rank 0 receives every slice's kept
indices (offset to layer positions), beta and the requantised K_out / V_out
rows into the whole-model result arrays at the slice's output rows. There is
no other exchange: the hot path needs no collective.
"""
from dataclasses import dataclass

import numpy as np


def auto_chunk(T, ratio):
    """The reference's auto chunk size for target_ratio `ratio` and no
    target_count (src/kv-compact-api.cpp:417-437, float arithmetic)."""
    f32 = np.float32
    re = f32(ratio)
    if re <= 0:
        re = f32(0.5)
    if re > 1:
        re = f32(1.0)
    if int(f32(T) * re) <= 256:
        return T
    cs = int(f32(256.0) / re)
    cs = max(cs, 64)
    return T if cs >= T else cs


def chunk_table(T, ratio, chunk=None):
    """[(start, C, t)] of every chunk of a layer (t = int(C * ratio) in
    float arithmetic, at least 1), chunked by `chunk` (default: auto)."""
    f32 = np.float32
    cs = auto_chunk(T, ratio) if chunk is None else chunk
    out = []
    for st in range(0, T, cs):
        C = min(cs, T - st)
        t = int(f32(C) * f32(ratio))
        out.append((st, C, max(1, min(t, C))))
    return out


@dataclass
class Slice:
    layer: int      # index into the model's filtered layers
    c0: int         # first chunk
    c1: int         # one past the last chunk
    tok0: int       # first token row
    tok1: int       # one past the last token row
    out0: int       # first output row of the layer's result arrays
    out1: int       # one past the last output row

    @property
    def tokens(self):
        return self.tok1 - self.tok0

    @property
    def kept(self):
        return self.out1 - self.out0


def partition(n_layers, T, ratio, world):
    """Per rank, the list of its slices: contiguous ranges of the flattened
    (layer, chunk) units with about total_tokens / world tokens each."""
    chunks = chunk_table(T, ratio)
    out_off = np.concatenate([[0], np.cumsum([c[2] for c in chunks])]).astype(int)
    units = [(l, c) for l in range(n_layers) for c in range(len(chunks))]
    w = np.array([chunks[c][1] for _, c in units], dtype=np.int64)
    cum = np.concatenate([[0], np.cumsum(w)])
    total = int(cum[-1])
    # rank r starts at the first unit whose preceding tokens reach r * total / world
    starts = [int(np.searchsorted(cum[:-1], r * total / world, side="left")) for r in range(world)]
    starts.append(len(units))
    ranks = []
    for r in range(world):
        a, b = starts[r], max(starts[r], starts[r + 1])
        sl = []
        i = a
        while i < b:
            l, c0 = units[i]
            j = i
            while j + 1 < b and units[j + 1][0] == l:
                j += 1
            c1 = units[j][1] + 1
            sl.append(Slice(l, c0, c1, chunks[c0][0], chunks[c1 - 1][0] + chunks[c1 - 1][1],
                            int(out_off[c0]), int(out_off[c1])))
            i = j + 1
        ranks.append(sl)
    return ranks


def layer_kept(T, ratio):
    """Kept positions of a whole layer."""
    return sum(c[2] for c in chunk_table(T, ratio))


def gather_to_root(dist, rank, world, plan, local, finals, H):
    """Merge every rank's slice outputs into rank 0's whole-model arrays.

    plan:   partition() result (the same on every rank).
    local:  on each rank, per slice of plan[rank] in order, a dict of flat
            tensors "sel" [kept] (indices relative to the slice start),
            "beta" [H * kept], "kout" [kept * k_row_bytes], "vout"
            [kept * v_row_bytes].
    finals: on rank 0, per layer, a dict of flat tensors "sel" [t],
            "beta" [H * t], "kout" [t * k_row_bytes], "vout" [t * v_row_bytes]
            (None on other ranks).
    Index offsets are added by the owner of the slice before it is sent.
    Returns after every transfer of this rank has completed.
    """
    for s, out in zip(plan[rank], local):
        out["sel"] += s.tok0                       # layer positions (src/kv-compact-api.cpp:533)
    if rank != 0:
        ops = []
        for s, out in zip(plan[rank], local):
            for k in ("sel", "beta", "kout", "vout"):
                ops.append(dist.P2POp(dist.isend, out[k].contiguous(), 0))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        return
    ops, beta_tmp = [], []
    for r in range(1, world):
        for s in plan[r]:
            f = finals[s.layer]
            kb = f["kout"].numel() // max(f["sel"].numel(), 1)
            vb = f["vout"].numel() // max(f["sel"].numel(), 1)
            bt = f["beta"].new_empty(H * s.kept)
            beta_tmp.append((s, bt))
            ops.append(dist.P2POp(dist.irecv, f["sel"][s.out0:s.out1], r))
            ops.append(dist.P2POp(dist.irecv, bt, r))
            ops.append(dist.P2POp(dist.irecv, f["kout"][s.out0 * kb:s.out1 * kb], r))
            ops.append(dist.P2POp(dist.irecv, f["vout"][s.out0 * vb:s.out1 * vb], r))
    works = dist.batch_isend_irecv(ops) if ops else []
    for s, out in zip(plan[0], local):             # rank 0's own slices
        f = finals[s.layer]
        kb = f["kout"].numel() // max(f["sel"].numel(), 1)
        vb = f["vout"].numel() // max(f["sel"].numel(), 1)
        t = f["sel"].numel()
        f["sel"][s.out0:s.out1].copy_(out["sel"])
        f["beta"].view(H, t)[:, s.out0:s.out1].copy_(out["beta"].view(H, s.kept))
        f["kout"][s.out0 * kb:s.out1 * kb].copy_(out["kout"])
        f["vout"][s.out0 * vb:s.out1 * vb].copy_(out["vout"])
    for w in works:
        w.wait()
    for s, bt in beta_tmp:                         # beta is head-major: place each head's run
        f = finals[s.layer]
        t = f["sel"].numel()
        f["beta"].view(H, t)[:, s.out0:s.out1].copy_(bt.view(H, s.kept))


class SliceJob:
    """A rank's slices, compacted through the device-resident batched API
    (kvc_compact_layers_dev): slices of equal token count share one batched
    call. K[l], V[l]: the model's block-format rows of filtered layer l
    (device uint8 tensors [T, row_bytes]); Q[l]: its reference queries."""

    def __init__(self, fns, slices, K, V, Q, T, H, d, k_type, v_type, params):
        from . import lib
        self.slices = slices
        self.H = H
        groups = {}
        for i, s in enumerate(slices):
            groups.setdefault(s.tokens, []).append(i)
        self.models = []
        for tokens, idx in groups.items():
            Ks = [K[slices[i].layer][slices[i].tok0:slices[i].tok1] for i in idx]
            Vs = [V[slices[i].layer][slices[i].tok0:slices[i].tok1] for i in idx]
            Qs = [Q[slices[i].layer] for i in idx]
            m = lib.BatchedModel(fns, Ks, Vs, Qs, tokens, H, d, d, k_type, v_type, params)
            for j, i in enumerate(idx):
                assert m.t[j] == slices[i].kept, (m.t[j], slices[i].kept)
            self.models.append((idx, m))

    def run(self, want_stats=True, gather=None):
        """Compact every slice; with a Gather, each batched call's slices are
        sent as soon as the call has returned."""
        outs = self.outputs() if gather is not None else None
        for idx, m in self.models:
            m.run(want_stats=want_stats)
            if gather is not None:
                gather.send(idx, outs)
        return outs

    def outputs(self):
        """Per slice, in order: flat views of its device results."""
        out = [None] * len(self.slices)
        for idx, m in self.models:
            for j, i in enumerate(idx):
                t = m.t[j]
                out[i] = {"sel": m.sel[j][:t], "beta": m.beta[j][:self.H * t], "kout": m.kout[j],
                          "vout": m.vout[j], "cv": m.cv[j][:self.H * t * m.md.d_v]}
        return out


class Gather:
    """The merge of gather_to_root, overlapped with the compute: rank 0 posts
    every receive before it starts computing (begin), every rank sends the
    slices of a batched call as soon as that call has returned (send), and
    finish() waits for all transfers and places rank 0's own slices and the
    head-major beta runs. Point-to-point operations between two ranks are
    posted in the same (slice, array) order on both sides."""

    def __init__(self, dist, rank, world, plan, finals, H):
        self.dist, self.rank, self.world, self.plan, self.finals, self.H = dist, rank, world, plan, finals, H
        self.works, self.beta_tmp = [], []
        self.ready, self.next = set(), 0

    def _rows(self, s):
        f = self.finals[s.layer]
        t = max(f["sel"].numel(), 1)
        return f, f["kout"].numel() // t, f["vout"].numel() // t

    def begin(self):
        self.works, self.beta_tmp = [], []
        self.ready, self.next = set(), 0
        if self.rank != 0:
            return
        d = self.dist
        for r in range(1, self.world):
            for s in self.plan[r]:
                f, kb, vb = self._rows(s)
                bt = f["beta"].new_empty(self.H * s.kept)
                self.beta_tmp.append((s, bt))
                ops = [d.P2POp(d.irecv, f["sel"][s.out0:s.out1], r), d.P2POp(d.irecv, bt, r),
                       d.P2POp(d.irecv, f["kout"][s.out0 * kb:s.out1 * kb], r),
                       d.P2POp(d.irecv, f["vout"][s.out0 * vb:s.out1 * vb], r)]
                self.works += d.batch_isend_irecv(ops)

    def send(self, idx, outs):
        """Slices plan[rank][i] for i in idx are computed (outs[i] their
        outputs). Sends leave in plan order whatever order the slices are
        computed in: a slice waits until every earlier slice of this rank
        has been sent, because rank 0 posted its receives in plan order and
        point-to-point operations between two ranks match in posting order."""
        d = self.dist
        for i in idx:
            s, out = self.plan[self.rank][i], outs[i]
            out["sel"] += s.tok0                 # layer positions (src/kv-compact-api.cpp:533)
            self.ready.add(i)
        while self.next in self.ready:
            i = self.next
            self.ready.discard(i)
            self.next += 1
            if self.rank == 0:
                continue
            ops = [d.P2POp(d.isend, outs[i][k].contiguous(), 0) for k in ("sel", "beta", "kout", "vout")]
            self.works += d.batch_isend_irecv(ops)

    def finish(self, outs):
        if self.next != len(self.plan[self.rank]):
            raise RuntimeError(f"rank {self.rank}: slices {sorted(set(range(len(self.plan[self.rank]))) - set(range(self.next)))} "
                               "were never sent")
        if self.rank == 0:
            H = self.H
            for s, out in zip(self.plan[0], outs):
                f, kb, vb = self._rows(s)
                t = f["sel"].numel()
                f["sel"][s.out0:s.out1].copy_(out["sel"])
                f["beta"].view(H, t)[:, s.out0:s.out1].copy_(out["beta"].view(H, s.kept))
                f["kout"][s.out0 * kb:s.out1 * kb].copy_(out["kout"])
                f["vout"][s.out0 * vb:s.out1 * vb].copy_(out["vout"])
        for w in self.works:
            w.wait()
        if self.rank == 0:
            for s, bt in self.beta_tmp:
                f = self.finals[s.layer]
                t = f["sel"].numel()
                f["beta"].view(self.H, t)[:, s.out0:s.out1].copy_(bt.view(self.H, s.kept))
        self.works, self.beta_tmp = [], []
