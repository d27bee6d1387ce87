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


def partition(n_layers, T, ratio, world, weights=None):
    """Per rank, the list of its slices: contiguous ranges of the flattened
    (layer, chunk) units with about total_tokens * weights[r] / sum(weights)
    tokens each (equal shares by default)."""
    chunks = chunk_table(T, ratio)
    out_off = np.concatenate([[0], np.cumsum([c[2] for c in chunks])]).astype(int)
    units = [(l, c) for l in range(n_layers) for c in range(len(chunks))]
    w = np.array([chunks[c][1] for _, c in units], dtype=np.int64)
    cum = np.concatenate([[0], np.cumsum(w)])
    total = int(cum[-1])
    wt = np.ones(world) if weights is None else np.asarray(weights, dtype=np.float64)
    if len(wt) != world or np.any(wt <= 0):
        raise ValueError("one positive weight per rank")
    bound = np.concatenate([[0.0], np.cumsum(wt)]) / wt.sum() * total
    # rank r starts at the first unit whose preceding tokens reach bound[r]
    starts = [int(np.searchsorted(cum[:-1], bound[r], side="left")) for r in range(world)]
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
    (kvc_compact_layers_dev) in one call: each slice is a layer of the call
    with its own token count (kvc_layer_desc.n_tokens). K[l], V[l]: the
    model's block-format rows of filtered layer l (device uint8 tensors
    [T, row_bytes]); Q[l]: its reference queries. out_ptrs: per slice, the
    device addresses (K_out, V_out) its requantised rows are written to
    (e.g. PeerGather.out_ptrs(): rank 0's result arrays, local or mapped),
    else buffers of its own."""

    def __init__(self, fns, slices, K, V, Q, T, H, d, k_type, v_type, params, out_ptrs=None):
        from . import lib
        self.slices = slices
        self.H = H
        self.models = []
        if not slices:
            return
        idx = list(range(len(slices)))
        Ks = [K[s.layer][s.tok0:s.tok1] for s in slices]
        Vs = [V[s.layer][s.tok0:s.tok1] for s in slices]
        Qs = [Q[s.layer] for s in slices]
        tokens = [s.tokens for s in slices]
        m = lib.BatchedModel(fns, Ks, Vs, Qs, max(tokens), H, d, d, k_type, v_type, params, tokens=tokens,
                             out_ptrs=out_ptrs)
        for j, s in enumerate(slices):
            assert m.t[j] == s.kept, (m.t[j], s.kept)
        self.models.append((idx, m))

    def run(self, want_stats=True, gather=None):
        """Compact every slice; with a Gather, each batched call's slices are
        sent as soon as the call has returned."""
        if gather is not None and getattr(self, "_outs", None) is None:
            self._outs = self.outputs()          # the same views every step
        outs = self._outs if gather is not None else None
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
        """Post rank 0's receives. First wait until the previous step's
        transfers are done: the library computes on its own stream, so the
        next batched call must not rewrite arrays that a send still reads."""
        import torch
        if torch.cuda.is_available():
            torch.cuda.current_stream().synchronize()
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


def root_weights(world, extra=0.03):
    """Partition weights that give rank 0 a larger share: the other ranks
    finish their compute earlier by about the time their peer copies into
    rank 0's result arrays take, so the copies land while rank 0 computes."""
    return [1.0 + extra * (world - 1)] + [1.0] * (world - 1)


def result_layout(n_layers, T, ratio, H, k_row_bytes, v_row_bytes, align=256):
    """Byte layout of one model's result arrays in a single buffer: per layer
    {"sel": (offset, bytes), "beta", "kout", "vout"}, each array aligned to
    `align` bytes; returns (layers, total bytes). sel int32 [t], beta fp32
    [H, t] (head-major, as the reference returns it), K_out / V_out rows."""
    t = layer_kept(T, ratio)
    sizes = (("sel", 4 * t), ("beta", 4 * H * t), ("kout", t * k_row_bytes), ("vout", t * v_row_bytes))
    off, layers = 0, []
    for _ in range(n_layers):
        d = {}
        for k, nb in sizes:
            d[k] = (off, nb)
            off += (nb + align - 1) // align * align
        layers.append(d)
    return layers, off


def put_ops(s, layout, T, ratio, H, k_row_bytes, v_row_bytes):
    """The copies that place slice s's outputs into the result buffer:
    ("1d", array, dst offset, src offset, bytes) and, for beta's H runs,
    ("2d", "beta", dst offset, dst pitch, src pitch, width, height). Source
    offsets are within the slice's own flat output arrays."""
    t = layer_kept(T, ratio)
    L = layout[s.layer]
    kept = s.kept
    return [("1d", "sel", L["sel"][0] + 4 * s.out0, 0, 4 * kept),
            ("2d", "beta", L["beta"][0] + 4 * s.out0, 4 * t, 4 * kept, 4 * kept, H),
            ("1d", "kout", L["kout"][0] + k_row_bytes * s.out0, 0, k_row_bytes * kept),
            ("1d", "vout", L["vout"][0] + v_row_bytes * s.out0, 0, v_row_bytes * kept)]


class _CudaBuffer:
    """A raw device allocation seen by torch.as_tensor (no copy)."""

    def __init__(self, ptr, nbytes, device_index):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}
        self.device_index = device_index


class PeerGather:
    """The reference's chunk merge across GPUs through peer memory: rank 0
    owns one buffer with the whole model's result arrays (result_layout),
    allocated through kvc_peer_alloc; every other rank maps it
    (kvc_peer_open). Each rank's batched call writes its slices' requantised
    K_out / V_out rows straight to their rows there (out_ptrs(), given to
    SliceJob: the requantisation kernels store over NVLink), and send() adds
    one kvc_place_slice launch per slice for the kept indices (offset to
    layer positions) and the head-major beta runs. finish() orders the step:
    a one-element all-reduce on every rank's current stream, which on the
    other ranks runs after their writes, so rank 0's arrays are complete once
    it returns. No receive is posted and nothing is copied twice. Construct
    and close() on every rank together (collective)."""

    def __init__(self, dist, fns, rank, world, plan, n_layers, T, ratio, H, k_row_bytes, v_row_bytes, device,
                 copy_rows=False):
        import ctypes
        import torch
        self.dist, self.lib, self.rank, self.world, self.plan = dist, fns["_lib"], rank, world, plan
        # copy_rows: K_out / V_out are requantised into the rank's own buffers
        # and each slice's two row arrays go to rank 0 as one copy-engine copy
        # each (out_ptrs() then gives None), instead of the requantisation
        # kernels storing them over NVLink
        self.copy_rows = copy_rows
        self.T, self.ratio, self.H, self.krb, self.vrb = T, ratio, H, k_row_bytes, v_row_bytes
        self.device = device
        self.layout, self.nbytes = result_layout(n_layers, T, ratio, H, k_row_bytes, v_row_bytes)
        self.ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        if rank == 0:
            rc = self.lib.kvc_peer_alloc(self.nbytes, ctypes.byref(self.ptr), handle)
            if rc != 0:
                raise RuntimeError(f"kvc_peer_alloc failed: {rc}")
        box = [bytes(handle)]
        dist.broadcast_object_list(box, src=0, device=device)
        if rank != 0:
            ctypes.memmove(handle, box[0], 64)
            rc = self.lib.kvc_peer_open(handle, ctypes.byref(self.ptr))
            if rc != 0:
                raise RuntimeError(f"kvc_peer_open failed: {rc}")
        self.base = self.ptr.value
        self.finals = None
        if rank == 0:
            buf = torch.as_tensor(_CudaBuffer(self.base, self.nbytes, device.index), device=device)
            t = layer_kept(T, ratio)
            self.finals = []
            for L in self.layout:
                view = lambda k, dt: buf[L[k][0]:L[k][0] + L[k][1]].view(dt)   # noqa: E731
                self.finals.append({"sel": view("sel", torch.int32), "beta": view("beta", torch.float32),
                                    "kout": view("kout", torch.uint8), "vout": view("vout", torch.uint8)})
            assert all(f["sel"].numel() == t for f in self.finals)
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)
        # per slice of this rank: (kept, tok0, sel address, beta address, K_out, V_out addresses)
        self.t = layer_kept(T, ratio)
        self.dst = []
        for s in plan[rank]:
            ops = {op[1]: op for op in put_ops(s, self.layout, T, ratio, H, k_row_bytes, v_row_bytes)}
            self.dst.append((s.kept, s.tok0, self.base + ops["sel"][2], self.base + ops["beta"][2],
                             self.base + ops["kout"][2], self.base + ops["vout"][2]))

    def begin(self):
        """Wait until the previous step's copies (and its all-reduce) are
        done: the library computes on its own stream, so the next batched
        call must not rewrite output arrays that a copy still reads."""
        import torch
        torch.cuda.current_stream(self.device).synchronize()

    def out_ptrs(self):
        """Per slice of this rank, the addresses of its K_out / V_out rows in
        rank 0's result buffer (put_ops' destinations)."""
        if self.copy_rows:
            return None
        return [(d[4], d[5]) for d in self.dst]

    def send(self, idx, outs):
        """Slices plan[rank][i] for i in idx are computed (outs[i] their
        outputs; their K_out / V_out rows are already in place)."""
        import torch
        st = torch.cuda.current_stream(self.device).cuda_stream
        for i in idx:
            kept, tok0, sel_dst, beta_dst = self.dst[i][:4]
            rc = self.lib.kvc_place_slice(outs[i]["sel"].data_ptr(), outs[i]["beta"].data_ptr(), kept, self.H, tok0,
                                          sel_dst, beta_dst, self.t, st)
            if rc != 0:
                raise RuntimeError(f"kvc_place_slice failed: {rc}")
            if self.copy_rows:
                for dst, src, nb in ((self.dst[i][4], outs[i]["kout"], kept * self.krb),
                                     (self.dst[i][5], outs[i]["vout"], kept * self.vrb)):
                    rc = self.lib.kvc_copy_async(dst, src.data_ptr(), nb, st)
                    if rc != 0:
                        raise RuntimeError(f"peer copy failed: {rc}")

    def finish(self, outs):
        self.dist.all_reduce(self.flag)          # after this rank's copies, on every rank

    def close(self):
        import torch
        torch.cuda.synchronize(self.device)
        if self.rank != 0 and self.base:
            self.lib.kvc_peer_close(self.base)
        self.dist.barrier()
        if self.rank == 0 and self.base:
            self.finals = None
            self.lib.kvc_peer_free(self.base)
        self.base = None
