#!/usr/bin/env python
"""Compaction throughput of the kv-compact hot path on B200.

Metric: compaction input tokens/s over all filtered layers x
KV heads, 100k context, 5x compression (20% retention). Default workload is
configuration 4: 48 layers x 8 KV heads x d=128, T=100,000, every 4th layer
compacted (12 layers), K/V stored Q8_0, SnapKV window W=32 over 32 query
heads with GQA 4 (n_q=128), dequant -> compact -> requant, stats included.

One step = one whole-model compaction (all 12 filtered layers) with the
caches resident in HBM (value), or through the drop-in C ABI
(kv_compact_quantized per layer) from pinned host buffers with the copies
inside the timed region (e2e). Inputs (2.6 GB) exceed the 126 MB L2, so no
flush is needed between steps.

Multi-GPU (torchrun): the ranks share ONE model ("strong" scaling): the
(layer, chunk) units are partitioned into contiguous token-balanced ranges
(kvc_b200.shard), each rank compacts its share, and the kept indices, beta
and requantised K/V rows are gathered to rank 0 over NCCL inside the timed
region; value = the model's tokens / max-over-ranks step time. --replicas
runs one independent model per rank instead ("weak" scaling).

--impl reference runs the reference's own CPU library (oracle/_ref, built
from the reference sources) with all host threads on a bounded sample of the
same workload; rank 0 only.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "kv-compact_b200", "python"))

import numpy as np  # noqa: E402

from kvc_b200 import ORACLE_PATH, REF_PATH, abi, dist as kdist, workloads  # noqa: E402

CONFIGS = {
    "cfg4_q8": dict(n_layers=48, interval=4, T=100_000, H=8, d=128, ktype=abi.KV_TYPE_Q8_0,
                    vtype=abi.KV_TYPE_Q8_0, ratio=0.2, window=32, group=4),
    "cfg4_q4": dict(n_layers=48, interval=4, T=100_000, H=8, d=128, ktype=abi.KV_TYPE_Q4_0,
                    vtype=abi.KV_TYPE_Q4_0, ratio=0.2, window=32, group=4),
    "cfg2": dict(n_layers=32, interval=1, T=16_384, H=8, d=128, ktype=abi.KV_TYPE_F16,
                 vtype=abi.KV_TYPE_F16, ratio=0.2, window=32, group=4),
}
TYPE_NAME = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 8: "Q8_0"}
METRIC = "compaction input tokens/s, all layers×KV-heads, 100k ctx 5x; % of roofline"


def filtered_layers(cfg):
    ls = [l for l in range(cfg["n_layers"]) if cfg["interval"] <= 1 or (l + 1) % cfg["interval"] == 0]
    return ls[:cfg["max_layers"]] if cfg.get("max_layers") else ls


def workload_desc(name, cfg):
    n = len(filtered_layers(cfg))
    return (f"{name}: {cfg['n_layers']} layers x {cfg['H']} KV heads x d={cfg['d']}, T={cfg['T']}, "
            f"{n} layers compacted (every {cfg['interval']}th), {TYPE_NAME[cfg['ktype']]} K/V, "
            f"ratio {cfg['ratio']}, SnapKV W={cfg['window']} x GQA {cfg['group']} (n_q={cfg['window'] * cfg['group']}), "
            f"dequant->compact->requant + quality stats")


def make_layers(cfg, seed, device, fns):
    """Quantised K/V and fp32 queries of every filtered layer, generated on `device`."""
    import torch
    from kvc_b200 import lib
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    T, H, d = cfg["T"], cfg["H"], cfg["d"]
    Kq, Vq, Q = [], [], []
    for _ in filtered_layers(cfg):
        K = workloads.torch_rope_keys(T, H, d, g, device)
        V = torch.randn((T, H * d), generator=g, device=device)
        Kq.append(lib.quantize_dev(fns, K, cfg["ktype"]))
        Vq.append(lib.quantize_dev(fns, V, cfg["vtype"]))
        Q.append(workloads.torch_snapkv_queries(H, d, g, device, cfg["window"], cfg["group"]).contiguous())
        del K, V
    return Kq, Vq, Q


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if gpu_id:
            cmd += ["-i", gpu_id]
        try:
            self.p = subprocess.Popen(cmd, stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        rows = [r.split(", ") for r in open(self.f.name).read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def host_cores():
    """Host threads this process may run on."""
    return len(os.sched_getaffinity(0))


def cpu_library():
    """(bound functions, kind): the reference library built from its sources
    (oracle/_ref) when present, else the C restatement of its CPU path."""
    if os.path.exists(REF_PATH):
        return abi.bind(ctypes.CDLL(REF_PATH, mode=ctypes.RTLD_LOCAL)), "reference"
    return abi.bind(ctypes.CDLL(ORACLE_PATH, mode=ctypes.RTLD_LOCAL), prefix="oracle_"), "port"


def cpu_sample_tokens(cfg, kind, cores):
    """Tokens of the bounded CPU sample: whole chunks of one filtered layer,
    two per host thread for the multi-threaded reference (every thread gets the
    same number of chunks, so the sample is not slowed by an idle tail), a
    4-chunk prefix for the single-threaded port."""
    cs = chunk_plan(cfg)[0][0]
    n = 2 * cores if kind == "reference" else 4
    return min(cfg["T"], n * cs)


def cpu_sample(fns, kind, cores, cfg, Kq_h, Vq_h, Q_h):
    """Time one kv_compact_quantized call of the reference CPU library (or the
    oracle port) on the first len(Kq_h) tokens of one filtered layer with
    `cores` OpenMP threads (params.n_threads set explicitly: under torchrun
    OMP_NUM_THREADS=1 would otherwise make the reference single-threaded).
    Returns (tokens/s of the whole model, details, seconds)."""
    H, d = cfg["H"], cfg["d"]
    tokens = Kq_h.shape[0]
    krb, vrb = Kq_h.shape[1], Vq_h.shape[1]
    p = abi.make_params(fns, target_ratio=cfg["ratio"], n_threads=cores if kind == "reference" else 1)
    r = abi.QuantResult()
    t0 = time.perf_counter()
    rc = fns["kv_compact_quantized"](abi.u8ptr(Kq_h), abi.u8ptr(Vq_h), abi.fptr(Q_h),
                                     cfg["ktype"], cfg["vtype"], krb, vrb, tokens, Q_h.shape[0], H, d, d,
                                     ctypes.byref(p), ctypes.byref(r))
    dt = time.perf_counter() - t0
    assert rc == 0, rc
    fns["quant_result_free"](ctypes.byref(r))
    n_layers = len(filtered_layers(cfg))
    value = tokens / (n_layers * dt)   # T tokens need n_layers layer-compactions
    n_chunks = -(-tokens // chunk_plan(cfg)[0][0])
    sample = (f"{tokens} tokens ({n_chunks} chunks) of 1 of {n_layers} filtered layers x {H} heads, "
              f"{TYPE_NAME[cfg['ktype']]}, {dt:.2f} s on {cores} threads; "
              f"model throughput = tokens / ({n_layers} x sample time)")
    return value, {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample}, dt


def reference_inputs(fns, cfg, tokens, seed):
    """One layer's first `tokens` rows with the workload's distributions,
    generated on the host (numpy) and quantised by `fns`' own kv_quantize_row."""
    rng = np.random.default_rng(seed)
    H, d = cfg["H"], cfg["d"]
    K = workloads.rope_keys(rng, tokens, H, d)
    V = rng.standard_normal((tokens, H * d)).astype(np.float32)
    Q = workloads.snapkv_queries(rng, H, d, cfg["window"], cfg["group"])
    return (abi.quantize_rows(fns, K, cfg["ktype"]), abi.quantize_rows(fns, V, cfg["vtype"]),
            np.ascontiguousarray(Q))


def run_reference(args, cfg, name):
    """The reference's own CPU library on the host cores: nothing of this
    repository's CUDA library is loaded in this process (inputs are generated
    with numpy and quantised by the reference's kv_quantize_row)."""
    rank, _, _ = kdist.env_ranks()
    if rank != 0:
        return
    cores = host_cores()
    os.environ["OMP_NUM_THREADS"] = str(cores)     # before the OpenMP runtime loads
    fns, kind = cpu_library()
    tokens = cpu_sample_tokens(cfg, kind, cores)
    Kh, Vh, Qh = reference_inputs(fns, cfg, tokens, 1000)
    times, vals, base = [], [], None
    for i in range(args.warmup + args.steps):
        v, base, dt = cpu_sample(fns, kind, cores, cfg, Kh, Vh, Qh)
        if i >= args.warmup:
            times.append(dt)
            vals.append(v)
    value = statistics.median(vals)
    base["value"] = value
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(times) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded numpy; cfg2 distributions quantised by the reference's kv_quantize_row)",
        "config": {"workload": workload_desc(name, cfg), "sample": base["sample"],
                   "threads": cores, "library": os.path.relpath(REF_PATH if kind == "reference" else ORACLE_PATH,
                                                                REPO)},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


# DRAM bytes per (layer, KV head) of 100k tokens measured by ncu for the
# kernels that can dominate a step (dram__bytes_read.sum + dram__bytes_write.sum
# of one launch over one cfg4 layer, divided by its 8 heads), from the capture
# summarised in profiles/main_kernels_cfg4_q8_1layer.md. Traffic grows in
# proportion to the layers of a launch, so a full-step launch is scaled by 12.
NCU_TRAFFIC_PER_LAYER_HEAD = {
    "k_score_tc": (113.8e6 + 358.3e6) / 8,
    "k_score": (410.2e6 + 366.6e6) / 8,
    "k_score_async": (410.2e6 + 366.6e6) / 8,
    "k_pv_tc": (538.6e6 + 33.0e6) / 8,
    "k_row_importance": (412.8e6 + 4.6e6) / 8,
    "k_lsq_factor": (123.2e6 + 43.4e6) / 8,
    "k_gather_softmax_x_reg": (409.7e6 + 69.3e6) / 8,
}


def chunk_plan(cfg):
    """(C, t) of every chunk of one layer, as the library plans them
    (auto chunk size 256 / ratio when more than 256 keys are kept)."""
    from kvc_b200 import shard
    return [(C, t) for _, C, t in shard.chunk_table(cfg["T"], cfg["ratio"])]


def measured_fp64_tflops(device):
    """cuBLAS DGEMM throughput on this GPU (4096^3, best of 3, CUDA events):
    the denominator of the fp64 tensor-core stages (MEASURED_PEAKS.json holds
    no fp64 figure)."""
    import torch
    n = 4096
    a = torch.randn((n, n), dtype=torch.float64, device=device)
    b = torch.randn((n, n), dtype=torch.float64, device=device)
    torch.matmul(a, b)
    best = None
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.matmul(a, b)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    del a, b
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def stage_rooflines(stage_times, cfg, n_steps, clocks, peaks, slices, fp64_tflops):
    """Roofline of every timed stage of this rank's step: algorithmic work per
    launch / measured average launch time, against the bound that applies.
    Work is counted over this rank's chunks (all of them at N=1)."""
    from kvc_b200 import shard
    H, d = cfg["H"], cfg["d"]
    nq = cfg["window"] * cfg["group"]
    table = shard.chunk_table(cfg["T"], cfg["ratio"])
    units = [(table[c][1], table[c][2]) for s in slices for c in range(s.c0, s.c1)]
    tokens = sum(C for C, _ in units)
    t = sum(tu for _, tu in units)
    hbm = peaks.get("hbm_gbs")
    hbm_src = "MEASURED_PEAKS.json hbm_gbs (of measured)"
    if hbm is None:
        hbm, hbm_src = 6650.0, "fallback 6.65 TB/s (of fallback)"
    hbm *= 1e9
    bf16 = peaks.get("bf16_tflops")
    bf16_src = "MEASURED_PEAKS.json bf16_tflops (burst, of measured)"
    if bf16 is None:
        bf16, bf16_src = 1590.0, "fallback 1.59 PFLOP/s (of fallback)"
    bf16 *= 1e12
    fp64 = fp64_tflops * 1e12
    fp64_src = "cuBLAS DGEMM 4096^3 measured in this run (MEASURED_PEAKS.json has no fp64 figure)"
    bpe = {abi.KV_TYPE_Q8_0: 34 / 32, abi.KV_TYPE_Q4_0: 18 / 32, abi.KV_TYPE_Q4_1: 20 / 32, abi.KV_TYPE_F16: 2.0}
    kb, vb = bpe[cfg["ktype"]], bpe[cfg["vtype"]]
    # a block-format V (Q8_0/Q4_0/Q4_1) is read as it is by the refit-target
    # kernel and never decoded; an F16 V is decoded to fp32 first
    v_blocks = cfg["vtype"] != abi.KV_TYPE_F16
    v_read = vb if v_blocks else 4.0
    # fp64 FMA of the LS refit per (unit, head): n = min(n_q, t_u) unknowns;
    # Gram n(n+1)/2 x k (k = t_u in the dual form, n_q in the primal), Cholesky n^3/3,
    # two triangular solves n^2 d, output t_u x d x n (dual) or right-hand side t_u x d x n_q (primal)
    gram = fac = outp = 0.0
    for _, tu in units:
        n = min(nq, tu)
        k = tu if nq < tu else nq
        gram += n * (n + 1) / 2 * k
        fac += n ** 3 / 3 + n * n * d
        outp += tu * d * (n if nq < tu else nq)
    per_h = lambda x: x * H                        # noqa: E731
    score_flops = 2.0 * nq * d * tokens * H
    model = {
        # K read in its block format once, S written once (fp32), row maxima
        "score": ("k_score_tc", "hbm", "GB/s", (kb * d + 4.0 * nq) * tokens * H + 4.0 * nq * H * len(units),
                  hbm, hbm_src),
        "refit_target": ("k_pv_tc", "hbm", "GB/s",
                         (4.0 * nq + v_read * d) * tokens * H + 4.0 * nq * d * H * len(units), hbm, hbm_src),
        # the scores are read (once, at least) and nothing of their size is written
        "softmax_importance": ("k_row_importance", "hbm", "GB/s", 4.0 * nq * tokens * H, hbm, hbm_src),
        # X = softmax(S[:, sel]): with a fifth of the keys kept, nearly every 32-byte
        # sector of S holds a kept score, so the bytes that must move are all of S
        # (read) and X (written)
        "x_build": ("k_gather_softmax_x_reg", "hbm", "GB/s", 4.0 * nq * (tokens + t) * H, hbm, hbm_src),
        "decode": ("k_decode_span", "hbm", "GB/s",
                   tokens * H * d * (kb + 4.0) + (0.0 if v_blocks else tokens * H * d * (vb + 4.0)), hbm, hbm_src),
        # K_out: kept K rows read and written in their stored format; V_out: C_v read (fp32), rows written
        "requant": ("k_transcode_rows_batch + k_encode_heads_batch", "hbm", "GB/s",
                    t * H * d * (2.0 * kb + 4.0 + vb), hbm, hbm_src),
        "ls_gram": ("k_dgemm (Gram)", "tensor", "TFLOP/s", 2.0 * per_h(gram), fp64, fp64_src),
        "ls_factor": ("k_lsq_factor", "tensor", "TFLOP/s", 2.0 * per_h(fac), fp64, fp64_src),
        "ls_out": ("k_dgemm (C_v = X^T Z)", "tensor", "TFLOP/s", 2.0 * per_h(outp), fp64, fp64_src),
    }
    out = {}
    for name, (ms, launches) in stage_times.items():
        if name not in model or not launches:
            continue
        kern, bound, unit, work, peak, src = model[name]
        launches_per_step = launches / max(n_steps, 1)
        per_launch_ms = ms / launches
        achieved = work / launches_per_step / (per_launch_ms * 1e-3)
        div = 1e9 if unit == "GB/s" else 1e12
        out[name] = {"kernel": kern, "bound": bound, "achieved": achieved / div, "peak": peak / div, "unit": unit,
                     "frac": achieved / peak, "ms_per_launch": per_launch_ms,
                     "launches_per_step": launches_per_step, "work_per_step": work, "peak_source": src}
        if name == "score":     # the contraction beside its memory roofline
            tf = score_flops / launches_per_step / (per_launch_ms * 1e-3)
            out[name]["tensor"] = {"achieved_tflops": tf / 1e12, "peak_tflops": bf16 / 1e12, "frac": tf / bf16,
                                   "peak_source": bf16_src,
                                   "note": "algorithmic 2*n_q*d flop per (key, head); executed: 2 fp16 pieces"}
    return out


def roofline_entry(stage_times, cfg, n_steps, clocks, peaks, slices, fp64_tflops):
    """Roofline of the stage with the largest device time per step."""
    rl = stage_rooflines(stage_times, cfg, n_steps, clocks, peaks, slices, fp64_tflops)
    if not rl:
        return None, rl
    name = max(rl, key=lambda k: stage_times[k][0])
    e = dict(rl[name])
    per_lh = NCU_TRAFFIC_PER_LAYER_HEAD.get(e["kernel"])
    n_layers_eq = sum(s.tokens for s in slices) / cfg["T"]
    e["traffic"] = None if per_lh is None else per_lh * cfg["H"] * n_layers_eq / e["launches_per_step"]
    e["traffic_unit"] = "bytes per launch (ncu DRAM read+write, scaled from a one-layer capture)"
    return e, rl


def run_kvc(args, cfg, name):
    import torch
    import torch.distributed as dist
    from kvc_b200 import lib, shard

    rank, world, local = kdist.env_ranks()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    kdist.init("nccl", device)
    fns = lib.load()
    T, H, d = cfg["T"], cfg["H"], cfg["d"]
    L = len(filtered_layers(cfg))
    replicas = args.replicas or world == 1
    # partition mode: every rank holds the same model (one seed) and compacts
    # its share of the (layer, chunk) units; replicas: one model per rank
    seed = kdist.rank_seed(1000, rank) if args.replicas else 1000
    Kq, Vq, Q = make_layers(cfg, seed, device, fns)
    cs = shard.auto_chunk(T, cfg["ratio"])
    params = abi.make_params(fns, target_ratio=cfg["ratio"], chunk_size=cs)
    gather = not replicas and world > 1
    peer = gather and args.gather in ("peer", "peer-copy")
    if replicas:
        plan = [shard.partition(L, T, cfg["ratio"], 1)[0] for _ in range(world)]
    else:
        # peer writes overlap rank 0's compute when rank 0 holds a larger share
        weights = shard.root_weights(world, args.root_extra) if peer else None
        plan = shard.partition(L, T, cfg["ratio"], world, weights)
    krb, vrb = Kq[0].shape[1], Vq[0].shape[1]
    finals, g = None, None
    if peer:
        g = shard.PeerGather(dist, fns, rank, world, plan, L, T, cfg["ratio"], H, krb, vrb, device,
                             copy_rows=args.gather == "peer-copy")
        finals = g.finals
    job = shard.SliceJob(fns, plan[rank], Kq, Vq, Q, T, H, d, cfg["ktype"], cfg["vtype"], params,
                         out_ptrs=g.out_ptrs() if peer else None)
    if gather and not peer:
        if rank == 0:
            t = shard.layer_kept(T, cfg["ratio"])
            finals = [{"sel": torch.empty(t, dtype=torch.int32, device=device),
                       "beta": torch.empty(H * t, dtype=torch.float32, device=device),
                       "kout": torch.empty(t * krb, dtype=torch.uint8, device=device),
                       "vout": torch.empty(t * vrb, dtype=torch.uint8, device=device)} for _ in range(L)]
        g = shard.Gather(dist, rank, world, plan, finals, H)

    def step():
        if g is None:
            job.run(want_stats=True)
            return
        g.begin()                      # previous step's transfers done; NCCL: receives posted
        outs = job.run(want_stats=True, gather=g)
        g.finish(outs)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    fp64_tflops = measured_fp64_tflops(device)
    lib.profile(fns, True)
    launches0 = fns["_lib"].kvc_launch_count()
    kdist.barrier(world)
    torch.cuda.synchronize()
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        uuid = str(local)
    sampler = ClockSampler(uuid)
    time.sleep(2.0)     # nvidia-smi's own start-up stays outside the timed region
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    launches = fns["_lib"].kvc_launch_count() - launches0
    stages = lib.profile(fns, False)
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = kdist.max_over_ranks(ms, world, device)
    kdist.barrier(world)
    # tokens of one step: every rank's own model (replicas) or the one model
    tokens_per_step = world * T if args.replicas else T
    value = tokens_per_step / (ms_max * 1e-3)

    # ---- the partitioned result checked against one GPU computing the whole
    # model (rank 0, after the timed region): kept indices, beta and the
    # requantised K/V rows must be identical bit for bit
    gather_check = None
    if gather and not args.no_check:
        if rank == 0:
            whole = shard.SliceJob(fns, shard.partition(L, T, cfg["ratio"], 1)[0], Kq, Vq, Q, T, H, d,
                                   cfg["ktype"], cfg["vtype"], params)
            whole.run(want_stats=False)
            ref = whole.outputs()
            torch.cuda.synchronize()
            bad = [l for l in range(L) for k in ("sel", "beta", "kout", "vout")
                   if not torch.equal(ref[l][k], finals[l][k])]
            gather_check = ("rank 0's whole-model arrays identical to one GPU's" if not bad
                            else f"MISMATCH in layers {sorted(set(bad))}")
            del whole, ref
        kdist.barrier(world)

    # ---- end to end through the drop-in C ABI: each rank's slices from
    # pinned host buffers (kv_compact_quantized per slice, results back in
    # its host memory), copies inside the timed region
    e2e = None
    if not args.no_e2e:
        need = sorted({s.layer for s in plan[rank]})
        Kh = {l: Kq[l].cpu().pin_memory() for l in need}
        Vh = {l: Vq[l].cpu().pin_memory() for l in need}
        Qh = {l: Q[l].cpu().pin_memory() for l in need}
        U8 = ctypes.POINTER(ctypes.c_uint8)
        FP = ctypes.POINTER(ctypes.c_float)

        def e2e_step():
            h2d = d2h = 0
            for s in plan[rank]:
                r = abi.QuantResult()
                kp = Kh[s.layer][s.tok0:s.tok1]
                vp = Vh[s.layer][s.tok0:s.tok1]
                rc = fns["kv_compact_quantized"](ctypes.cast(kp.data_ptr(), U8), ctypes.cast(vp.data_ptr(), U8),
                                                 ctypes.cast(Qh[s.layer].data_ptr(), FP), cfg["ktype"], cfg["vtype"],
                                                 krb, vrb, s.tokens, Qh[s.layer].shape[0], H, d, d,
                                                 ctypes.byref(params), ctypes.byref(r))
                assert rc == 0, rc
                t = r.base.t
                h2d += s.tokens * (krb + vrb) + Qh[s.layer].numel() * 4
                d2h += t * 4 + H * t * 4 + H * t * d * 4 + t * (krb + vrb)
                fns["quant_result_free"](ctypes.byref(r))
            return h2d, d2h

        e2e_step()
        n_e2e = max(1, min(args.steps, 3))
        kdist.barrier(world)
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(n_e2e):
            h2d, d2h = e2e_step()
        f1.record()
        torch.cuda.synchronize()
        e_ms = kdist.max_over_ranks(f0.elapsed_time(f1) / n_e2e, world, device)
        h2d = int(kdist.sum_over_ranks(h2d, world, device))
        d2h = int(kdist.sum_over_ranks(d2h, world, device))
        e2e = {"value": tokens_per_step / (e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms, "steps": n_e2e,
               "path": "kv_compact_quantized per slice (whole layers at N=1), pinned host inputs; "
                       "results land in each rank's host memory"}

    # ---- CPU baseline on the host cores (rank 0, N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cfns, kind = cpu_library()
        cores = host_cores() if kind == "reference" else 1
        n = cpu_sample_tokens(cfg, kind, cores)
        _, cpu, _ = cpu_sample(cfns, kind, cores, cfg, np.ascontiguousarray(Kq[0][:n].cpu().numpy()),
                               np.ascontiguousarray(Vq[0][:n].cpu().numpy()), Q[0].cpu().numpy())

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    roof, roof_all = roofline_entry(stages, cfg, args.steps, clocks, peaks, plan[rank], fp64_tflops)
    if rank == 0:
        units_r = [sum(s.c1 - s.c0 for s in pr) for pr in plan]
        if args.replicas:
            par = f"replicas x{world} (one cache per rank, no collective)"
        elif world == 1:
            par = "one GPU"
        else:
            rows = ("one copy-engine copy per slice and row array" if args.gather == "peer-copy"
                    else "requantisation kernels store K_out/V_out rows in place")
            how = (f"writes into rank 0's result buffer over NVLink (CUDA IPC: {rows}, one kernel places indices "
                   f"and beta), rank 0 weighted {shard.root_weights(world, args.root_extra)[0]:.2f}x"
                   if peer else "NCCL send/recv to rank 0")
            par = (f"(layer, chunk) partition x{world}: {units_r} units per rank; merge of the kept indices, "
                   f"beta and requantised K/V rows into rank 0's whole-model arrays inside the timed region by "
                   f"{how}, each batched call's slices sent as it returns (C_v stays on the rank that computed it)")
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "weak" if args.replicas else "strong",
            "vs_baseline": None, "dtype": "fp32 (scores: fp16-split operands on the tensor cores, fp32 accumulate)",
            "data": "synthetic (seeded; cfg2 distributions quantised)",
            "config": {"workload": workload_desc(name, cfg), "global_batch": 1 if not args.replicas else world,
                       "seq_len": T, "parallelism": par,
                       "l2": "inputs (2.6 GB) exceed L2; no flush needed"},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
            "clocks": clocks,
            **({"gather_check": gather_check} if gather_check else {}),
            "stage_ms_per_step": {k: round(v[0] / args.steps, 3) for k, v in stages.items() if v[1]},
            "stage_roofline": {k: {"kernel": v["kernel"], "bound": v["bound"], "frac": round(v["frac"], 3),
                                   "achieved": round(v["achieved"], 2), "unit": v["unit"]}
                               for k, v in roof_all.items()},
        }
        print(json.dumps(line))
    del job, finals
    if peer:
        g.close()
    kdist.finish(world)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="kvc", choices=["kvc", "reference"])
    ap.add_argument("--config", default="cfg4_q8", choices=sorted(CONFIGS))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--replicas", action="store_true",
                    help="N>1: every rank compacts its own model (weak scaling) instead of a share of one model")
    ap.add_argument("--gather", default="peer", choices=["peer", "peer-copy", "nccl"],
                    help="N>1 partition: merge into rank 0's buffer by the requantisation kernels' stores "
                         "(peer) or by one copy-engine copy per slice and row array (peer-copy), or NCCL send/recv")
    ap.add_argument("--root-extra", type=float, default=0.03,
                    help="peer merge: rank 0's share is 1 + extra*(N-1) times another rank's")
    ap.add_argument("--no-check", action="store_true",
                    help="N>1 partition: skip comparing rank 0's gathered result with one GPU's")
    ap.add_argument("--layers", type=int, default=0,
                    help="compact only the first N filtered layers (small cases for profiling)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.layers > 0:
        cfg["max_layers"] = args.layers
    if args.impl == "reference":
        run_reference(args, cfg, args.config)
    else:
        run_kvc(args, cfg, args.config)


if __name__ == "__main__":
    main()
