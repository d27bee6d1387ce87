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

Multi-GPU (torchrun): every rank compacts its own independent cache
(different seed), no collective on the data path; value = all tokens of
all ranks / max-over-ranks time ("weak" scaling).

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

from kvc_b200 import ORACLE_PATH, REF_PATH, abi, workloads  # noqa: E402

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


def cpu_sample(cfg, Kq_h, Vq_h, Q_h, max_seconds=30.0):
    """Time the reference CPU library (or the oracle port) on one filtered
    layer; returns (tokens/s of the whole model extrapolated, details)."""
    T, H, d = cfg["T"], cfg["H"], cfg["d"]
    if os.path.exists(REF_PATH):
        fns = abi.bind(ctypes.CDLL(REF_PATH, mode=ctypes.RTLD_LOCAL))
        kind, cores = "reference", len(os.sched_getaffinity(0))
        tokens = T
    else:
        fns = abi.bind(ctypes.CDLL(ORACLE_PATH, mode=ctypes.RTLD_LOCAL), prefix="oracle_")
        kind, cores = "port", 1
        tokens = min(T, 20 * 1280)   # the single-threaded port: a 20-chunk prefix
    krb, vrb = Kq_h.shape[1], Vq_h.shape[1]
    p = abi.make_params(fns, target_ratio=cfg["ratio"])
    r = abi.QuantResult()
    t0 = time.perf_counter()
    rc = fns["kv_compact_quantized"](abi.u8ptr(np.ascontiguousarray(Kq_h[:tokens])),
                                     abi.u8ptr(np.ascontiguousarray(Vq_h[:tokens])), abi.fptr(Q_h),
                                     cfg["ktype"], cfg["vtype"], krb, vrb, tokens, Q_h.shape[0], H, d, d,
                                     ctypes.byref(p), ctypes.byref(r))
    dt = time.perf_counter() - t0
    assert rc == 0, rc
    fns["quant_result_free"](ctypes.byref(r))
    n_layers = len(filtered_layers(cfg))
    value = tokens / (n_layers * dt)   # T tokens need n_layers layer-compactions
    sample = (f"1 of {n_layers} filtered layers, {tokens} tokens x {H} heads, {TYPE_NAME[cfg['ktype']]}, "
              f"{dt:.2f} s; model throughput = tokens / ({n_layers} x layer time)")
    return value, {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample}, dt


def run_reference(args, cfg, name):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    device = "cuda:0" if torch.cuda.is_available() else "cpu"
    from kvc_b200 import lib
    fns = lib.load()
    if device == "cpu":
        print(json.dumps({"impl": "reference", "unavailable": "data generation needs the CUDA device"}))
        return
    Kq, Vq, Q = make_layers(cfg, 1000, device, fns)
    Kh, Vh, Qh = Kq[0].cpu().numpy(), Vq[0].cpu().numpy(), Q[0].cpu().numpy()
    del Kq, Vq, Q
    torch.cuda.empty_cache()
    times, vals, base = [], [], None
    for i in range(args.warmup + args.steps):
        v, base, dt = cpu_sample(cfg, Kh, Vh, Qh)
        if i >= args.warmup:
            times.append(dt)
            vals.append(v)
    value = statistics.median(vals)
    base["value"] = value
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(times) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded; cfg2 distributions quantised)",
        "config": {"workload": workload_desc(name, cfg), "sample": base["sample"]},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def roofline_entry(stage_times, cfg, n_steps, clocks, peaks):
    """Roofline of the stage with the largest device time."""
    T, H, d = cfg["T"], cfg["H"], cfg["d"]
    L = len(filtered_layers(cfg))
    nq = cfg["window"] * cfg["group"]
    tokens = T * L
    name, (ms, launches) = max(stage_times.items(), key=lambda kv: kv[1][0])
    per_launch_ms = ms / max(launches, 1)
    launches_per_step = launches / max(n_steps, 1)
    sm_max = (clocks.get("sm_max_mhz") or 1965.0) * 1e6
    fp32_issue = 148 * 128 * sm_max            # fp32 instructions/s (one flop each without FMA)
    if name == "score":
        # 2*n_q*d flops per (token, head): separate multiply and add per term
        work = 2.0 * nq * d * tokens * H / launches_per_step
        return {"kernel": "k_score", "bound": "fp32_simt", "achieved": work / (per_launch_ms * 1e-3) / 1e12,
                "peak": fp32_issue / 1e12, "unit": "TFLOP/s",
                "peak_source": "derived: 148 SMs x 128 FP32 lanes x max SM clock, no-FMA issue rate "
                               "(MEASURED_PEAKS.json has no FP32 figure)",
                "frac": (work / (per_launch_ms * 1e-3)) / fp32_issue, "traffic": None,
                "ms_per_launch": per_launch_ms}
    if name == "refit_target":
        work = 2.0 * nq * d * tokens * H / launches_per_step
        peak = 2 * fp32_issue
        return {"kernel": "k_pv", "bound": "fp32_simt", "achieved": work / (per_launch_ms * 1e-3) / 1e12,
                "peak": peak / 1e12, "unit": "TFLOP/s", "peak_source": "derived FP32 FMA peak",
                "frac": work / (per_launch_ms * 1e-3) / peak, "traffic": None, "ms_per_launch": per_launch_ms}
    hbm = peaks.get("hbm_gbs", 6650.0)
    return {"kernel": name, "bound": "unclassified", "achieved": None, "peak": hbm, "unit": "GB/s",
            "frac": None, "traffic": None, "ms_per_launch": per_launch_ms}


def run_kvc(args, cfg, name):
    import torch
    import torch.distributed as dist
    from kvc_b200 import lib

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    fns = lib.load()
    T, H, d = cfg["T"], cfg["H"], cfg["d"]
    Kq, Vq, Q = make_layers(cfg, 1000 + rank, device, fns)
    params = abi.make_params(fns, target_ratio=cfg["ratio"])
    model = lib.BatchedModel(fns, Kq, Vq, Q, T, H, d, d, cfg["ktype"], cfg["vtype"], params)
    for _ in range(args.warmup):
        model.run(want_stats=True)
    torch.cuda.synchronize()
    lib.profile(fns, True)
    launches0 = fns["_lib"].kvc_launch_count()
    if world > 1:
        dist.barrier()
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
        model.run(want_stats=True)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    launches = fns["_lib"].kvc_launch_count() - launches0
    stages = lib.profile(fns, False)
    ms = e0.elapsed_time(e1) / args.steps
    t_max = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        dist.barrier()
    ms_max = float(t_max.item())
    value = world * T / (ms_max * 1e-3)

    # ---- end to end through the drop-in C ABI, host buffers, copies timed
    e2e = None
    if not args.no_e2e:
        Kh = [k.cpu().pin_memory() for k in Kq]
        Vh = [v.cpu().pin_memory() for v in Vq]
        Qh = [q.cpu().pin_memory() for q in Q]
        krb, vrb = Kh[0].shape[1], Vh[0].shape[1]
        U8 = ctypes.POINTER(ctypes.c_uint8)
        FP = ctypes.POINTER(ctypes.c_float)

        def e2e_step():
            h2d = d2h = 0
            for l in range(len(Kh)):
                r = abi.QuantResult()
                rc = fns["kv_compact_quantized"](ctypes.cast(Kh[l].data_ptr(), U8), ctypes.cast(Vh[l].data_ptr(), U8),
                                                 ctypes.cast(Qh[l].data_ptr(), FP), cfg["ktype"], cfg["vtype"],
                                                 krb, vrb, T, Qh[l].shape[0], H, d, d, ctypes.byref(params),
                                                 ctypes.byref(r))
                assert rc == 0, rc
                t = r.base.t
                h2d += T * (krb + vrb) + Qh[l].numel() * 4
                d2h += t * 4 + H * t * 4 + H * t * d * 4 + t * (krb + vrb)
                fns["quant_result_free"](ctypes.byref(r))
            return h2d, d2h

        e2e_step()
        n_e2e = max(1, min(args.steps, 3))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(n_e2e):
            h2d, d2h = e2e_step()
        f1.record()
        torch.cuda.synchronize()
        e_ms = f0.elapsed_time(f1) / n_e2e
        te = torch.tensor([e_ms], device=device)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": world * T / (float(te.item()) * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": float(te.item()), "steps": n_e2e,
               "path": "kv_compact_quantized per filtered layer, pinned host inputs"}

    # ---- CPU baseline on the host cores (rank 0, N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        _, cpu, _ = cpu_sample(cfg, Kq[0].cpu().numpy(), Vq[0].cpu().numpy(), Q[0].cpu().numpy())

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    roof = roofline_entry(stages, cfg, args.steps, clocks, peaks)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded per rank; cfg2 distributions quantised)",
            "config": {"workload": workload_desc(name, cfg), "global_batch": world, "seq_len": T,
                       "parallelism": f"replicas x{world} (one cache per rank, no collective)",
                       "l2": "inputs (2.6 GB per rank) exceed L2; no flush needed"},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
            "clocks": clocks,
            "stage_ms_per_step": {k: round(v[0] / args.steps, 3) for k, v in stages.items() if v[1]},
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="kvc", choices=["kvc", "reference"])
    ap.add_argument("--config", default="cfg4_q8", choices=sorted(CONFIGS))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
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
