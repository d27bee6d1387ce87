"""Multi-process plumbing of the benchmark: one process per GPU.

The compaction path has no exchange step: every (layer, chunk) unit is
independent. N ranks either share one model's units (kvc_b200.shard: a
partition plus a final gather of the compacted rows to rank 0) or each
compact their own cache (weak scaling); the other collectives are a barrier
before timing and the maximum of the per-rank step times afterwards. These helpers hold that logic so it can be exercised on
CPU with the gloo backend (tests/test_dist_cpu.py) and on GPUs with NCCL
(bench.py under torchrun).
"""
import datetime
import os


def env_ranks():
    """(rank, world_size, local_rank) from the torchrun environment (1 process: 0, 1, 0)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend, device=None, timeout_s=300):
    """Join the process group when there is more than one rank; returns (rank, world)."""
    import torch.distributed as dist
    rank, world, _ = env_ranks()
    # keep stdout to the benchmark's single JSON line (NCCL would add its version banner)
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    if world > 1 and not dist.is_initialized():
        kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if device is not None and backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(backend, **kw)
    return rank, world


def barrier(world):
    import torch.distributed as dist
    if world > 1:
        dist.barrier()


def max_over_ranks(value, world, device="cpu"):
    """The maximum of a per-rank float over all ranks (the job's step time)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, world, device="cpu"):
    """The sum of a per-rank number over all ranks."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def rank_seed(base, rank):
    """Each rank compacts a different synthetic cache."""
    return int(base) + int(rank)


def job_tokens_per_s(world, tokens_per_rank, ms_per_step):
    """Whole-job throughput: every rank's tokens over the slowest rank's step time."""
    return world * tokens_per_rank / (ms_per_step * 1e-3)


def finish(world):
    import torch.distributed as dist
    if world > 1 and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
