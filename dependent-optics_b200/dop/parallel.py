"""Multi-GPU plumbing for the block lens: one process per GPU, NCCL through
torch.distributed.

Data parallelism over the batch: every rank runs the block lens on its own
batch with the same parameters, then the ranks sum their parameter adjoints
(`reduce_adjoint`).  Expert parallelism: every rank still runs attention
and the router on its own batch, but owns E / world experts and runs them
for every rank's tokens (the exchange is inside the block, over CUDA IPC
mappings set up by `connect_expert_parallel`); only the shared slice of the
adjoint (before the first expert) is summed over ranks.  The crate has no parallel execution (its cluster plan
runs windows one at a time, src/dist.rs:243-275); this is the exchange the
data-parallel workloads need.
"""
from __future__ import annotations

import datetime
import os


def init_from_env(backend: str = "nccl", timeout_s: float = 600.0, device=None):
    """Join the process group torchrun describes (RANK, WORLD_SIZE,
    MASTER_ADDR, MASTER_PORT) with a bounded collective timeout."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and not dist.is_initialized():
        kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if device is not None and backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(backend, **kw)
    return world, int(os.environ.get("RANK", "0"))


def max_over_ranks(value: float, device=None) -> float:
    """Largest value over all ranks (a step's time is the slowest rank's)."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def adjoint_buckets(n: int, bucket: int) -> list:
    """Contiguous [start, stop) ranges covering n elements, each <= bucket."""
    assert n >= 0 and bucket > 0
    return [(a, min(n, a + bucket)) for a in range(0, n, bucket)]


def reduce_adjoint(dparams, bucket: int = 1 << 28, async_op: bool = False):
    """Sum the parameter adjoint over the data-parallel ranks in place, in
    buckets of at most `bucket` elements (each bucket is one all-reduce, so a
    caller may start the early buckets while later gradients are still being
    produced).  Returns the list of work handles when async_op."""
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return []
    flat = dparams.view(-1)
    works = []
    for a, b in adjoint_buckets(flat.numel(), bucket):
        w = dist.all_reduce(flat[a:b], async_op=async_op)
        if async_op:
            works.append(w)
    return works


def ep_mode(world: int, experts: int, bf16: bool) -> bool:
    """Whether a block of `experts` experts runs expert-parallel on `world`
    ranks: bf16, more than one rank, and the experts split evenly."""
    return bf16 and 1 < world <= 8 and experts % world == 0


def connect_expert_parallel(block, device=None) -> None:
    """All-gather every rank's workspace IPC handle over the process group
    and map the peers' workspaces into `block` (an expert-parallel
    dop.mixtral.Block).  Every rank calls it once, before the first
    forward."""
    import torch
    import torch.distributed as dist
    h = block.ep_handle()
    world = dist.get_world_size()
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    mine = torch.tensor(list(h), dtype=torch.uint8, device=dev)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    block.ep_connect(b"".join(bytes(t.cpu().tolist()) for t in every))


def heartbeat(step: int) -> None:
    """Announce on the process group's store that this rank reached `step`."""
    import torch.distributed as dist
    if not dist.is_initialized():
        return
    store = dist.distributed_c10d._get_default_store()
    store.set(f"dop/alive/{dist.get_rank()}/{step}", "1")


def peers_alive(step: int, timeout_s: float = 5.0) -> bool:
    """True when every rank announced `step` within timeout_s.  Ranks call it
    between steps, before launching the next step's kernels and collectives,
    so a rank that left is noticed on the host instead of inside a
    collective."""
    import datetime
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return True
    store = dist.distributed_c10d._get_default_store()
    keys = [f"dop/alive/{r}/{step}" for r in range(dist.get_world_size())]
    try:
        store.wait(keys, datetime.timedelta(seconds=timeout_s))
        return True
    except Exception:
        return False
