"""A rank that leaves between steps, noticed on the host (2 GPUs, NCCL).

Two ranks run data-parallel block lenses (forward, backward, NCCL
all-reduce of the parameter adjoint) with NVLS off.  After step 0, rank 1
finishes its device work (stream synchronised: none of its kernels or
collectives in flight) and exits without announcing step 1.  Rank 0 runs
step 1's local forward and backward, announces the step, and checks before
the step's all-reduce that every rank announced it (`dop.parallel.heartbeat`
/ `peers_alive` on the process group's store).  The check must fail within
its limit, the all-reduce must never be launched, and rank 0's GPU must
still run a block afterwards.  The crate's counterpart is the control
plane's member timeout (src/dist.rs:36-56).
"""
import os
import socket
import time
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, port: int, q) -> None:
    import datetime

    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(WORLD), NCCL_NVLS_ENABLE="0")
        from dop import DOP_BF16, lib, parallel
        from dop.mixtral import Block, MixtralConfig, layer_layout
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=30), device_id=dev)
        cfg = MixtralConfig(vocab=64, dim=256, layers=1, heads=4, kv_heads=2, head_dim=128,
                            intermediate=256, experts=8, top_k=2, rms_eps=1e-5, rope_theta=1e4,
                            sliding_window=96)
        batch, seq = 2, 128
        ll = layer_layout(cfg)
        g = torch.Generator(device=dev).manual_seed(3)
        P = (torch.randn(ll.total, generator=g, device=dev) * 0.05).bfloat16()
        blk = Block(cfg, batch, seq, DOP_BF16)
        X = torch.randn(batch * seq, cfg.dim, generator=g, device=dev)
        DY = torch.randn(batch * seq, cfg.dim, generator=g, device=dev)
        dP = torch.zeros(ll.total, device=dev)

        def local_step():
            dP.zero_()
            blk.forward(P, X)
            blk.backward(P, DY, dP)

        # step 0: everybody
        local_step()
        parallel.heartbeat(0)
        assert parallel.peers_alive(0, timeout_s=20.0)
        parallel.reduce_adjoint(dP)
        torch.cuda.synchronize(dev)
        if rank == 1:
            # leave between steps: nothing of this rank is in flight
            torch.cuda.synchronize(dev)
            q.put((rank, True, "left after step 0"))
            q.close()
            q.join_thread()
            os._exit(0)
        # step 1 on rank 0: local work, then the check before the collective
        local_step()
        torch.cuda.synchronize(dev)
        parallel.heartbeat(1)
        t0 = time.perf_counter()
        alive = parallel.peers_alive(1, timeout_s=2.0)
        waited = time.perf_counter() - t0
        assert not alive, "the rank that left was reported alive"
        assert waited < 10.0, f"detection took {waited:.1f} s"
        # the all-reduce of step 1 is not launched; the GPU still works
        local_step()
        torch.cuda.synchronize(dev)
        assert torch.isfinite(dP).all()
        assert lib().dop_device_status() == 0
        q.put((rank, True, f"detected after {waited:.2f} s"))
        q.close()
        q.join_thread()
        # skip the NCCL teardown with a peer gone
        os._exit(0)
    except Exception:
        q.put((rank, False, traceback.format_exc()))
        q.close()
        q.join_thread()
        os._exit(1)


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_rank_that_leaves_between_steps_is_noticed_before_the_next_collective():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            r, ok, msg = q.get(timeout=240)
            results[r] = (ok, msg)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert results[1][0] and results[0][0], results
