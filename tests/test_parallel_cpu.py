"""The multi-rank host logic on CPU: two gloo ranks (no GPU).

Covers the data-parallel adjoint reduction and the max-over-ranks step time
that bench.py uses, and host-side failure detection: a rank that dies before
a collective makes the survivor's collective end with an error within the
process group's timeout instead of hanging.
"""
import multiprocessing as mp
import os
import socket
import traceback

import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world))
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, os.path.join(root, "dependent-optics_b200"))
        import torch
        import torch.distributed as dist
        from dop import parallel
        timeout = 60.0
        parallel.init_from_env("gloo", timeout_s=timeout)
        if mode == "reduce":
            n = 1000
            dP = torch.arange(n, dtype=torch.float32) * (rank + 1)
            parallel.reduce_adjoint(dP, bucket=128)  # 8 buckets, last one ragged
            expect = torch.arange(n, dtype=torch.float32) * sum(r + 1 for r in range(world))
            ok = torch.equal(dP, expect)
            works = parallel.reduce_adjoint(torch.ones(300), bucket=100, async_op=True)
            for w in works:
                w.wait()
            t = parallel.max_over_ranks(10.0 + rank)
            q.put((rank, ok and len(works) == 3 and t == 10.0 + world - 1, ""))
        elif mode == "dead_rank":
            # step 0 completes on both ranks; rank 1 leaves between steps
            parallel.heartbeat(0)
            both = parallel.peers_alive(0, timeout_s=20.0)
            parallel.reduce_adjoint(torch.ones(16))
            if rank == 1:
                q.put((rank, both, "leaving after step 0"))
                q.close()
                q.join_thread()  # flush before leaving without cleanup
                os._exit(0)
            parallel.heartbeat(1)
            alive = parallel.peers_alive(1, timeout_s=3.0)  # noticed on the host
            q.put((rank, both and not alive, f"peers alive at step 1: {alive}"))
            q.close()
            q.join_thread()
            os._exit(0)
        if dist.is_initialized() and mode != "dead_rank":
            dist.destroy_process_group()
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, ok, msg = q.get(timeout=timeout)
        results[r] = (ok, msg)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


def test_adjoint_reduction_and_max_over_ranks_gloo():
    res = _run("reduce")
    assert all(ok for ok, _ in res.values()), res


def test_rank_that_leaves_is_detected_on_the_host():
    res = _run("dead_rank")
    assert res[1][0] and res[0][0], res


def test_buckets_cover_the_adjoint():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "dependent-optics_b200"))
    from dop.parallel import adjoint_buckets
    assert adjoint_buckets(10, 4) == [(0, 4), (4, 8), (8, 10)]
    assert adjoint_buckets(0, 4) == []
    with pytest.raises(AssertionError):
        adjoint_buckets(5, 0)
