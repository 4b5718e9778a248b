"""The staging plan (src/cluster.rs vocabulary) and its executor, on CPU.

Plan tests: every (layer, micro-batch, pass) is scheduled once per replica;
each device runs a one-forward-one-backward program whose forwards precede
their backwards; every hop is produced before it is consumed; the StageError
cases (no GPU, parameters or residuals too large, no route) raise their
codes; derive_links and route_message follow src/cluster.rs:307-398;
StagePlan::check accepts the plan for the model's parameter count only.

Executor tests: gloo ranks run a plan of a 4-layer stack whose blocks are
stand-in linear lenses (y = x W, dx = dy W^T, dW += x^T dy) with one lens
object per residual slot, so a wrong slot assignment would mix two
micro-batches' residuals; outputs, input gradients and the replicas'
reduced adjoints must equal a single-process run, and each rank's recorded
events must equal the plan's trace projected on that rank.
"""
import multiprocessing as mp
import os
import socket
import traceback

import pytest

from dop import DOP_F32, DopError
from dop import cluster
from dop.mixtral import MixtralConfig, layer_layout


def small_cfg(layers=4):
    return MixtralConfig(vocab=64, dim=32, layers=layers, heads=4, kv_heads=2, head_dim=8,
                         intermediate=64, experts=4, top_k=2, rms_eps=1e-5, rope_theta=1e4,
                         sliding_window=16)


def big_cfg(layers=4):
    return MixtralConfig(vocab=32000, dim=4096, layers=layers, heads=32, kv_heads=8, head_dim=128,
                         intermediate=14336, experts=8, top_k=2, rms_eps=1e-5, rope_theta=1e6,
                         sliding_window=4096)


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_plan_schedules_every_window_once_in_order(n):
    cfg = big_cfg()
    plan = cluster.stage_mixtral(cfg, 32, 4096, 8, 1, cluster.b200s(n))
    pp = max(p for p in range(1, min(4, n) + 1) if 4 % p == 0 and n % p == 0)
    dp = n // pp
    blocks = [w for w in plan.windows if w.exec == cluster.EXEC_BLOCK]
    keys = [(w.replica, w.layer, w.micro, w.pass_) for w in blocks]
    assert len(keys) == len(set(keys)) == 4 * 8 * 2
    assert {w.micro % dp == w.replica for w in blocks} == {True}
    pos = {k: i for i, k in enumerate(keys)}
    for (r, l, m, ps), i in pos.items():
        if ps == 1:
            assert pos[(r, l, m, 0)] < i          # forward before backward
            if l < 3:
                assert pos[(r, l + 1, m, 1)] < i  # backward runs from the top layer down
        elif l > 0:
            assert pos[(r, l - 1, m, 0)] < i
    # each hop is sent (outbound of its producer) before it is received
    produced = {}
    for i, w in enumerate(plan.windows):
        for h in w.outbound:
            produced[h.index] = i
        for h in w.inbound:
            if h.kind != cluster.HOP_ADJOINT or w.exec == cluster.EXEC_BLOCK:
                assert produced[h.index] < i
    # stage s holds min(pp - s, micro-batches of its replica) residual slots per block
    for d in range(n):
        s = d % pp
        assert set(plan.slots(d).values()) == {min(pp - s, 8 // dp)}
    assert len(plan.stage_groups()) == pp and all(len(g) == dp for g in plan.stage_groups())
    plan.check(4 * layer_layout(cfg).total)
    with pytest.raises(DopError):
        plan.check(4 * layer_layout(cfg).total + 1)
    trace = plan.trace()
    assert trace[0] == f"MEMBERS {n}" and trace[-1] == "DONE"
    assert sum(line.startswith("COMPUTE") for line in trace) == len(plan.windows)


def test_stage_errors():
    cfg = big_cfg()
    with pytest.raises(DopError, match="NO_DEVICE"):
        cluster.stage_mixtral(cfg, 32, 4096, 8, 1, [cluster.Device("cpu0", cluster.DEVICE_CPU)])
    with pytest.raises(DopError, match="PARAMS_EXCEED_CLUSTER"):
        cluster.stage_mixtral(cfg, 32, 4096, 8, 1, cluster.b200s(2, buffer_bytes=8 * 10**9))
    with pytest.raises(DopError, match="TILE_EXCEEDS_DEVICES"):
        cluster.stage_mixtral(cfg, 32, 4096, 8, 1, cluster.b200s(8, buffer_bytes=15 * 10**9))
    with pytest.raises(DopError, match="TAPE_EXCEEDS_CLUSTER"):
        cluster.stage_mixtral(cfg, 32, 4096, 8, 1, cluster.b200s(4, buffer_bytes=40 * 10**9))
    # GPUs 0 and 1 share no link and no intermediate device can carry the message
    with pytest.raises(DopError, match="ROUTE_UNAVAILABLE"):
        cluster.stage_mixtral(cfg, 32, 4096, 8, 1, cluster.b200s(2), links=[(0, 0)])


def test_links_and_routes():
    devs = [cluster.Device("cpu0", cluster.DEVICE_CPU), cluster.Device("cpu1", cluster.DEVICE_CPU)] + \
        [cluster.Device(f"g{i}") for i in range(4)]
    links = set(cluster.derive_links(devs))
    # CPUs form a fabric; GPU i attaches to CPU i mod 2 and peers the GPUs on that CPU
    assert links == {(0, 1), (2, 0), (3, 1), (4, 0), (5, 1), (2, 4), (3, 5)}
    assert set(cluster.derive_links(cluster.b200s(3))) == {(0, 1), (0, 2), (1, 2)}
    free = [100] * 6
    assert cluster.route_message(sorted(links), free, 2, 5, 50) == [2, 0, 1, 5]
    free[0] = 10  # the message does not fit through CPU 0
    with pytest.raises(DopError, match="ROUTE_UNAVAILABLE"):
        cluster.route_message(sorted(links), free, 2, 5, 50)
    assert cluster.route_message(sorted(links), free, 2, 4, 50) == [2, 4]


def test_p2p_order_covers_every_message_hop_once():
    """Every hop of every block message appears once, under its own (src,
    dst) pair; a message's first hop follows its producer's position and its
    relayed hops follow the consumer's, in route order."""
    plan = cluster.stage_mixtral(small_cfg(4), 8, 6, 8, DOP_F32, cluster.b200s(4),
                                 links=[(0, 2), (2, 1), (1, 3), (3, 0)])
    order = plan.p2p_order()
    listed = [h.index for hops in order.values() for h in hops]
    msg_hops = [h.index for w in plan.windows if w.exec == cluster.EXEC_BLOCK for h in w.inbound]
    assert sorted(listed) == sorted(msg_hops) and len(set(listed)) == len(listed)
    for (a, b), hops in order.items():
        assert all((h.src, h.dst) == (a, b) for h in hops)
    # every message hop follows a link (src/cluster.rs:2174-2230, hops_follow_links)
    ring = {frozenset(l) for l in [(0, 2), (2, 1), (1, 3), (3, 0)]}
    assert all(frozenset((h.src, h.dst)) in ring for hops in order.values() for h in hops)
    pos = {}
    produced = {w.outbound[0].index: w.index for w in plan.windows
                if w.exec == cluster.EXEC_BLOCK and w.outbound}
    for w in plan.windows:
        if w.exec == cluster.EXEC_BLOCK and w.inbound:
            pos[w.inbound[0].index] = (produced[w.inbound[0].index], 0)
            for i, h in enumerate(w.inbound[1:], 1):
                pos[h.index] = (w.index, i)
    for hops in order.values():
        keys = [pos[h.index] for h in hops]
        assert keys == sorted(keys)
    # fully connected B200s: every message is one hop
    dense = cluster.stage_mixtral(small_cfg(4), 8, 6, 8, DOP_F32, cluster.b200s(4))
    assert all(len(w.inbound) <= 1 for w in dense.windows if w.exec == cluster.EXEC_BLOCK)


def test_executor_needs_one_process_per_device():
    plan = cluster.stage_mixtral(small_cfg(4), 8, 6, 8, DOP_F32, cluster.b200s(2))
    with pytest.raises(ValueError, match="one process per device"):
        cluster.run_plan(plan, 0, None, {}, {}, {}, {}, None)


# ------------------------------------------------------------ executor
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


ROWS, MICRO = 6, 8


class LinearLens:
    def forward(self, W, x):
        self.x = x
        return x @ W

    def backward(self, W, dy, dW):
        dW += self.x.T @ dy
        return dy @ W.T


def _data(LAYERS):
    import torch
    g = torch.Generator().manual_seed(3)
    D = small_cfg().dim
    Ws = [torch.randn(D, D, generator=g) / D ** 0.5 for _ in range(LAYERS)]
    xs = [torch.randn(ROWS, D, generator=g) for _ in range(MICRO)]
    dys = [torch.randn(ROWS, D, generator=g) for _ in range(MICRO)]
    return Ws, xs, dys


def _reference(LAYERS):
    import torch
    Ws, xs, dys = _data(LAYERS)
    dWs = [torch.zeros_like(W) for W in Ws]
    ys, dxs = {}, {}
    for m in range(MICRO):
        lenses = [LinearLens() for _ in range(LAYERS)]
        h = xs[m]
        for l in range(LAYERS):
            h = lenses[l].forward(Ws[l], h)
        ys[m] = h
        g = dys[m]
        for l in reversed(range(LAYERS)):
            g = lenses[l].backward(Ws[l], g, dWs[l])
        dxs[m] = g
    return ys, dxs, dWs


def _worker(rank, world, LAYERS, port, q, links=None):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world))
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, os.path.join(root, "dependent-optics_b200"))
        import torch
        import torch.distributed as dist
        from dop import cluster as cl
        from dop import parallel
        parallel.init_from_env("gloo", timeout_s=60.0)
        cfg = small_cfg(LAYERS)
        # ROWS rows per micro-batch: micro-batches of one sequence of ROWS tokens
        plan = cl.stage_mixtral(cfg, MICRO, ROWS, MICRO, DOP_F32, cl.b200s(world), links=links)
        groups = {tuple(g): dist.new_group(g) for g in plan.stage_groups()}
        Ws, xs, dys = _data(LAYERS)
        mine = {h.layer for h in plan.homes if h.device == rank and h.kind == cl.HOME_PARAM}
        dWs = {l: torch.zeros_like(Ws[l]) for l in mine}
        lenses = {}

        def lens_for(layer, slot):
            return lenses.setdefault((layer, slot), LinearLens())

        out = cl.run_plan(plan, rank, lens_for, Ws, dWs, xs, dys,
                          lambda r, c: torch.empty(r, c), groups=groups)
        ys, dxs, ref_dW = _reference(LAYERS)
        ok = all(torch.allclose(out["outputs"][m], ys[m], atol=1e-5) for m in out["outputs"])
        ok &= all(torch.allclose(out["input_grads"][m], dxs[m], atol=1e-5)
                  for m in out["input_grads"])
        ok &= all(torch.allclose(dWs[l], ref_dW[l], atol=1e-4) for l in mine)
        ok &= out["trace"] == plan.rank_trace(rank)
        n_out = len(out["outputs"]) + len(out["input_grads"])
        q.put((rank, ok, n_out, ""))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, False, 0, traceback.format_exc()))


# sparse links: messages between stages that share no link are relayed
RING3 = [(0, 2), (1, 2)]
RING4 = [(0, 2), (2, 1), (1, 3), (3, 0)]


@pytest.mark.parametrize("world,layers,links", [(2, 4, None), (4, 2, None), (3, 3, RING3),
                                                (4, 4, RING4)],
                         ids=["pp2", "pp2xdp2", "pp3-relay", "pp4-relays"])
def test_executor_matches_single_process(world, layers, links):
    """2 ranks x 4 layers: PP 2, two blocks chained on each GPU; 4 ranks x 2
    layers: PP 2 x DP 2, replicas' adjoints summed by the Sgd windows.  With
    sparse links the planner routes messages through intermediate devices
    (in the 3-rank case stage 2 relays between stages 0 and 1 while running
    its own blocks; in the 4-rank ring relayed and direct messages share
    pairs of ranks), and the executor's relays forward them: the crate's
    bridge test (src/dist.rs:1008-1053) in this executor's terms, where each
    hop of a route is one message, sent once and received once."""
    if links:
        plan = cluster.stage_mixtral(small_cfg(layers), MICRO, ROWS, MICRO, DOP_F32,
                                     cluster.b200s(world), links=links)
        assert any(len(w.inbound) > 1 for w in plan.windows if w.exec == cluster.EXEC_BLOCK)
        n_hops = sum(len(w.inbound) for w in plan.windows if w.exec == cluster.EXEC_BLOCK)
        hop_events = sum(line.startswith("HOP") for r in range(world)
                         for line in plan.rank_trace(r))
        assert hop_events == 2 * n_hops
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, layers, port, q, links))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, n_out, err in sorted(res):
        assert ok, f"rank {rank}: {err}"
    # every micro-batch's output and input gradient came out somewhere
    assert sum(n for _, _, n, _ in res) == 2 * MICRO


def _dying_worker(rank, world, port, q):
    """Rank 1's first block window raises and its process exits without
    leaving the group; rank 0 runs the plan until its next exchange with
    rank 1."""
    import time
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world))
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, os.path.join(root, "dependent-optics_b200"))
        import torch
        from dop import cluster as cl
        from dop import parallel
        parallel.init_from_env("gloo", timeout_s=10.0)
        cfg = small_cfg(2)
        plan = cl.stage_mixtral(cfg, MICRO, ROWS, MICRO, DOP_F32, cl.b200s(world))
        Ws, xs, dys = _data(2)
        mine = {h.layer for h in plan.homes if h.device == rank and h.kind == cl.HOME_PARAM}
        dWs = {l: torch.zeros_like(Ws[l]) for l in mine}

        class Dying(LinearLens):
            def forward(self, W, x):
                raise RuntimeError("stage died")

        lens = Dying() if rank == 1 else LinearLens()
        t0 = time.monotonic()
        try:
            cl.run_plan(plan, rank, lambda l, s: lens, Ws, dWs, xs, dys,
                        lambda r, c: torch.empty(r, c))
            q.put((rank, "finished", time.monotonic() - t0))
        except Exception as e:  # the failure as this rank sees it
            q.put((rank, f"error: {type(e).__name__}", time.monotonic() - t0))
    except Exception:
        q.put((rank, "setup: " + traceback.format_exc(), 0.0))
    q.close()
    q.join_thread()  # the report reaches the parent before the abrupt exit
    os._exit(0)  # leave without tearing the group down, like a crashed rank


def test_executor_reports_a_dead_stage():
    """A stage that dies between windows: the surviving stage's next
    point-to-point exchange with it ends with an error (within the process
    group's 10 s timeout) instead of waiting for good."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (s, t)) for r, s, t in (q.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    assert res[1][0].startswith("error: RuntimeError"), res
    assert res[0][0].startswith("error"), res
    assert res[0][1] < 60.0, res
