"""The staged pipeline on 2 GPUs: a 2-block bf16 Mixtral stack, 4
micro-batches, one block per GPU (PP 2), run by dop.cluster.run_plan with
block lenses executing their windows through dop_run_window, NCCL carrying
the activations and their adjoints.  A single-GPU sequential run of the
same blocks on the same micro-batches (forward through both blocks, then
backward, micro-batch by micro-batch) must give the same bits: every
output, every input gradient and each block's parameter adjoint (both runs
accumulate a block's micro-batches in the same order).  Each rank's events
must equal the plan's trace projected on it.
"""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD, MICRO, SEQ = 2, 4, 128


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    from dop.mixtral import MixtralConfig
    return MixtralConfig(vocab=64, dim=256, layers=2, heads=4, kv_heads=2, head_dim=128,
                         intermediate=256, experts=8, top_k=2, rms_eps=1e-5, rope_theta=1e4,
                         sliding_window=96)


def _inputs(cfg, dev):
    from dop.mixtral import layer_layout
    ll = layer_layout(cfg)
    g = torch.Generator(device=dev).manual_seed(11)
    Ps = []
    for _ in range(cfg.layers):
        P = (torch.randn(ll.total, generator=g, device=dev) * 0.05).bfloat16()
        P[ll.attn_norm: ll.attn_norm + cfg.dim] = 1.0
        P[ll.ffn_norm: ll.ffn_norm + cfg.dim] = 1.0
        Ps.append(P)
    xs = [torch.randn(SEQ, cfg.dim, generator=g, device=dev) for _ in range(MICRO)]
    dys = [torch.randn(SEQ, cfg.dim, generator=g, device=dev) for _ in range(MICRO)]
    return ll, Ps, xs, dys


def _rank_main(rank: int, port: int) -> None:
    import torch.distributed as dist
    from dop import DOP_BF16, lib
    from dop import cluster
    from dop.mixtral import Block

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(WORLD))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        cfg = _cfg()
        ll, Ps, xs, dys = _inputs(cfg, dev)
        plan = cluster.stage_mixtral(cfg, MICRO, SEQ, MICRO, DOP_BF16, cluster.b200s(WORLD))
        one = _cfg()
        blocks = {}

        def lens_for(layer, slot):
            if (layer, slot) not in blocks:
                blocks[(layer, slot)] = cluster.BlockLens(Block(one, 1, SEQ, DOP_BF16))
            return blocks[(layer, slot)]

        mine = [h.layer for h in plan.homes if h.device == rank and h.kind == cluster.HOME_PARAM]
        dPs = {l: torch.zeros(ll.total, device=dev) for l in mine}
        out = cluster.run_plan(plan, rank, lens_for, Ps, dPs, xs, dys,
                               lambda r, c: torch.empty(r, c, device=dev))
        torch.cuda.synchronize(dev)
        assert lib().dop_device_status() == 0
        assert out["trace"] == plan.rank_trace(rank)
        # the same blocks, one GPU, micro-batch by micro-batch
        ref = [Block(one, 1, SEQ, DOP_BF16) for _ in range(cfg.layers)]
        ref_dP = [torch.zeros(ll.total, device=dev) for _ in range(cfg.layers)]
        for m in range(MICRO):
            h = xs[m]
            for l in range(cfg.layers):
                h = ref[l].forward(Ps[l], h)
            if m in out["outputs"]:
                assert torch.equal(out["outputs"][m], h), f"output of micro-batch {m}"
            g = dys[m]
            for l in reversed(range(cfg.layers)):
                g = ref[l].backward(Ps[l], g, ref_dP[l])
            if m in out["input_grads"]:
                assert torch.equal(out["input_grads"][m], g), f"input gradient of micro-batch {m}"
        for l in mine:
            assert torch.equal(dPs[l], ref_dP[l]), f"adjoint of block {l}"
        assert len(out["outputs"]) == (MICRO if rank == WORLD - 1 else 0)
        assert len(out["input_grads"]) == (MICRO if rank == 0 else 0)
        torch.cuda.synchronize(dev)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_pipeline_matches_sequential_stack():
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(_free_port(),), nprocs=WORLD, join=True)
