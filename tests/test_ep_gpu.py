"""Expert-parallel block lens on 2 GPUs (one process per GPU, NCCL for the
handle exchange and the reference sums).

Each rank runs the expert-parallel block on its own batch and, on the same
GPU, a single-GPU block on the same batch.  The expert-parallel outputs must
equal the single-GPU ones: a row's expert GEMMs and the slot-ordered combine
do not depend on where the row sits, so y and the shared adjoint slice are
bit-identical and dx agrees to fp32 rounding.  The adjoint of each rank's
own experts must equal the sum over ranks of the single-GPU adjoints (fp32
tolerance: the two sum the same products in a different order), and the
other experts' slices must stay untouched.  Three steps run back to back:
balanced routing, a router bias that sends most rows to rank 0's experts,
and one that sends most rows to expert 0 alone.  Under the skewed steps the
plan gives part of the hot experts' rows to rank 1, which returns their
partial weight adjoints to rank 0; the bars are the same.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel(a, b) -> float:
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _rank_main(rank: int, port: int) -> None:
    import datetime

    import torch.distributed as dist

    from dop import DOP_BF16, lib
    from dop import parallel
    from dop.mixtral import Block, MixtralConfig, layer_layout

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(WORLD))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        cfg = MixtralConfig(vocab=64, dim=256, layers=1, heads=4, kv_heads=2, head_dim=128,
                            intermediate=256, experts=8, top_k=2, rms_eps=1e-5, rope_theta=1e4,
                            sliding_window=96)
        batch, seq = 2, 256
        T = batch * seq
        ll = layer_layout(cfg)
        g = torch.Generator(device=dev).manual_seed(7)  # same weights on both ranks
        P = (torch.randn(ll.total, generator=g, device=dev) * 0.05).bfloat16()
        P[ll.attn_norm: ll.attn_norm + cfg.dim] = 1.0
        P[ll.ffn_norm: ll.ffn_norm + cfg.dim] = 1.0
        gx = torch.Generator(device=dev).manual_seed(100 + rank)  # own batch per rank
        ep_blk = Block(cfg, batch, seq, DOP_BF16, ep=(rank, WORLD))
        parallel.connect_expert_parallel(ep_blk, device=dev)
        ref_blk = Block(cfg, batch, seq, DOP_BF16)
        per = cfg.experts // WORLD
        stride = ll.expert_stride
        own = slice(ll.gate0 + rank * per * stride, ll.gate0 + (rank + 1) * per * stride)
        for step in range(3):
            if step >= 1:
                bias = torch.zeros(cfg.experts, device=dev)
                if step == 1:
                    bias[:per] = 3.0  # most rows go to rank 0's experts
                else:
                    bias[0] = 6.0  # one expert takes most rows: split over both ranks
                ep_blk.set_router_bias(bias)
                ref_blk.set_router_bias(bias)
            X = torch.randn(T, cfg.dim, generator=gx, device=dev)
            DY = torch.randn(T, cfg.dim, generator=gx, device=dev)
            dP_ep = torch.zeros(ll.total, device=dev)
            dP_ref = torch.zeros(ll.total, device=dev)
            y_ep = ep_blk.forward(P, X)
            dx_ep = ep_blk.backward(P, DY, dP_ep)
            y_ref = ref_blk.forward(P, X)
            dx_ref = ref_blk.backward(P, DY, dP_ref)
            torch.cuda.synchronize(dev)
            assert lib().dop_device_status() == 0
            assert torch.equal(y_ep, y_ref), f"rank {rank} step {step}: y differs"
            assert _rel(dx_ep, dx_ref) < 1e-5, f"rank {rank} step {step}: dx {_rel(dx_ep, dx_ref)}"
            assert torch.equal(dP_ep[:ll.gate0], dP_ref[:ll.gate0]), "shared adjoint differs"
            dist.all_reduce(dP_ref)  # the experts' adjoints summed over every rank's tokens
            assert _rel(dP_ep[own], dP_ref[own]) < 1e-4, f"own experts {_rel(dP_ep[own], dP_ref[own])}"
            others = torch.ones(ll.total, dtype=torch.bool, device=dev)
            others[: ll.gate0] = False
            others[own] = False
            assert not dP_ep[others].any(), "another rank's expert slice was written"
        torch.cuda.synchronize(dev)
        dist.barrier()
        ep_blk.close()
        ref_blk.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_expert_parallel_matches_single_gpu():
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(_free_port(),), nprocs=WORLD, join=True)
