"""Full-size checks.

The small-Mixtral block (batch 4, seq 512, d 512, 8/2 heads, hd 64, window
128, 8 experts x 1408, top-2, fp32) is compared with the oracle at its full
size (the oracle takes about a minute here).  The Mixtral-8x7B block (batch 8,
seq 4096, bf16) is too large for the oracle (about 0.2 tokens/s); at that size
the tests check properties that hold for any size: the put is linear in the
output cotangent (doubling dy doubles dx and every parameter adjoint, bit for
bit, since scaling by 2 is exact in fp32 and bf16), two runs give identical
bytes, the permutation is the stable expert sort, and every output is finite.
"""
import numpy as np
import pytest
import torch

import oracle_ffi as orc
from dop import DOP_BF16, DOP_F32
from dop.mixtral import Block, MixtralConfig, layer_layout
from test_block_gpu import (F32_TOL, c2_cfg, check_routing, compare, make_inputs, run_gpu,
                            run_oracle)

pytestmark = pytest.mark.gpu


def test_small_mixtral_block_full_size_matches_oracle(cuda):
    cfg = c2_cfg()
    batch, seq = 4, 512
    lp, x, dy = make_inputs(cfg, batch, seq, seed=21)
    gpu = run_gpu(cfg, batch, seq, lp, x, dy, DOP_F32)
    ref = run_oracle(cfg, batch, seq, lp, x, dy)
    forced = check_routing(cfg, gpu, ref, 1e-6, 0.01)
    if forced is not None:
        ref = run_oracle(cfg, batch, seq, lp, x, dy, forced=forced)
    compare(cfg, gpu, ref, F32_TOL)


def test_mixtral8x7b_block_full_size_properties(cuda):
    cfg = MixtralConfig(vocab=32000, dim=4096, layers=1, heads=32, kv_heads=8, head_dim=128,
                        intermediate=14336, experts=8, top_k=2, rms_eps=1e-5, rope_theta=1e6,
                        sliding_window=4096)
    batch, seq = 8, 4096
    T = batch * seq
    ll = layer_layout(cfg)
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(5)
    P = torch.empty(ll.total, dtype=torch.bfloat16, device=dev)
    for a in range(0, ll.total, 1 << 28):
        b = min(ll.total, a + (1 << 28))
        P[a:b] = (torch.randn(b - a, generator=g, device=dev) * 0.02).bfloat16()
    P[ll.attn_norm: ll.attn_norm + cfg.dim] = 1.0
    P[ll.ffn_norm: ll.ffn_norm + cfg.dim] = 1.0
    X = torch.randn(T, cfg.dim, generator=g, device=dev)
    DY = torch.randn(T, cfg.dim, generator=g, device=dev)
    blk = Block(cfg, batch, seq, DOP_BF16)

    def run(dy):
        dP = torch.zeros(ll.total, device=dev)
        y = blk.forward(P, X)
        dx = blk.backward(P, dy, dP)
        torch.cuda.synchronize()
        return y, dx, dP

    y1, dx1, dP1 = run(DY)
    y2, dx2, dP2 = run(DY)
    assert torch.equal(y1, y2) and torch.equal(dx1, dx2) and torch.equal(dP1, dP2)
    for t in (y1, dx1, dP1):
        assert torch.isfinite(t).all()
    _, dx3, dP3 = run(2 * DY)
    assert torch.equal(dx3, 2 * dx1)
    assert torch.equal(dP3, 2 * dP1)
    # the permutation is the stable sort of (token, slot) pairs by expert
    top_i = blk.routing()[0].cpu().numpy().reshape(-1)
    slot_row, seg_off, _ = (t.cpu().numpy() for t in blk.permutation())
    counts = np.bincount(top_i, minlength=cfg.experts)
    off = np.concatenate([[0], np.cumsum((counts + 255) // 256 * 256)])
    assert np.array_equal(seg_off, off)
    order = np.argsort(top_i, kind="stable")
    sorted_e = top_i[order]
    expect = np.empty(T * cfg.top_k, np.int64)
    for e in range(cfg.experts):
        start = np.searchsorted(sorted_e, e)
        expect[order[start: start + counts[e]]] = off[e] + np.arange(counts[e])
    assert np.array_equal(slot_row, expect)
