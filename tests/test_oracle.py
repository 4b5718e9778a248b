"""The oracle pinned against the crate's own tests (CPU, no GPU needed).

The crate ships no golden vectors.  What pins its tensor lenses are its
tests: parameter counts (src/mixtral.rs:1239-1245, README.md:287), finite
differences on the demo model (src/mixtral.rs:1248-1279) and on the kernel.rs
programs (src/kernel.rs:1008-1012), zero adjoint of unselected experts
(:1281-1314), SGD descent (:1316-1321) and tape sizes (src/kernel.rs:982-1005).
Each is restated here against the C++ oracle, plus a float64 torch-autograd
referee for the block's backward pass.
"""
import numpy as np
import pytest
import torch

import oracle_ffi as orc
from dop import kernel as K
from dop.mixtral import (DEMO_LR, MixtralConfig, demo_batch, init_params, init_router, layout,
                         parameter_count)


def test_parameter_counts():
    n = parameter_count(MixtralConfig.mixtral_8x7b())
    assert 46_500_000_000 <= n < 47_000_000_000
    assert n == 46_702_792_704
    assert parameter_count(MixtralConfig.demo()) == 45_472
    for cfg in (MixtralConfig.demo(), MixtralConfig.mixtral_8x7b()):
        assert orc.parameter_count(cfg) == parameter_count(cfg)
        lay = layout(cfg)
        per_layer = (lay.final_norm - lay.layers[0].attn_norm) // cfg.layers
        assert orc.layer_params(cfg) == per_layer
        assert lay.layers[1].attn_norm - lay.layers[0].attn_norm == per_layer


def _demo():
    c = MixtralConfig.demo()
    p = init_params(c)
    init_router(c, p)
    return c, p


def test_demo_adjoint_matches_finite_differences():
    c, p = _demo()
    lay = layout(c)
    batch, seq, tokens, targets = demo_batch(c)
    loss, grad, _ = orc.mixtral_forward_backward(c, p, tokens, targets, batch, seq)
    eps = np.float32(1e-3)
    probes = [lay.embed + 3, lay.layers[0].attn_norm + 1, lay.layers[0].q + 10,
              lay.layers[0].o + 4, lay.layers[1].gate[3] + 7, lay.layers[0].down[2] + 5,
              lay.final_norm + 2, lay.lm_head + 9]
    for i in probes:
        plus, minus = p.copy(), p.copy()
        plus[i] += eps
        minus[i] -= eps
        lp = orc.mixtral_forward_backward(c, plus, tokens, targets, batch, seq)[0]
        lm = orc.mixtral_forward_backward(c, minus, tokens, targets, batch, seq)[0]
        num = (np.float32(lp) - np.float32(lm)) / (np.float32(2.0) * eps)
        assert abs(num - grad[i]) < 2e-2, (i, grad[i], num)


def test_demo_unselected_experts_get_no_gradient_and_sgd_descends():
    c, p = _demo()
    lay = layout(c)
    batch, seq, tokens, targets = demo_batch(c)
    loss0, grad, _ = orc.mixtral_forward_backward(c, p, tokens, targets, batch, seq)
    # routing of every layer: run the block lenses layer by layer
    D = c.dim
    x = np.stack([p[lay.embed + t * D: lay.embed + (t + 1) * D] for t in tokens]).reshape(-1)
    used = [False] * c.experts
    for L in lay.layers:
        lp = p[L.attn_norm: L.attn_norm + orc.layer_params(c)]
        r = orc.block_forward(c, lp, x, batch, seq)
        ti = r.routing()[0]
        for e in ti.reshape(-1):
            used[int(e)] = True
        x = r.y
    assert any(used) and not all(used), used
    for e, on in enumerate(used):
        if on:
            continue
        start = lay.layers[0].gate[e]
        stop = lay.layers[0].down[e] + c.intermediate * c.dim
        assert np.abs(grad[start:stop]).sum() < 1e-6
    step = p.copy()
    gnorm = orc.sgd_step(step, grad, DEMO_LR)
    assert np.isfinite(gnorm) and gnorm > 0
    loss1 = orc.mixtral_forward_backward(c, step, tokens, targets, batch, seq)[0]
    assert loss1 < loss0


def test_program_tape_sizes():
    mlp = K.Program.mlp(2, [3, 4, 2])
    assert mlp.tape_f32 == 2 * 3 + 2 * 4 and mlp.tape_u8 == 2 * 4
    assert mlp.param_len == 3 * 4 + 4 + 4 * 2 + 2
    blk = K.Program.resnet_block(2, 4, 6)
    assert blk.tape_f32 == 2 * 4 + 2 * 6 and blk.tape_u8 == 2 * 6
    assert isinstance(blk.stages[-1], K.Add) and blk.stages[-1].from_ == 0
    tr = K.Program.transformer_block(2, 3, 4, 8)
    n = 2 * 3 * 4
    assert tr.tape_f32 == n + 2 * 3 * 3 + n + 2 * 3 * 8 and tr.tape_u8 == 2 * 3 * 8


@pytest.mark.parametrize("prog", [K.Program.mlp(2, [3, 4, 2]), K.Program.resnet_block(2, 3, 4),
                                  K.Program.transformer_block(1, 3, 4, 5)],
                         ids=["mlp", "resnet", "transformer"])
def test_programs_match_finite_differences(prog):
    x = K.init(prog.input_len, 0.5)
    params = K.init(prog.param_len, 0.25)
    y, dx, dp = orc.program_forward_backward(prog, x, params)
    eps = np.float32(1e-3)

    def fd(xx, pp):
        return orc.program_forward_backward(prog, xx, pp)[0].sum(dtype=np.float32)

    for i in range(prog.input_len):
        x1, x0 = x.copy(), x.copy()
        x1[i] += eps
        x0[i] -= eps
        num = (fd(x1, params) - fd(x0, params)) / (2 * eps)
        assert abs(num - dx[i]) < 2e-2, (i, dx[i], num)
    for i in range(prog.param_len):
        p1, p0 = params.copy(), params.copy()
        p1[i] += eps
        p0[i] -= eps
        num = (fd(x, p1) - fd(x, p0)) / (2 * eps)
        assert abs(num - dp[i]) < 2e-2, (i, dp[i], num)


def _small_cfg(**kw):
    base = dict(vocab=32, dim=32, layers=1, heads=4, kv_heads=2, head_dim=8, intermediate=24,
                experts=4, top_k=2, rms_eps=1e-5, rope_theta=1e4, sliding_window=5)
    base.update(kw)
    return MixtralConfig(**base)


@pytest.mark.parametrize("kw", [{}, {"experts": 1, "top_k": 1, "kv_heads": 4, "sliding_window": 64}],
                         ids=["moe", "dense"])
def test_oracle_block_matches_float64_autograd(kw):
    import torch_block
    c = _small_cfg(**kw)
    batch, seq = 2, 7
    g = torch.Generator().manual_seed(0)
    n = orc.layer_params(c)
    lp = (torch.randn(n, generator=g) * 0.2).float().numpy()
    x = torch.randn(batch * seq * c.dim, generator=g).float().numpy()
    dy = torch.randn(batch * seq * c.dim, generator=g).float().numpy()
    r = orc.block_forward(c, lp, x, batch, seq)
    dx, dlp = orc.block_backward(c, lp, r, dy)
    lp64 = torch.tensor(lp, dtype=torch.float64, requires_grad=True)
    x64 = torch.tensor(x, dtype=torch.float64).view(batch * seq, c.dim).requires_grad_(True)
    y64, top_i = torch_block.block_forward(c, lp64, x64, batch, seq)
    (y64 * torch.tensor(dy, dtype=torch.float64).view_as(y64)).sum().backward()
    assert np.array_equal(np.array(top_i), r.routing()[0])

    def rel(a, b):
        b = np.asarray(b, np.float64)
        return np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30)

    assert rel(r.y, y64.detach().numpy().reshape(-1)) < 1e-5
    assert rel(dx, x64.grad.numpy().reshape(-1)) < 1e-4
    assert rel(dlp, lp64.grad.numpy()) < 1e-4
    # the vectorised model (the referee of the full-size GPU check) agrees too
    lpb = torch.tensor(lp, dtype=torch.float64, requires_grad=True)
    xb = torch.tensor(x, dtype=torch.float64).view(batch * seq, c.dim).requires_grad_(True)
    yb, _, top_b = torch_block.block_forward_batched(c, lpb, xb, seq)
    (yb * torch.tensor(dy, dtype=torch.float64).view_as(yb)).sum().backward()
    assert np.array_equal(top_b.numpy(), r.routing()[0])
    assert rel(r.y, yb.detach().numpy().reshape(-1)) < 1e-5
    assert rel(dx, xb.grad.numpy().reshape(-1)) < 1e-4
    assert rel(dlp, lpb.grad.numpy()) < 1e-4


@pytest.mark.parametrize("threads", [1, 3, 8])
def test_threaded_loops_give_the_literal_loops_bytes(threads):
    """The oracle's interchanged, threaded loop nests keep every output's
    accumulation sequence, so they give the bytes of the crate's literal
    loop order (src/mixtral.rs:616-659): checked at the small-Mixtral widths,
    where every contraction takes the threaded path, for y, dx, the whole
    adjoint, the routing and the router stage."""
    c = MixtralConfig(vocab=32, dim=512, layers=1, heads=8, kv_heads=2, head_dim=64,
                      intermediate=1408, experts=8, top_k=2, rms_eps=1e-5, rope_theta=1e6,
                      sliding_window=24)
    batch, seq = 2, 20
    g = torch.Generator().manual_seed(5)
    n = orc.layer_params(c)
    lp = (torch.randn(n, generator=g) * 0.02).float().numpy()
    x = torch.randn(batch * seq * c.dim, generator=g).float().numpy()
    dy = torch.randn(batch * seq * c.dim, generator=g).float().numpy()
    outs = []
    try:
        for literal in (True, False):
            orc.set_literal(literal)
            orc.set_threads(threads)
            r = orc.block_forward(c, lp, x, batch, seq)
            dx, dlp = orc.block_backward(c, lp, r, dy)
            stage = orc.router_stage(c, lp, r.y)
            outs.append([r.y.copy(), dx, dlp, r.routing()[0], *stage])
    finally:
        orc.set_literal(False)
        orc.set_threads(0)
    for a, b in zip(*outs):
        assert a.dtype == b.dtype and np.array_equal(a.view(np.uint8), b.view(np.uint8))
