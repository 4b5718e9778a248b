"""The whole-model lens on the GPU (dop_model_forward_backward) against the
oracle's mixtral::forward_backward on the crate's demo model, and the crate's
own demo tests (src/mixtral.rs:1248-1325) run through the GPU lens: finite
differences on the same 8 probes, zero adjoint of unselected experts, and one
SGD step descending."""
import numpy as np
import pytest
import torch

import oracle_ffi as orc
from dop import DOP_F32
from dop.mixtral import (DEMO_LR, Model, MixtralConfig, demo_batch, init_params, init_router,
                         layout, sgd_step)

pytestmark = pytest.mark.gpu
TOL = 1e-4


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    m = np.abs(b).max()
    return float(np.abs(a - b).max() / m) if m > 0 else float(np.abs(a).max())


def regions(cfg):
    lay = layout(cfg)
    out = {"embed": (lay.embed, lay.layers[0].attn_norm), "final_norm": (lay.final_norm, lay.lm_head),
           "lm_head": (lay.lm_head, lay.total)}
    for i, L in enumerate(lay.layers):
        D, qd, kvd, I = cfg.dim, cfg.q_dim(), cfg.kv_dim(), cfg.intermediate
        out[f"l{i}.attn_norm"] = (L.attn_norm, L.q)
        out[f"l{i}.q"] = (L.q, L.k)
        out[f"l{i}.k"] = (L.k, L.v)
        out[f"l{i}.v"] = (L.v, L.o)
        out[f"l{i}.o"] = (L.o, L.ffn_norm)
        out[f"l{i}.ffn_norm"] = (L.ffn_norm, L.router)
        out[f"l{i}.router"] = (L.router, L.gate[0])
        for e in range(cfg.experts):
            out[f"l{i}.gate{e}"] = (L.gate[e], L.gate[e] + D * I)
            out[f"l{i}.up{e}"] = (L.up[e], L.up[e] + D * I)
            out[f"l{i}.down{e}"] = (L.down[e], L.down[e] + I * D)
    return out


def demo():
    c = MixtralConfig.demo()
    p = init_params(c)
    init_router(c, p)
    batch, seq, tokens, targets = demo_batch(c)
    return c, p, batch, seq, tokens, targets


def gpu_fb(m, P, tokens, targets):
    r = m.forward_backward(P, tokens, targets)
    torch.cuda.synchronize()
    return r


def test_demo_model_matches_oracle(cuda):
    c, p, batch, seq, tokens, targets = demo()
    loss_r, grad_r, logits_r = orc.mixtral_forward_backward(c, p, tokens, targets, batch, seq)
    m = Model(c, batch, seq, DOP_F32)
    tk = torch.tensor(tokens, device="cuda")
    tg = torch.tensor(targets, device="cuda")
    r = gpu_fb(m, torch.tensor(p, device="cuda"), tk, tg)
    assert abs(r.loss.item() - loss_r) <= 1e-5 * abs(loss_r)
    assert rel(r.logits.cpu().numpy().reshape(-1), logits_r) < TOL
    g = r.grad.cpu().numpy()
    for name, (a, b) in regions(c).items():
        assert rel(g[a:b], grad_r[a:b]) < TOL, name


def test_demo_finite_differences_unselected_experts_and_descent(cuda):
    c, p, batch, seq, tokens, targets = demo()
    lay = layout(c)
    m = Model(c, batch, seq, DOP_F32)
    tk = torch.tensor(tokens, device="cuda")
    tg = torch.tensor(targets, device="cuda")
    P = torch.tensor(p, device="cuda")
    r = gpu_fb(m, P, tk, tg)
    grad = r.grad.cpu().numpy()
    loss0 = r.loss.item()
    eps = 1e-3
    probes = [lay.embed + 3, lay.layers[0].attn_norm + 1, lay.layers[0].q + 10,
              lay.layers[0].o + 4, lay.layers[1].gate[3] + 7, lay.layers[0].down[2] + 5,
              lay.final_norm + 2, lay.lm_head + 9]
    for i in probes:
        Pp, Pm = P.clone(), P.clone()
        Pp[i] += eps
        Pm[i] -= eps
        lp = gpu_fb(m, Pp, tk, tg).loss.item()
        lm = gpu_fb(m, Pm, tk, tg).loss.item()
        assert abs((lp - lm) / (2 * eps) - grad[i]) < 2e-2, i
    # experts that no token selected in layer 0 (routing from the oracle) get no adjoint
    D = c.dim
    x = np.stack([p[lay.embed + t * D: lay.embed + (t + 1) * D] for t in tokens]).reshape(-1)
    used = [False] * c.experts
    for L in lay.layers:
        res = orc.block_forward(c, p[L.attn_norm: L.attn_norm + orc.layer_params(c)], x, batch, seq)
        for e in res.routing()[0].reshape(-1):
            used[int(e)] = True
        x = res.y
    assert any(used) and not all(used)
    for e, on in enumerate(used):
        if not on:
            a, b = lay.layers[0].gate[e], lay.layers[0].down[e] + c.intermediate * c.dim
            assert np.abs(grad[a:b]).sum() < 1e-6
    sgd_step(P, r.grad, DEMO_LR)
    loss1 = gpu_fb(m, P, tk, tg).loss.item()
    assert loss1 < loss0
