"""Parity of the device block lens with the CPU oracle.

Bars (stated per test): routing indices and the permutation bit-exact
(tokens whose router decision margin is below the stated gap excluded);
fp32 lens within 1e-4 relative, bf16-weight / fp32-accumulate lens within
2e-2 relative, both max-abs normalised per output tensor and per parameter
matrix.  The bf16 lens is compared with the oracle evaluated on the same
bf16-rounded weights and inputs.
"""
import numpy as np
import pytest
import torch

import oracle_ffi as orc
from dop import DOP_BF16, DOP_F32
from dop.lens import Lens, compose
from dop.mixtral import Block, MixtralConfig, layer_layout

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 2e-2
ROUTER_GAP = 1e-6  # top-k decision gap below which a routing difference is excused
PROB_TOL = 1e-6    # router probabilities and renormalised gates, absolute


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    m = np.abs(b).max() if b.size else 0.0
    if m == 0.0:
        return float(np.abs(a).max()) if a.size else 0.0
    return float(np.abs(a - b).max() / m)


def param_slices(cfg):
    ll = layer_layout(cfg)
    D, I = cfg.dim, cfg.intermediate
    out = {"attn_norm": (ll.attn_norm, ll.q), "q": (ll.q, ll.k), "k": (ll.k, ll.v),
           "v": (ll.v, ll.o), "o": (ll.o, ll.ffn_norm), "ffn_norm": (ll.ffn_norm, ll.router),
           "router": (ll.router, ll.gate0)}
    for e in range(cfg.experts):
        g = ll.gate0 + e * ll.expert_stride
        out[f"gate{e}"] = (g, g + D * I)
        out[f"up{e}"] = (g + D * I, g + 2 * D * I)
        out[f"down{e}"] = (g + 2 * D * I, g + 3 * D * I)
    return out


def max_param_rel(cfg, got, ref):
    worst, name = 0.0, ""
    for n, (a, b) in param_slices(cfg).items():
        r = rel(got[a:b], ref[a:b])
        if r > worst:
            worst, name = r, n
    return worst, name


def decision_gap(prob_row, k):
    p = np.sort(np.asarray(prob_row, np.float64))[::-1]
    return float(min(p[i] - p[i + 1] for i in range(min(k, len(p) - 1)))) if len(p) > 1 else 1.0


def make_inputs(cfg, batch, seq, seed=0):
    """Synthetic workload: matrices ~ N(0, 0.02^2), RMSNorm weights 1,
    x ~ N(0, 1), dy ~ N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    n = orc.layer_params(cfg)
    lp = torch.randn(n, generator=g) * 0.02
    ll = layer_layout(cfg)
    lp[ll.attn_norm: ll.attn_norm + cfg.dim] = 1.0
    lp[ll.ffn_norm: ll.ffn_norm + cfg.dim] = 1.0
    T = batch * seq
    x = torch.randn(T * cfg.dim, generator=g)
    dy = torch.randn(T * cfg.dim, generator=g)
    return lp.float().numpy(), x.float().numpy(), dy.float().numpy()


def bf16_round(a):
    return torch.tensor(a).bfloat16().float().numpy()


def run_gpu(cfg, batch, seq, lp, x, dy, precision, bias=None):
    blk = Block(cfg, batch, seq, precision)
    dev = torch.device("cuda:0")
    P = torch.tensor(lp, device=dev)
    if precision == DOP_BF16:
        P = P.bfloat16()
    X = torch.tensor(x, device=dev).view(batch * seq, cfg.dim)
    DY = torch.tensor(dy, device=dev).view(batch * seq, cfg.dim)
    dP = torch.zeros(lp.size, dtype=torch.float32, device=dev)
    if bias is not None:
        blk.set_router_bias(torch.tensor(bias, device=dev))
    y = blk.forward(P, X)
    dx = blk.backward(P, DY, dP)
    torch.cuda.synchronize()
    ti, tw, tp, pr = blk.routing()
    perm = blk.permutation()
    return dict(blk=blk, y=y.cpu().numpy().reshape(-1), dx=dx.cpu().numpy().reshape(-1),
                dP=dP.cpu().numpy(), top_i=ti.cpu().numpy(), probs=pr.cpu().numpy(),
                perm=[t.cpu().numpy() for t in perm], P=P, X=X, DY=DY)


def run_oracle(cfg, batch, seq, lp, x, dy, bias=None, forced=None):
    r = orc.block_forward(cfg, lp, x, batch, seq, bias, forced)
    dx, dlp = orc.block_backward(cfg, lp, r, dy)
    ti, tw, tp, pr = r.routing()
    return dict(y=r.y, dx=dx, dP=dlp, top_i=ti, probs=pr)


def check_routing(cfg, gpu, ref, max_gap, max_frac):
    """Routing equal except at near-ties; returns the forced selection for
    the oracle rerun (or None when everything matched)."""
    diff = np.nonzero((gpu["top_i"] != ref["top_i"]).any(axis=1))[0]
    for t in diff:
        gap = decision_gap(ref["probs"][t], cfg.top_k)
        assert gap < max_gap, f"token {t}: routing differs with decision gap {gap}"
    assert len(diff) <= max_frac * len(gpu["top_i"]), f"{len(diff)} routing flips"
    return None if len(diff) == 0 else gpu["top_i"].astype(np.int64)


def check_router_stage(cfg, blk, lp, bias=None):
    """The device's routing equals the oracle's router stage run on the
    device's own feed-forward input (the device reproduces the crate's
    arithmetic there, so the probabilities agree to the last bit except
    where an exp result is rounded differently): indices equal except at
    decision gaps below 1e-6.  Returns (tokens whose indices differ, fraction
    of tokens whose probability row is bit-identical)."""
    mid = blk.ffn_input().cpu().numpy()
    ti_ref, tw_ref, _, pr_ref = orc.router_stage(cfg, lp, mid, bias)
    ti, tw, _, pr = (t.cpu().numpy() for t in blk.routing())
    assert np.abs(pr - pr_ref).max() < PROB_TOL, "router probabilities"
    diff = np.nonzero((ti != ti_ref).any(axis=1))[0]
    for t in diff:
        gap = decision_gap(pr_ref[t], cfg.top_k)
        assert gap < ROUTER_GAP, f"token {t}: router stage differs at decision gap {gap}"
    same = np.setdiff1d(np.arange(ti.shape[0]), diff)
    assert np.abs(tw[same] - tw_ref[same]).max() < PROB_TOL, "renormalised gates"
    exact = float((pr.view(np.uint32) == pr_ref.view(np.uint32)).all(axis=1).mean())
    return len(diff), exact


def compare(cfg, gpu, ref, tol):
    ry, rdx = rel(gpu["y"], ref["y"]), rel(gpu["dx"], ref["dx"])
    rp, worst = max_param_rel(cfg, gpu["dP"], ref["dP"])
    assert ry < tol, f"y rel err {ry}"
    assert rdx < tol, f"dx rel err {rdx}"
    assert rp < tol, f"dparams rel err {rp} in {worst}"
    return ry, rdx, rp


def small_cfg(**kw):
    base = dict(vocab=32, dim=64, layers=1, heads=4, kv_heads=2, head_dim=16, intermediate=96,
                experts=4, top_k=2, rms_eps=1e-5, rope_theta=1e6, sliding_window=24)
    base.update(kw)
    return MixtralConfig(**base)


def c2_cfg():
    return MixtralConfig(vocab=32, dim=512, layers=1, heads=8, kv_heads=2, head_dim=64,
                         intermediate=1408, experts=8, top_k=2, rms_eps=1e-5, rope_theta=1e6,
                         sliding_window=128)


@pytest.mark.parametrize("shape", [(2, 64), (3, 45)], ids=["b2s64", "b3s45-ragged"])
def test_f32_block_matches_oracle(cuda, shape):
    cfg = small_cfg()
    batch, seq = shape
    lp, x, dy = make_inputs(cfg, batch, seq, seed=1)
    gpu = run_gpu(cfg, batch, seq, lp, x, dy, DOP_F32)
    ref = run_oracle(cfg, batch, seq, lp, x, dy)
    forced = check_routing(cfg, gpu, ref, 1e-6, 0.01)
    if forced is not None:
        ref = run_oracle(cfg, batch, seq, lp, x, dy, forced=forced)
    compare(cfg, gpu, ref, F32_TOL)


def test_f32_block_c2_widths(cuda):
    """Small-Mixtral widths (d 512, 8/2 heads, hd 64, W 128, 8 experts x 1408,
    top-2) at batch 1, seq 160 so the oracle finishes in seconds."""
    cfg = c2_cfg()
    lp, x, dy = make_inputs(cfg, 1, 160, seed=2)
    gpu = run_gpu(cfg, 1, 160, lp, x, dy, DOP_F32)
    ref = run_oracle(cfg, 1, 160, lp, x, dy)
    forced = check_routing(cfg, gpu, ref, 1e-6, 0.01)
    if forced is not None:
        ref = run_oracle(cfg, 1, 160, lp, x, dy, forced=forced)
    compare(cfg, gpu, ref, F32_TOL)


def test_f32_block_long_contraction(cuda):
    """batch 4, seq 200: the weight gradients contract over 800 tokens into
    64-wide outputs, which the CUDA-core GEMM splits over the contraction
    (partials summed in split order)."""
    cfg = small_cfg()
    lp, x, dy = make_inputs(cfg, 4, 200, seed=4)
    gpu = run_gpu(cfg, 4, 200, lp, x, dy, DOP_F32)
    ref = run_oracle(cfg, 4, 200, lp, x, dy)
    forced = check_routing(cfg, gpu, ref, 1e-6, 0.01)
    if forced is not None:
        ref = run_oracle(cfg, 4, 200, lp, x, dy, forced=forced)
    compare(cfg, gpu, ref, F32_TOL)
    again = run_gpu(cfg, 4, 200, lp, x, dy, DOP_F32)
    for k in ("y", "dx", "dP"):
        assert np.array_equal(gpu[k], again[k]), k


@pytest.mark.parametrize("kind", ["moe", "dense", "moe-hd128"])
def test_bf16_block_matches_oracle_on_rounded_inputs(cuda, kind):
    if kind == "moe":
        cfg = small_cfg(dim=128, head_dim=32, intermediate=192)
    elif kind == "moe-hd128":  # head_dim 128: tensor-core attention, window < seq
        cfg = small_cfg(dim=256, heads=4, kv_heads=2, head_dim=128, intermediate=256,
                        sliding_window=100)
    else:
        cfg = small_cfg(dim=128, heads=4, kv_heads=4, head_dim=32, intermediate=192, experts=1,
                        top_k=1, sliding_window=10_000, rope_theta=1e4)
    batch, seq = (2, 200) if kind == "moe-hd128" else (2, 80)
    lp, x, dy = make_inputs(cfg, batch, seq, seed=3)
    lp, x, dy = bf16_round(lp), bf16_round(x), bf16_round(dy)
    gpu = run_gpu(cfg, batch, seq, lp, x, dy, DOP_BF16)
    check_router_stage(cfg, gpu["blk"], lp)  # the 1e-6 bar on the lens's own input
    ref = run_oracle(cfg, batch, seq, lp, x, dy)
    forced = check_routing(cfg, gpu, ref, 1e-2, 0.03)
    if forced is not None:
        ref = run_oracle(cfg, batch, seq, lp, x, dy, forced=forced)
    compare(cfg, gpu, ref, BF16_TOL)
    if kind == "dense":  # E = 1: the router's adjoint is exactly zero (src/mixtral.rs:531)
        a, b = param_slices(cfg)["router"]
        assert np.all(gpu["dP"][a:b] == 0.0)


@pytest.mark.parametrize("dim, experts, top_k", [(100, 12, 3), (98, 6, 2), (256, 16, 4)],
                         ids=["d100-e12-k3", "d98-e6-k2", "d256-e16-k4"])
def test_router_stage_odd_widths(cuda, dim, experts, top_k):
    """The router stage's two kernels off the Mixtral shape: a model width
    that is not a multiple of the 64-column tile (100), one that is not a
    multiple of 4 (98: scalar loads), and 12 / 6 / 16 experts (16 logit
    chains per row, 8 with unused ones).  Same 1e-6 gap bar on the lens's own
    feed-forward input, probability rows bit-identical but for rare
    last-bit exp roundings (at most 4 of the 160 rows)."""
    cfg = small_cfg(dim=dim, experts=experts, top_k=top_k)
    lp, x, dy = make_inputs(cfg, 2, 80, seed=7)
    gpu = run_gpu(cfg, 2, 80, lp, x, dy, DOP_F32)
    _, exact = check_router_stage(cfg, gpu["blk"], lp)
    assert exact >= 156 / 160, f"only {exact:.4f} of the probability rows are bit-identical"


def test_permutation_is_the_stable_expert_sort(cuda):
    cfg = small_cfg(experts=8, top_k=2)
    batch, seq = 4, 100
    lp, x, dy = make_inputs(cfg, batch, seq, seed=4)
    gpu = run_gpu(cfg, batch, seq, lp, x, dy, DOP_F32)
    slot_row, seg_off, row_token = gpu["perm"]
    top_i = gpu["top_i"].reshape(-1)
    T, k, E = batch * seq, cfg.top_k, cfg.experts
    # reference: stable counting sort of (token, slot) pairs by expert,
    # segments padded to 256 rows
    counts = np.bincount(top_i, minlength=E)
    off = np.zeros(E + 1, np.int64)
    for e in range(E):
        off[e + 1] = off[e] + (counts[e] + 255) // 256 * 256
    assert np.array_equal(seg_off, off)
    fill = off[:-1].copy()
    exp_row = np.zeros(T * k, np.int64)
    exp_tok = np.full(row_token.size, -1, np.int64)
    for p in range(T * k):
        e = top_i[p]
        exp_row[p] = fill[e]
        exp_tok[fill[e]] = p // k
        fill[e] += 1
    assert np.array_equal(slot_row, exp_row)
    assert np.array_equal(row_token[: off[-1]], exp_tok[: off[-1]])


def test_deterministic_and_accumulating(cuda):
    cfg = small_cfg()
    batch, seq = 2, 64
    lp, x, dy = make_inputs(cfg, batch, seq, seed=5)
    a = run_gpu(cfg, batch, seq, lp, x, dy, DOP_F32)
    b = run_gpu(cfg, batch, seq, lp, x, dy, DOP_F32)
    for key in ("y", "dx", "dP"):
        assert np.array_equal(a[key].view(np.uint32), b[key].view(np.uint32)), key
    # a second backward on the same handle adds the same adjoint again
    dP = torch.tensor(a["dP"], device="cuda")
    a["blk"].backward(a["P"], a["DY"], dP)
    torch.cuda.synchronize()
    assert rel(dP.cpu().numpy(), 2 * a["dP"]) < 1e-6


def test_router_bias_skews_routing(cuda):
    cfg = small_cfg(experts=8)
    batch, seq = 2, 64
    lp, x, dy = make_inputs(cfg, batch, seq, seed=6)
    bias = (2.0 * np.arange(1, 9, dtype=np.float32) ** -1.2).astype(np.float32)
    gpu = run_gpu(cfg, batch, seq, lp, x, dy, DOP_F32, bias=bias)
    ref = run_oracle(cfg, batch, seq, lp, x, dy, bias=bias)
    forced = check_routing(cfg, gpu, ref, 1e-6, 0.01)
    if forced is not None:
        ref = run_oracle(cfg, batch, seq, lp, x, dy, bias=bias, forced=forced)
    compare(cfg, gpu, ref, F32_TOL)
    counts = np.bincount(gpu["top_i"].reshape(-1), minlength=8)
    assert counts[0] > counts[-1]


def test_compose_two_blocks(cuda):
    """compose(g, f): forward g(f(x)); backward runs g's put then f's."""
    cfg = small_cfg()
    batch, seq = 2, 32
    lp1, x, dy = make_inputs(cfg, batch, seq, seed=7)
    lp2, _, _ = make_inputs(cfg, batch, seq, seed=8)
    dev = "cuda"
    f_blk, g_blk = Block(cfg, batch, seq, DOP_F32), Block(cfg, batch, seq, DOP_F32)
    P1, P2 = torch.tensor(lp1, device=dev), torch.tensor(lp2, device=dev)
    dP1, dP2 = torch.zeros_like(P1), torch.zeros_like(P2)
    lens = compose(Lens.of_block(g_blk, P2, dP2), Lens.of_block(f_blk, P1, dP1))
    X = torch.tensor(x, device=dev).view(-1, cfg.dim)
    y = lens.forward(X)
    dx = lens.backward(torch.tensor(dy, device=dev).view(-1, cfg.dim))
    torch.cuda.synchronize()
    r1 = orc.block_forward(cfg, lp1, x, batch, seq)
    r2 = orc.block_forward(cfg, lp2, r1.y, batch, seq)
    dmid, g2 = orc.block_backward(cfg, lp2, r2, dy)
    dx_ref, g1 = orc.block_backward(cfg, lp1, r1, dmid)
    assert rel(y.cpu().numpy().reshape(-1), r2.y) < F32_TOL
    assert rel(dx.cpu().numpy().reshape(-1), dx_ref) < F32_TOL
    assert max_param_rel(cfg, dP1.cpu().numpy(), g1)[0] < F32_TOL
    assert max_param_rel(cfg, dP2.cpu().numpy(), g2)[0] < F32_TOL
    lens.close()
