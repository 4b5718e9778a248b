"""An independent torch-autograd model of the Mixtral block, used as a
float64 referee for the C++ oracle (and nothing else).

Same mathematics as src/mixtral.rs:291-598, written with torch ops and
autograd instead of hand-written adjoints, so agreement between the two is
evidence that the oracle's restated backward pass is right.
"""
from __future__ import annotations

import torch


def split_layer(cfg, lp: torch.Tensor):
    D, qd, kvd, E, I = cfg.dim, cfg.q_dim(), cfg.kv_dim(), cfg.experts, cfg.intermediate
    at = 0

    def take(n, shape):
        nonlocal at
        t = lp[at: at + n].view(*shape)
        at += n
        return t

    p = {"attn_norm": take(D, (D,)), "q": take(D * qd, (D, qd)), "k": take(D * kvd, (D, kvd)),
         "v": take(D * kvd, (D, kvd)), "o": take(qd * D, (qd, D)), "ffn_norm": take(D, (D,)),
         "router": take(D * E, (D, E))}
    p["gate"], p["up"], p["down"] = [], [], []
    for _ in range(E):
        p["gate"].append(take(D * I, (D, I)))
        p["up"].append(take(D * I, (D, I)))
        p["down"].append(take(I * D, (I, D)))
    return p


def rmsnorm(x, w, eps):
    r = 1.0 / torch.sqrt((x * x).mean(-1, keepdim=True) + eps)
    return x * r * w


def rope(x, S, heads, hd, theta):
    T = x.shape[0]
    half = hd // 2
    i = torch.arange(half, dtype=torch.float32)
    freq = torch.tensor(theta, dtype=torch.float32) ** (-(2.0 * i) / hd)
    pos = (torch.arange(T) % S).to(torch.float32)
    ang = pos[:, None] * freq[None, :]
    c = torch.cos(ang).to(x.dtype)[:, None, :]
    s = torch.sin(ang).to(x.dtype)[:, None, :]
    xh = x.view(T, heads, hd)
    x1, x2 = xh[..., :half], xh[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).reshape(T, heads * hd)


def block_forward(cfg, lp, x, batch, seq, bias=None):
    """Returns y (autograd-connected to lp and x) and the routing top_i."""
    p = split_layer(cfg, lp)
    H, KV, hd = cfg.heads, cfg.kv_heads, cfg.head_dim
    T = batch * seq
    xn = rmsnorm(x, p["attn_norm"], cfg.rms_eps)
    q = rope(xn @ p["q"], seq, H, hd, cfg.rope_theta)
    k = rope(xn @ p["k"], seq, KV, hd, cfg.rope_theta)
    v = xn @ p["v"]
    qh = q.view(batch, seq, H, hd).transpose(1, 2)
    kh = k.view(batch, seq, KV, hd).transpose(1, 2).repeat_interleave(H // KV, dim=1)
    vh = v.view(batch, seq, KV, hd).transpose(1, 2).repeat_interleave(H // KV, dim=1)
    s = (qh @ kh.transpose(-1, -2)) / (hd ** 0.5)
    iq = torch.arange(seq)[:, None]
    jk = torch.arange(seq)[None, :]
    vis = (jk <= iq) & (iq - jk < cfg.sliding_window)
    s = s.masked_fill(~vis, float("-inf"))
    pr = torch.softmax(s, -1)
    mix = (pr @ vh).transpose(1, 2).reshape(T, H * hd)
    mid = x + mix @ p["o"]
    xn2 = rmsnorm(mid, p["ffn_norm"], cfg.rms_eps)
    logits = xn2 @ p["router"]
    if bias is not None:
        logits = logits + bias
    probs = torch.softmax(logits, -1)
    # selection is by (prob desc, index asc); the indices carry no gradient
    with torch.no_grad():
        top_i = []
        for t in range(T):
            row = probs[t].tolist()
            order = sorted(range(cfg.experts), key=lambda e: (-row[e], e))
            top_i.append(order[: cfg.top_k])
    mixed = torch.zeros_like(x)
    rows = []
    for t in range(T):
        sel = top_i[t]
        ps = probs[t, sel]
        w = ps / ps.sum()
        acc = torch.zeros(cfg.dim, dtype=x.dtype)
        for kk, e in enumerate(sel):
            g = xn2[t] @ p["gate"][e]
            u = xn2[t] @ p["up"][e]
            h = torch.nn.functional.silu(g) * u
            acc = acc + w[kk] * (h @ p["down"][e])
        rows.append(acc)
    mixed = torch.stack(rows)
    return mid + mixed, top_i


def block_forward_batched(cfg, lp, x, seq, forced_top_i=None):
    """The same block on any device, vectorised over tokens: x is [T, D] for
    T = n * seq tokens of n sequences; lp the layer's parameters (leaf
    tensor; autograd flows into it).  Expert selection is by (prob desc,
    index asc); `forced_top_i` [T, k] replaces it (the indices carry no
    gradient).  Returns (y, probs, top_i)."""
    p = split_layer(cfg, lp)
    H, KV, hd = cfg.heads, cfg.kv_heads, cfg.head_dim
    T, D = x.shape
    n = T // seq
    dev = x.device
    xn = rmsnorm(x, p["attn_norm"], cfg.rms_eps)
    half = hd // 2
    i = torch.arange(half, dtype=torch.float32, device=dev)
    freq = torch.tensor(cfg.rope_theta, dtype=torch.float32, device=dev) ** (-(2.0 * i) / hd)
    ang = (torch.arange(T, device=dev) % seq).to(torch.float32)[:, None] * freq[None, :]
    cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]

    def rot(t, heads):
        th = t.view(T, heads, hd)
        a, b = th[..., :half], th[..., half:]
        return torch.cat([a * cos - b * sin, b * cos + a * sin], -1)

    q = rot(xn @ p["q"], H).view(n, seq, H, hd).transpose(1, 2)
    k = rot(xn @ p["k"], KV).view(n, seq, KV, hd).transpose(1, 2)
    v = (xn @ p["v"]).view(n, seq, KV, hd).transpose(1, 2)
    k = k.repeat_interleave(H // KV, dim=1)
    v = v.repeat_interleave(H // KV, dim=1)
    iq = torch.arange(seq, device=dev)[:, None]
    jk = torch.arange(seq, device=dev)[None, :]
    vis = (jk <= iq) & (iq - jk < cfg.sliding_window)
    s = (q @ k.transpose(-1, -2)) / (hd ** 0.5)
    pr = torch.softmax(s.masked_fill(~vis, float("-inf")), -1)
    mix = (pr @ v).transpose(1, 2).reshape(T, H * hd)
    mid = x + mix @ p["o"]
    xn2 = rmsnorm(mid, p["ffn_norm"], cfg.rms_eps)
    probs = torch.softmax(xn2 @ p["router"], -1)
    with torch.no_grad():
        order = torch.sort(probs, dim=-1, descending=True, stable=True).indices
        top_i = order[:, : cfg.top_k]
    sel = top_i if forced_top_i is None else forced_top_i
    ps = probs.gather(1, sel)
    w = ps / ps.sum(-1, keepdim=True)
    mixed = torch.zeros_like(x)
    for e in range(cfg.experts):
        tok, slot = (sel == e).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        xe = xn2[tok]
        h = torch.nn.functional.silu(xe @ p["gate"][e]) * (xe @ p["up"][e])
        mixed = mixed.index_add(0, tok, w[tok, slot, None] * (h @ p["down"][e]))
    return mid + mixed, probs, top_i
