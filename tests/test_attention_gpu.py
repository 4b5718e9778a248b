"""The sliding-window GQA lens (dop_gqa_forward / dop_gqa_backward) against
a float64 torch autograd reference on the same bf16 inputs; head_dim 128
runs the tcgen05 flash kernels.  Bars: o within 1e-2, lse within 1e-3
absolute, dq/dk/dv within 2e-2 (max-abs normalised)."""
import pytest
import torch

from dop._lib import DOP_BF16, DOP_F32, check, lib

pytestmark = pytest.mark.gpu


def reference(q, k, v, dout, B, S, H, KV, hd, W):
    q64, k64, v64 = (t.double().requires_grad_(True) for t in (q, k, v))
    qh = q64.view(B, S, H, hd).transpose(1, 2)
    kh = k64.view(B, S, KV, hd).transpose(1, 2).repeat_interleave(H // KV, 1)
    vh = v64.view(B, S, KV, hd).transpose(1, 2).repeat_interleave(H // KV, 1)
    s = qh @ kh.transpose(-1, -2) / hd ** 0.5
    i = torch.arange(S, device=q.device)[:, None]
    j = torch.arange(S, device=q.device)[None, :]
    s = s.masked_fill(~((j <= i) & (i - j < W)), float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = (torch.softmax(s, -1) @ vh).transpose(1, 2).reshape(B * S, H, hd)
    o.backward(dout.double())
    return o.detach(), lse.detach(), q64.grad, k64.grad, v64.grad


def rel(a, b):
    return ((a.double() - b.double()).abs().max() / b.double().abs().max()).item()


@pytest.mark.parametrize("B,S,H,KV,W,qs", [(2, 200, 4, 2, 150, 1.0), (1, 256, 2, 2, 10_000, 1.0),
                                            (1, 384, 8, 2, 100, 1.0), (2, 130, 4, 1, 64, 1.0),
                                            (1, 1024, 4, 2, 10_000, 3.0)],
                         ids=["ragged-window", "causal", "gqa4", "mqa", "wide-scores"])
def test_gqa_tensor_core_matches_float64(cuda, B, S, H, KV, W, qs):
    """qs scales q: wide score distributions make rows of one warp raise
    their running max at different key tiles (the divergent O rescale)."""
    hd = 128
    g = torch.Generator(device="cuda").manual_seed(S + H)
    q = (qs * torch.randn(B * S, H, hd, generator=g, device="cuda")).bfloat16()
    k = torch.randn(B * S, KV, hd, generator=g, device="cuda").bfloat16()
    v = torch.randn(B * S, KV, hd, generator=g, device="cuda").bfloat16()
    dout = torch.randn(B * S, H, hd, generator=g, device="cuda").bfloat16()
    o = torch.empty_like(q)
    lse = torch.empty(B, H, S, device="cuda")
    check(lib().dop_gqa_forward(B, S, H, KV, hd, W, DOP_BF16, q.data_ptr(), k.data_ptr(),
                                v.data_ptr(), o.data_ptr(), lse.data_ptr(), None))
    dq = torch.empty(B * S, H, hd, device="cuda")
    dk = torch.empty(B * S, KV, hd, device="cuda")
    dv = torch.empty(B * S, KV, hd, device="cuda")
    delta = torch.empty(B * H * S, device="cuda")
    check(lib().dop_gqa_backward(B, S, H, KV, hd, W, DOP_BF16, q.data_ptr(), k.data_ptr(),
                                 v.data_ptr(), o.data_ptr(), dout.data_ptr(), lse.data_ptr(),
                                 delta.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                 None))
    torch.cuda.synchronize()
    assert lib().dop_device_status() == 0
    o_r, lse_r, dq_r, dk_r, dv_r = reference(q, k, v, dout, B, S, H, KV, hd, W)
    assert rel(o, o_r) < 1e-2
    assert (lse.double() - lse_r).abs().max().item() < 1e-3
    assert rel(dq, dq_r) < 2e-2
    assert rel(dk, dk_r) < 2e-2
    assert rel(dv, dv_r) < 2e-2


@pytest.mark.parametrize("B,S,H,KV,hd,W", [(2, 70, 4, 2, 64, 33), (1, 200, 6, 2, 128, 150),
                                             (2, 130, 8, 1, 16, 1000), (1, 96, 2, 2, 38, 50),
                                             (3, 64, 12, 3, 64, 64), (1, 300, 10, 1, 64, 200)],
                         ids=["gqa2-hd64", "gqa3-hd128", "mqa8-hd16", "mha-hd38", "gqa4-one-tile",
                              "mqa10-hd64"])
def test_gqa_f32_cuda_core_matches_float64(cuda, B, S, H, KV, hd, W):
    """fp32 CUDA-core attention: padded head dims 32 / 64 / 128, a head_dim
    that is not a multiple of 4 (scalar loads), dK/dV clusters of 1, 2, 3, 4,
    5 and 8 CTAs (10 query heads on one KV head: 5 CTAs of 2 heads each),
    ragged last tiles.  Bar 1e-5 against float64; the backward is bitwise
    reproducible."""
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn(B * S, H, hd, generator=g, device="cuda")
    k = torch.randn(B * S, KV, hd, generator=g, device="cuda")
    v = torch.randn(B * S, KV, hd, generator=g, device="cuda")
    dout = torch.randn(B * S, H, hd, generator=g, device="cuda")
    o, lse = torch.empty_like(q), torch.empty(B, H, S, device="cuda")
    check(lib().dop_gqa_forward(B, S, H, KV, hd, W, DOP_F32, q.data_ptr(), k.data_ptr(),
                                v.data_ptr(), o.data_ptr(), lse.data_ptr(), None))
    outs = []
    for _ in range(2):
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        delta = torch.empty(B * H * S, device="cuda")
        check(lib().dop_gqa_backward(B, S, H, KV, hd, W, DOP_F32, q.data_ptr(), k.data_ptr(),
                                     v.data_ptr(), o.data_ptr(), dout.data_ptr(), lse.data_ptr(),
                                     delta.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                     dv.data_ptr(), None))
        outs.append((dq, dk, dv))
    torch.cuda.synchronize()
    o_r, lse_r, dq_r, dk_r, dv_r = reference(q, k, v, dout, B, S, H, KV, hd, W)
    dq, dk, dv = outs[0]
    for a, b in ((o, o_r), (dq, dq_r), (dk, dk_r), (dv, dv_r)):
        assert rel(a, b) < 1e-5
    assert (lse.double() - lse_r).abs().max().item() < 1e-5
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)


def test_exp2_polynomial_error_bound(cuda):
    """The FMA-pipe exponential of the forward softmax (dop_exp2_poly, a
    quarter of its exponentials) against exp2 in float64: relative error
    below 1e-4 over [-125, 100) (the fit's bound is 7.6e-5; a bf16
    probability rounds at 3.9e-3), and below -125 a value under 2e-38, where
    the MUFU's flush-to-zero exp2 gives 0."""
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.cat([torch.linspace(-125.0, 99.99, 1_000_001, device="cuda"),
                   torch.rand(1_000_000, generator=g, device="cuda") * -20.0,
                   torch.tensor([0.0, -0.5, 0.5, 8.0, -1e-30], device="cuda")])
    y = torch.empty_like(x)
    check(lib().dop_exp2_poly(x.data_ptr(), y.data_ptr(), x.numel(), None))
    ref = torch.exp2(x.double())
    assert ((y.double() - ref).abs() / ref).max().item() < 1e-4
    lo = torch.tensor([-125.5, -126.0, -200.0, -1e30, float("-inf")], device="cuda")
    ylo = torch.empty_like(lo)
    check(lib().dop_exp2_poly(lo.data_ptr(), ylo.data_ptr(), lo.numel(), None))
    torch.cuda.synchronize()
    assert bool(((ylo >= 0) & (ylo < 2e-38)).all())
