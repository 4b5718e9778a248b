"""The allocation-free fp32 attention backward (dop_gqa_backward_f32_noalloc).

It serves callers that may not call cudaMalloc because their device memory
belongs to another allocator.  Its scratch lives in the library's own device
memory, so this test checks, through the C ABI, that two calls in a row give
the same dq/dk/dv as dop_gqa_backward(..., DOP_F32, ...) with a caller-provided
scratch buffer (bit for bit: both run the same kernels), that the second
call is not disturbed by what the first left in the shared scratch (the
first problem is the larger, so every entry the second reads holds a value
the first wrote), and that a shape beyond the built-in scratch is rejected.  The file name sorts last so a
run that stops at the first failure has run every other test first.
"""
import pytest
import torch

from dop._lib import DOP_F32, check, lib

pytestmark = pytest.mark.gpu


def make(B, S, H, KV, hd, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    t = lambda *s: torch.randn(*s, generator=g, device="cuda")
    q, k, v = t(B * S, H, hd), t(B * S, KV, hd), t(B * S, KV, hd)
    dout = t(B * S, H, hd)
    return q, k, v, dout


def forward(B, S, H, KV, hd, W, q, k, v):
    o, lse = torch.empty_like(q), torch.empty(B, H, S, device="cuda")
    check(lib().dop_gqa_forward(B, S, H, KV, hd, W, DOP_F32, q.data_ptr(), k.data_ptr(),
                                v.data_ptr(), o.data_ptr(), lse.data_ptr(), None))
    return o, lse


def backward_with_scratch(B, S, H, KV, hd, W, q, k, v, o, dout, lse):
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(B * H * S, device="cuda")
    check(lib().dop_gqa_backward(B, S, H, KV, hd, W, DOP_F32, q.data_ptr(), k.data_ptr(),
                                 v.data_ptr(), o.data_ptr(), dout.data_ptr(), lse.data_ptr(),
                                 delta.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                 None))
    return dq, dk, dv


def backward_no_alloc(B, S, H, KV, hd, W, q, k, v, o, dout, lse):
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    check(lib().dop_gqa_backward_f32_noalloc(B, S, H, KV, hd, W, q.data_ptr(), k.data_ptr(),
                                             v.data_ptr(), o.data_ptr(), dout.data_ptr(),
                                             lse.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                             dv.data_ptr(), None))
    return dq, dk, dv


def test_no_alloc_backward_matches_the_scratch_entry_point_twice(cuda):
    # two different problems back to back: the first fills 1 x 8 x 130 =
    # 1040 delta entries, the second reads 2 x 4 x 96 = 768 of them
    for (B, S, H, KV, hd, W, seed) in [(1, 130, 8, 2, 32, 1000, 12), (2, 96, 4, 2, 64, 40, 11)]:
        q, k, v, dout = make(B, S, H, KV, hd, seed)
        o, lse = forward(B, S, H, KV, hd, W, q, k, v)
        ref = backward_with_scratch(B, S, H, KV, hd, W, q, k, v, o, dout, lse)
        got = backward_no_alloc(B, S, H, KV, hd, W, q, k, v, o, dout, lse)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)


@pytest.mark.parametrize("shape", [(1, 8193, 128, 8, 64),       # 1,048,704 > 1,048,576
                                   (1 << 22, 1 << 22, 1 << 22, 1 << 22, 64)],  # product wraps int64
                         ids=["just-over", "overflowing-product"])
def test_no_alloc_backward_rejects_shapes_beyond_its_scratch(cuda, shape):
    B, S, H, KV, hd = shape
    q = torch.empty(1, device="cuda")
    st = lib().dop_gqa_backward_f32_noalloc(B, S, H, KV, hd, S, q.data_ptr(), q.data_ptr(),
                                            q.data_ptr(), q.data_ptr(), q.data_ptr(),
                                            q.data_ptr(), q.data_ptr(), q.data_ptr(),
                                            q.data_ptr(), None)
    assert st == -1
    assert "exceeds the built-in scratch" in lib().dop_last_error().decode()
