"""Device-side failure detection: a bounded wait that runs out.

With the wait limits shortened to 50 ms, each self-test makes one wait run
out on purpose (an mbarrier that nothing arrives at, held with TMEM
allocated; the expert exchange's barrier on a peer flag that nothing
writes).  The test checks that the call returns within a bounded time, that
the device's error word holds the wait's code, that a later tensor-core
kernel skips its work (its output is left untouched), and that after the
word is cleared the same kernel computes the right answer, so the context
stayed usable.  Nothing faults, traps or hangs.  The file sorts after the
other GPU tests, so a failure here cannot mask theirs.
"""
import time

import pytest
import torch

from dop._lib import DOP_SELFTEST_MBARRIER_CODE, check, lib

pytestmark = pytest.mark.gpu

LIMIT_NS = 50_000_000  # 50 ms per wait


@pytest.fixture
def short_limits(cuda):
    torch.cuda.synchronize()
    check(lib().dop_set_wait_limits(LIMIT_NS, LIMIT_NS))
    yield
    lib().dop_clear_device_status()
    check(lib().dop_set_wait_limits(0, 0))


def gemm(A, B, C):
    M, K = A.shape
    N = B.shape[1]
    check(lib().dop_gemm_bf16(M, N, K, A.data_ptr(), K, 0, B.data_ptr(), N, 0, C.data_ptr(), N,
                              1, 0, None))


@pytest.mark.parametrize("which, code", [(0, DOP_SELFTEST_MBARRIER_CODE), (1, 60)],
                         ids=["mbarrier", "exchange-barrier"])
def test_wait_runs_out_and_later_kernels_skip(short_limits, which, code):
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randn(256, 512, generator=g, device="cuda").bfloat16()
    B = torch.randn(512, 384, generator=g, device="cuda").bfloat16()
    C = torch.full((256, 384), -7.0, device="cuda")
    assert lib().dop_device_status() == 0
    t0 = time.perf_counter()
    check(lib().dop_selftest_wait_expiry(which, None))
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0, "the expired wait did not return promptly"
    assert lib().dop_device_status() == code
    # the sticky error: a later tensor-core kernel skips its work
    gemm(A, B, C)
    torch.cuda.synchronize()
    assert torch.equal(C, torch.full_like(C, -7.0))
    assert lib().dop_device_status() == code
    # cleared, the same launch computes again
    check(lib().dop_clear_device_status())
    assert lib().dop_device_status() == 0
    gemm(A, B, C)
    torch.cuda.synchronize()
    ref = A.double() @ B.double()
    assert ((C.double() - ref).abs().max() / ref.abs().max()).item() < 1e-5
    assert lib().dop_device_status() == 0


def test_wait_limits_reject_negative(cuda):
    assert lib().dop_set_wait_limits(-1, 0) == -1
