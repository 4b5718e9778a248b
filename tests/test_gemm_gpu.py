"""The tensor-core GEMM (tcgen05 + TMA + TMEM) against a float64 product of
the same bf16 operands, for every operand major, ragged edges, bf16 output
and accumulation (dop_gemm_bf16)."""
import ctypes as C

import pytest
import torch

from dop._lib import check, lib

pytestmark = pytest.mark.gpu


def run(M, N, K, a_t, b_t, c_f32=True, accumulate=False, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K, generator=g, device="cuda").bfloat16()
    B = torch.randn(K, N, generator=g, device="cuda").bfloat16()
    As = A.t().contiguous() if a_t else A  # stored [K, M] when M-major
    Bs = B.t().contiguous() if b_t else B  # stored [N, K] when K-major
    lda = As.shape[1]
    ldb = Bs.shape[1]
    Cm = torch.randn(M, N, generator=g, device="cuda") if accumulate else torch.zeros(M, N, device="cuda")
    C0 = Cm.clone()
    if not c_f32:
        Cm = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    check(lib().dop_gemm_bf16(M, N, K, As.data_ptr(), lda, int(a_t), Bs.data_ptr(), ldb, int(b_t),
                              Cm.data_ptr(), N, int(c_f32), int(accumulate), None))
    torch.cuda.synchronize()
    assert lib().dop_device_status() == 0
    ref = A.double() @ B.double()
    if accumulate:
        ref = ref + C0.double()
    err = (Cm.double() - ref).abs().max().item() / ref.abs().max().item()
    return err


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
def test_gemm_majors(cuda, a_t, b_t):
    assert run(256, 512, 256, a_t, b_t) < 1e-5


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
def test_gemm_ragged_edges(cuda, a_t, b_t):
    assert run(200, 296, 136, a_t, b_t) < 1e-5


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
def test_gemm_pair_partial_tile(cuda, a_t, b_t):
    # 296 rows on pairs of SMs: the last 256-row tile has 40 rows in its first
    # CTA's half and none in its second's; ragged N and K as well (strides
    # stay multiples of 16 bytes, as TMA requires)
    assert run(296, 264, 200, a_t, b_t) < 1e-5


def test_gemm_bf16_out_and_accumulate(cuda):
    assert run(384, 768, 512, False, False, c_f32=False) < 8e-3
    assert run(384, 768, 512, True, False, accumulate=True) < 1e-5


def test_gemm_large_many_tiles(cuda):
    # more tiles than SMs: exercises the persistent schedule and both TMEM buffers
    assert run(2048, 4096, 1024, False, False) < 1e-5
    assert run(1024, 1024, 4096, True, False) < 1e-5
