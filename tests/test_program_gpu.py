"""Parity of the device kernel.rs programs with the oracle (fp32 path,
1e-4 relative, max-abs normalised), including the MLP workload:
batch 64, 128 -> 256 -> 128, ReLU hidden, MSE against targets."""
import numpy as np
import pytest
import torch

import oracle_ffi as orc
from dop import kernel as K

pytestmark = pytest.mark.gpu
TOL = 1e-4


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def mlp_inputs(seed=0):
    """x, targets ~ N(0,1); W ~ N(0, 1/fan_in); b = 0; seed 0."""
    prog = K.Program.mlp(64, [128, 256, 128])
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(prog.input_len, generator=g)
    t = torch.randn(prog.output_len, generator=g)
    params = torch.zeros(prog.param_len)
    for st in prog.stages:
        n = st.din * st.dout
        params[st.param_at: st.param_at + n] = torch.randn(n, generator=g) / st.din ** 0.5
    return prog, x.numpy(), t.numpy(), params.numpy()


def test_mlp_mse_matches_oracle(cuda):
    prog, x, t, params = mlp_inputs()
    cp = K.CompiledProgram(prog)
    X, P, Tt = (torch.tensor(a, device="cuda") for a in (x, params, t))
    y = cp.forward(X, P)
    loss, dy = K.mse_loss_grad(y, Tt)
    dx, dp = cp.backward(P, dy)
    torch.cuda.synchronize()
    yr = orc.program_forward_backward(prog, x, params)[0]
    dyr = (2.0 * (yr - t) / yr.size).astype(np.float32)
    _, dxr, dpr = orc.program_forward_backward(prog, x, params, dy=dyr)
    assert rel(y.cpu().numpy(), yr) < TOL
    assert abs(loss.item() - float(np.mean((yr - t) ** 2))) < 1e-4 * abs(float(np.mean((yr - t) ** 2)))
    assert rel(dx.cpu().numpy(), dxr) < TOL
    for st in prog.stages:  # per weight matrix and bias
        n = st.din * st.dout
        assert rel(dp.cpu().numpy()[st.param_at: st.param_at + n], dpr[st.param_at: st.param_at + n]) < TOL
        b = st.param_at + n
        assert rel(dp.cpu().numpy()[b: b + st.dout], dpr[b: b + st.dout]) < TOL


@pytest.mark.parametrize("prog", [K.Program.mlp(2, [3, 4, 2]), K.Program.resnet_block(2, 3, 4),
                                  K.Program.transformer_block(1, 3, 4, 5),
                                  K.Program.resnet_block(16, 64, 96),
                                  K.Program.transformer_block(2, 33, 32, 48)],
                         ids=["mlp", "resnet", "transformer", "resnet-wide", "transformer-wide"])
def test_programs_sum_loss_match_oracle(cuda, prog):
    # the crate's own test inputs (src/kernel.rs:1016-1018)
    x = K.init(prog.input_len, 0.5)
    params = K.init(prog.param_len, 0.25)
    y, dx, dp = K.forward_backward(prog, torch.tensor(x, device="cuda"),
                                   torch.tensor(params, device="cuda"))
    torch.cuda.synchronize()
    yr, dxr, dpr = orc.program_forward_backward(prog, x, params)
    # the crate's GPU tolerance |a-b| <= 1e-3 + 1e-3|b| (src/kernel.rs:858) and ours
    for a, b in ((y.cpu().numpy(), yr), (dx.cpu().numpy(), dxr), (dp.cpu().numpy(), dpr)):
        assert np.all(np.abs(a - b) <= 1e-3 + 1e-3 * np.abs(b))
        assert rel(a, b) < TOL


@pytest.mark.parametrize("prog", [K.Program.mlp(64, [128, 256, 128]),
                                  K.Program.transformer_block(2, 33, 32, 48)],
                         ids=["mlp", "transformer-wide"])
def test_program_step_replays_from_a_cuda_graph(cuda, prog):
    """Forward and backward only enqueue work on their stream, so a step
    (forward, head, backward) captured in a CUDA graph replays to the same
    bytes as the eager step."""
    x = torch.tensor(K.init(prog.input_len, 0.5), device="cuda")
    params = torch.tensor(K.init(prog.param_len, 0.25), device="cuda")
    target = torch.linspace(-1.0, 1.0, prog.output_len, device="cuda")
    cp = K.CompiledProgram(prog)
    s = torch.cuda.Stream()

    def step(stream):
        y = cp.forward(x, params, stream=stream)
        loss, dy = K.mse_loss_grad(y, target, stream=stream)
        dx, dp = cp.backward(params, dy, stream=stream)
        # the sum-loss put (dy = NULL) as well
        dx1, dp1 = cp.backward(params, None, stream=stream)
        return y, loss, dx, dp, dx1, dp1

    with torch.cuda.stream(s):
        eager = [t.clone() for t in step(s)]
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        outs = step(torch.cuda.current_stream())
    for t in outs:
        t.fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(outs, eager):
        assert torch.equal(a, b)
    cp.close()
