"""Writes tests/golden/golden.npz: the oracle's outputs on fixed inputs.

The crate (Rust) cannot run here and ships no numeric golden vectors, so
these fixtures are the oracle's own answers, taken after the oracle was
pinned by the crate's tests (tests/test_oracle.py).  They freeze those
answers: tests/test_golden.py checks that the oracle still reproduces them,
and device tests can compare against them without running the oracle.

Cases:
- demo: the crate's demo model (src/mixtral.rs:69-84) with its
  deterministic parameters, router and batch (init_params, init_router,
  demo_batch; :190-210, :1003-1009): loss, parameter gradient, logits.
- prog_mlp / prog_resnet / prog_transformer: the kernel.rs test programs
  on the crate's own inputs (init(n, 0.5) and init(n, 0.25), sum loss;
  src/kernel.rs:1016-1018): y, dx, dparams.
- c1: the MLP workload (batch 64, 128 -> 256 -> 128, ReLU, MSE against
  targets; seed 0): y, loss, dx, and dparams sampled every 16th element.
- block: one f32 Mixtral block (d 32, 4/2 heads, hd 8, 4 experts x 24,
  top-2, window 5, batch 2, seq 7; seed 0): y, dx, dparams, top_i.

Run from the repository root: python tests/golden/make_golden.py
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT / "dependent-optics_b200"), str(ROOT / "tests")]

import oracle_ffi as orc  # noqa: E402
from dop import kernel as K  # noqa: E402
from dop.mixtral import MixtralConfig, demo_batch, init_params, init_router  # noqa: E402

C1_STRIDE = 16


def block_cfg():
    return MixtralConfig(vocab=32, dim=32, layers=1, heads=4, kv_heads=2, head_dim=8,
                         intermediate=24, experts=4, top_k=2, rms_eps=1e-5, rope_theta=1e4,
                         sliding_window=5)


def c1_inputs():
    """x, targets ~ N(0,1); W ~ N(0, 1/fan_in); b = 0 (torch generator, seed 0)."""
    import torch
    prog = K.Program.mlp(64, [128, 256, 128])
    g = torch.Generator().manual_seed(0)
    x = torch.randn(prog.input_len, generator=g)
    t = torch.randn(prog.output_len, generator=g)
    params = torch.zeros(prog.param_len)
    for st in prog.stages:
        n = st.din * st.dout
        params[st.param_at: st.param_at + n] = torch.randn(n, generator=g) / st.din ** 0.5
    return prog, x.numpy(), t.numpy(), params.numpy()


def block_inputs():
    import torch
    cfg = block_cfg()
    g = torch.Generator().manual_seed(0)
    lp = (torch.randn(orc.layer_params(cfg), generator=g) * 0.2).float().numpy()
    x = torch.randn(2 * 7 * cfg.dim, generator=g).float().numpy()
    dy = torch.randn(2 * 7 * cfg.dim, generator=g).float().numpy()
    return cfg, lp, x, dy


def compute() -> dict:
    out = {}
    cfg = MixtralConfig.demo()
    p = init_params(cfg)
    init_router(cfg, p)
    batch, seq, tokens, targets = demo_batch(cfg)
    loss, grad, logits = orc.mixtral_forward_backward(cfg, p, tokens, targets, batch, seq)
    out.update(demo_loss=np.float32(loss), demo_grad=grad, demo_logits=logits)
    progs = {"mlp": K.Program.mlp(2, [3, 4, 2]), "resnet": K.Program.resnet_block(2, 3, 4),
             "transformer": K.Program.transformer_block(1, 3, 4, 5)}
    for name, prog in progs.items():
        y, dx, dp = orc.program_forward_backward(prog, K.init(prog.input_len, 0.5),
                                                 K.init(prog.param_len, 0.25))
        out.update({f"prog_{name}_y": y, f"prog_{name}_dx": dx, f"prog_{name}_dp": dp})
    prog, x, t, params = c1_inputs()
    y = orc.program_forward_backward(prog, x, params)[0]
    dy = (np.float32(2.0) * (y - t) / np.float32(y.size)).astype(np.float32)
    _, dx, dp = orc.program_forward_backward(prog, x, params, dy=dy)
    out.update(c1_y=y, c1_loss=np.float32(np.mean((y.astype(np.float64) - t) ** 2)), c1_dx=dx,
               c1_dp_sampled=dp[::C1_STRIDE])
    cfg, lp, x, dy = block_inputs()
    r = orc.block_forward(cfg, lp, x, 2, 7)
    dxb, dlp = orc.block_backward(cfg, lp, r, dy)
    out.update(block_y=r.y.copy(), block_dx=dxb, block_dparams=dlp,
               block_top_i=r.routing()[0].astype(np.int64))
    return out


if __name__ == "__main__":
    path = Path(__file__).resolve().parent / "golden.npz"
    np.savez_compressed(path, **compute())
    print(path, path.stat().st_size, "bytes")
