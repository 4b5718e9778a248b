"""The small tensor-lens programs of the crate's `kernel` module.

Mirrors src/kernel.rs: `Stage` (:27-52), `Program` (:53-61) with the
builders `mlp`, `resnet_block`, `transformer_block` (:129-169) laying out the
tape and parameters exactly as `Built` does (:63-126), `init` (:173-177) and
`forward_backward` (:181-240), which here runs on the GPU through libdop.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

from . import _lib
from ._lib import DOP_STAGE_ADD, DOP_STAGE_ATTENTION, DOP_STAGE_GEMM, check, lib, ptr, stream_ptr


@dataclass
class Gemm:
    batch: int
    din: int
    dout: int
    relu: bool
    save_at: int
    mask_at: int
    param_at: int


@dataclass
class Attention:
    batch: int
    tokens: int
    dim: int
    x_at: int
    probs_at: int


@dataclass
class Add:
    from_: int
    len: int


@dataclass
class Program:
    name: str
    stages: list = field(default_factory=list)
    input_len: int = 0
    output_len: int = 0
    param_len: int = 0
    tape_f32: int = 0
    tape_u8: int = 0

    # --- builders (src/kernel.rs:78-126)
    def _gemm(self, batch, din, dout, relu):
        self.stages.append(Gemm(batch, din, dout, relu, self.tape_f32, self.tape_u8,
                                self.param_len))
        self.tape_f32 += batch * din
        if relu:
            self.tape_u8 += batch * dout
        self.param_len += din * dout + dout
        self.output_len = batch * dout

    def _attention(self, batch, tokens, dim):
        x_at = self.tape_f32
        n = batch * tokens * dim
        self.tape_f32 += n
        probs_at = self.tape_f32
        self.tape_f32 += batch * tokens * tokens
        self.stages.append(Attention(batch, tokens, dim, x_at, probs_at))
        self.output_len = n
        return x_at

    def _add(self, from_, length):
        self.stages.append(Add(from_, length))

    @staticmethod
    def mlp(batch: int, dims: list) -> "Program":
        """`Program::mlp` (src/kernel.rs:129-139): ReLU between linear layers."""
        assert len(dims) >= 2, "an MLP needs an input and an output width"
        p = Program("mlp", input_len=batch * dims[0], output_len=batch * dims[0])
        for i in range(len(dims) - 1):
            p._gemm(batch, dims[i], dims[i + 1], i + 1 < len(dims) - 1)
        return p

    @staticmethod
    def resnet_block(batch: int, dim: int, hidden: int) -> "Program":
        """`Program::resnet_block` (src/kernel.rs:141-154)."""
        p = Program("resnet_block", input_len=batch * dim, output_len=batch * dim)
        x_at = p.tape_f32
        p._gemm(batch, dim, hidden, True)
        p._gemm(batch, hidden, dim, False)
        p._add(x_at, batch * dim)
        p.output_len = batch * dim
        return p

    @staticmethod
    def transformer_block(batch: int, tokens: int, dim: int, mlp_hidden: int) -> "Program":
        """`Program::transformer_block` (src/kernel.rs:156-169)."""
        n = batch * tokens * dim
        p = Program("transformer_block", input_len=n, output_len=n)
        x_at = p._attention(batch, tokens, dim)
        p._add(x_at, n)
        y_at = p.tape_f32
        p._gemm(batch * tokens, dim, mlp_hidden, True)
        p._gemm(batch * tokens, mlp_hidden, dim, False)
        p._add(y_at, n)
        p.output_len = n
        return p

    def stages_c(self):
        arr = (_lib.StageC * max(1, len(self.stages)))()
        for i, st in enumerate(self.stages):
            c = arr[i]
            if isinstance(st, Gemm):
                c.kind, c.relu = DOP_STAGE_GEMM, int(st.relu)
                c.batch, c.din, c.dout = st.batch, st.din, st.dout
                c.save_at, c.mask_at, c.param_at = st.save_at, st.mask_at, st.param_at
            elif isinstance(st, Attention):
                c.kind = DOP_STAGE_ATTENTION
                c.batch, c.tokens, c.dim, c.x_at, c.probs_at = (st.batch, st.tokens, st.dim,
                                                                 st.x_at, st.probs_at)
            else:
                c.kind, c.from_, c.len = DOP_STAGE_ADD, st.from_, st.len
        return arr


def init(n: int, scale: float):
    """`init` (src/kernel.rs:173-177): scale * ((i % 7) + 1) / 8."""
    import numpy as np
    i = np.arange(n)
    return (np.float32(scale) * ((i % 7).astype(np.float32) + np.float32(1.0))
            / np.float32(8.0)).astype(np.float32)


class CompiledProgram:
    """A Program bound to the device (dop_program)."""

    def __init__(self, prog: Program):
        self.prog = prog
        h = C.c_void_p()
        arr = prog.stages_c()
        check(lib().dop_program_create(arr, len(prog.stages), prog.input_len, prog.output_len,
                                       prog.param_len, prog.tape_f32, prog.tape_u8, C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().dop_program_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def launches(self) -> int:
        """Kernels launched on this handle since creation."""
        return int(lib().dop_program_launches(self._h))

    def forward(self, x, params, stream=None):
        import torch
        y = torch.empty(self.prog.output_len, dtype=torch.float32, device=x.device)
        check(lib().dop_program_forward(self._h, ptr(x), ptr(params), ptr(y), stream_ptr(stream)))
        return y

    def backward(self, params, dy=None, stream=None):
        import torch
        dx = torch.empty(self.prog.input_len, dtype=torch.float32, device=params.device)
        dp = torch.empty(self.prog.param_len, dtype=torch.float32, device=params.device)
        check(lib().dop_program_backward(self._h, ptr(params), ptr(dy), ptr(dx), ptr(dp),
                                         stream_ptr(stream)))
        return dx, dp


def forward_backward(prog: Program, x, params, dy=None):
    """`kernel::forward_backward` (src/kernel.rs:181-240) on the GPU:
    returns (y, dx, dparams); dy=None is the crate's sum loss (dy = 1)."""
    cp = CompiledProgram(prog)
    try:
        y = cp.forward(x, params)
        dx, dp = cp.backward(params, dy)
        return y, dx, dp
    finally:
        cp.close()


def mse_loss_grad(y, target, stream=None):
    """MSE head: (loss, dy) with loss = mean((y-t)^2), dy = 2 (y-t) / n."""
    import torch
    loss = torch.empty((), dtype=torch.float32, device=y.device)
    dy = torch.empty_like(y)
    check(lib().dop_mse_loss_grad(ptr(y), ptr(target), y.numel(), ptr(loss), ptr(dy),
                                  stream_ptr(stream)))
    return loss, dy
