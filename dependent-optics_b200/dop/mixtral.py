"""Mixtral configuration, parameter layout and the block lens.

Python mirror of the crate's `mixtral` module (src/mixtral.rs): the same
names (`MixtralConfig`, `layout`, `parameter_count`, `init_params`,
`init_router`, `demo_batch`, `DEMO_LR`), with the block's forward (get) and
backward (put) running on the B200 through libdop's C ABI.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

from . import _lib
from ._lib import DOP_BF16, DOP_F32, DOP_IPC_HANDLE_BYTES, check, lib, ptr, stream_ptr


@dataclass
class MixtralConfig:
    """`MixtralConfig` (src/mixtral.rs:34-48)."""
    vocab: int
    dim: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    experts: int
    top_k: int
    rms_eps: float
    rope_theta: float
    sliding_window: int

    @staticmethod
    def mixtral_8x7b() -> "MixtralConfig":
        """Published Mixtral-8x7B-v0.1 configuration (src/mixtral.rs:51-66)."""
        return MixtralConfig(32_000, 4096, 32, 32, 8, 128, 14_336, 8, 2, 1e-5, 1_000_000.0, 4096)

    @staticmethod
    def demo() -> "MixtralConfig":
        """The crate's demo block (src/mixtral.rs:69-84)."""
        return MixtralConfig(32, 32, 2, 4, 2, 8, 48, 4, 2, 1e-5, 1_000_000.0, 4)

    def q_dim(self) -> int:
        return self.heads * self.head_dim

    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def group(self) -> int:
        assert self.heads % self.kv_heads == 0
        return self.heads // self.kv_heads

    def to_c(self) -> _lib.MixtralCfg:
        return _lib.MixtralCfg(self.vocab, self.dim, self.layers, self.heads, self.kv_heads,
                               self.head_dim, self.intermediate, self.experts, self.top_k,
                               self.rms_eps, self.rope_theta, self.sliding_window)


@dataclass
class LayerLayout:
    """`LayerLayout` (src/mixtral.rs:115-126), offsets into the flat P."""
    attn_norm: int
    q: int
    k: int
    v: int
    o: int
    ffn_norm: int
    router: int
    gate: list = field(default_factory=list)
    up: list = field(default_factory=list)
    down: list = field(default_factory=list)


@dataclass
class Layout:
    """`Layout` (src/mixtral.rs:104-111)."""
    embed: int
    layers: list
    final_norm: int
    lm_head: int
    total: int


def layout(cfg: MixtralConfig) -> Layout:
    """`layout` (src/mixtral.rs:128-181): every matrix row-major, contraction
    index first, W[k * dout + n]."""
    at = 0
    embed = at
    at += cfg.vocab * cfg.dim
    layers = []
    for _ in range(cfg.layers):
        ll = LayerLayout(0, 0, 0, 0, 0, 0, 0)
        ll.attn_norm = at; at += cfg.dim
        ll.q = at; at += cfg.dim * cfg.q_dim()
        ll.k = at; at += cfg.dim * cfg.kv_dim()
        ll.v = at; at += cfg.dim * cfg.kv_dim()
        ll.o = at; at += cfg.q_dim() * cfg.dim
        ll.ffn_norm = at; at += cfg.dim
        ll.router = at; at += cfg.dim * cfg.experts
        for _e in range(cfg.experts):
            ll.gate.append(at); at += cfg.dim * cfg.intermediate
            ll.up.append(at); at += cfg.dim * cfg.intermediate
            ll.down.append(at); at += cfg.intermediate * cfg.dim
        layers.append(ll)
    final_norm = at
    at += cfg.dim
    lm_head = at
    at += cfg.dim * cfg.vocab
    return Layout(embed, layers, final_norm, lm_head, at)


def layer_params(cfg: MixtralConfig) -> int:
    """Floats in one layer's parameter slice (attn_norm .. last expert's down)."""
    lay = layout(MixtralConfig(**{**cfg.__dict__, "layers": 1}))
    return lay.final_norm - lay.layers[0].attn_norm


def layer_layout(cfg: MixtralConfig) -> _lib.LayerLayout:
    """Offsets inside one layer slice, from the library (dop_layer_layout_of)."""
    out = _lib.LayerLayout()
    check(lib().dop_layer_layout_of(C.byref(cfg.to_c()), C.byref(out)))
    return out


def parameter_count(cfg: MixtralConfig) -> int:
    """`parameter_count` (src/mixtral.rs:183-185)."""
    return layout(cfg).total


def init_params(cfg: MixtralConfig) -> list:
    """`init_params` (src/mixtral.rs:190-198): 0.02 * (i % 5 + 1)."""
    import numpy as np
    n = layout(cfg).total
    i = np.arange(n)
    return (np.float32(0.02) * ((i % 5).astype(np.float32) + np.float32(1.0))).astype(np.float32)


def init_router(cfg: MixtralConfig, params) -> None:
    """`init_router` (src/mixtral.rs:200-210)."""
    import numpy as np
    lay = layout(cfg)
    d = np.arange(cfg.dim, dtype=np.float32)[:, None]
    e = np.arange(cfg.experts, dtype=np.float32)[None, :]
    block = (np.float32(0.05) * (e + np.float32(1.0)) + np.float32(0.001) * d).astype(np.float32)
    for layer in lay.layers:
        params[layer.router: layer.router + cfg.dim * cfg.experts] = block.reshape(-1)


def demo_batch(cfg: MixtralConfig):
    """`demo_batch` (src/mixtral.rs:1003-1009)."""
    batch, seq = 2, 8
    tokens = [(i * 5 + 1) % cfg.vocab for i in range(batch * seq)]
    targets = [(t + 3) % cfg.vocab for t in tokens]
    return batch, seq, tokens, targets


DEMO_LR = 0.05


class Block:
    """One Mixtral block as a tensor lens on the GPU.

    `forward(params, x) -> y` is the get of `forward_layer`
    (src/mixtral.rs:291-380) and keeps its residual in the handle;
    `backward(params, dy, dparams) -> dx` is the put of `backward_layer`
    (src/mixtral.rs:434-598) and ACCUMULATES into `dparams` like the crate's
    `add_assign` into `grad`.  Tensors are torch CUDA tensors: `params` is the
    layer slice (fp32 for precision DOP_F32, bf16 for DOP_BF16), x/y/dy/dx are
    fp32 [batch*seq, dim], dparams is fp32.
    """

    def __init__(self, cfg: MixtralConfig, batch: int, seq: int, precision: int = DOP_F32,
                 ep: tuple | None = None):
        """`ep = (rank, world)` makes an expert-parallel block (bf16; rank owns
        experts [rank*E/world, (rank+1)*E/world)); connect it to its peers
        with `dop.parallel.connect_expert_parallel` before the first forward."""
        self.cfg, self.batch, self.seq, self.precision = cfg, batch, seq, precision
        self.ep = ep
        h = C.c_void_p()
        if ep is None:
            check(lib().dop_block_create(C.byref(cfg.to_c()), batch, seq, precision, C.byref(h)))
        else:
            rank, world = ep
            check(lib().dop_block_create_ep(C.byref(cfg.to_c()), batch, seq, precision, rank,
                                            world, C.byref(h)))
        self._h = h
        self._bias = None

    def ep_handle(self) -> bytes:
        """This rank's workspace IPC handle (DOP_IPC_HANDLE_BYTES bytes)."""
        buf = C.create_string_buffer(DOP_IPC_HANDLE_BYTES)
        check(lib().dop_block_ep_handle(self._h, buf))
        return buf.raw

    def ep_connect(self, handles: bytes) -> None:
        """Map the peers' workspaces (world handles concatenated in rank order)."""
        assert len(handles) == DOP_IPC_HANDLE_BYTES * self.ep[1]
        buf = C.create_string_buffer(handles, len(handles))
        check(lib().dop_block_ep_connect(self._h, buf))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().dop_block_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def handle(self):
        return self._h

    def set_router_bias(self, bias) -> None:
        """Per-expert logit bias added before the router softmax (fp32 [E])."""
        self._bias = bias
        check(lib().dop_block_set_router_bias(self._h, ptr(bias)))

    def forward(self, params, x, y=None, stream=None):
        import torch
        if y is None:
            y = torch.empty_like(x)
        check(lib().dop_block_forward(self._h, ptr(params), ptr(x), ptr(y), stream_ptr(stream)))
        return y

    def backward(self, params, dy, dparams, dx=None, stream=None):
        import torch
        if dx is None:
            dx = torch.empty_like(dy)
        check(lib().dop_block_backward(self._h, ptr(params), ptr(dy), ptr(dx), ptr(dparams),
                                       stream_ptr(stream)))
        return dx

    def routing(self):
        """(top_i int32 [T,k], top_w, top_p, router_probs) of the last forward."""
        import torch
        T = self.batch * self.seq
        k, E = self.cfg.top_k, self.cfg.experts
        ti = torch.empty(T, k, dtype=torch.int32, device="cuda")
        tw = torch.empty(T, k, dtype=torch.float32, device="cuda")
        tp = torch.empty(T, k, dtype=torch.float32, device="cuda")
        pr = torch.empty(T, E, dtype=torch.float32, device="cuda")
        check(lib().dop_block_routing(self._h, ptr(ti), ptr(tw), ptr(tp), ptr(pr), None))
        torch.cuda.synchronize()
        return ti, tw, tp, pr

    def permutation(self):
        """(slot_row [T*k], seg_off [E+1], row_token [rows]) of the last forward."""
        import torch
        T = self.batch * self.seq
        rows = lib().dop_block_permuted_rows(self._h)
        sr = torch.empty(T * self.cfg.top_k, dtype=torch.int32, device="cuda")
        so = torch.empty(self.cfg.experts + 1, dtype=torch.int32, device="cuda")
        rt = torch.empty(rows, dtype=torch.int32, device="cuda")
        check(lib().dop_block_permutation(self._h, ptr(sr), ptr(so), ptr(rt), None))
        torch.cuda.synchronize()
        return sr, so, rt

    def ffn_input(self):
        """mid = x + attention [T, D] (fp32) of the last forward: the router's input."""
        import torch
        mid = torch.empty(self.batch * self.seq, self.cfg.dim, dtype=torch.float32, device="cuda")
        check(lib().dop_block_ffn_input(self._h, ptr(mid), None))
        torch.cuda.synchronize()
        return mid

    def set_adjoint_stream(self, stream) -> None:
        """Make `stream` (a torch.cuda.Stream or None) wait, in every backward,
        until the experts' parameter adjoints are final."""
        check(lib().dop_block_set_adjoint_stream(self._h, stream_ptr(stream)))

    def set_timing(self, on: bool = True) -> None:
        check(lib().dop_block_set_timing(self._h, int(on)))

    def phase_times(self) -> list:
        """[(phase name, ms)] of the last forward + backward (timing on)."""
        out = []
        for i in range(lib().dop_block_phase_count(self._h)):
            name, ms = C.c_char_p(), C.c_float()
            check(lib().dop_block_phase(self._h, i, C.byref(name), C.byref(ms)))
            out.append((name.value.decode(), ms.value))
        return out

    def launches(self) -> int:
        return int(lib().dop_block_launches(self._h))

    def workspace_bytes(self) -> int:
        return int(lib().dop_block_workspace_bytes(self._h))


class LossGrad:
    """`LossGrad` (src/mixtral.rs:231-235): loss, grad and logits (device tensors)."""

    def __init__(self, loss, grad, logits):
        self.loss, self.grad, self.logits = loss, grad, logits


class Model:
    """The whole model lens on the GPU (dop_model)."""

    def __init__(self, cfg: MixtralConfig, batch: int, seq: int, precision: int = DOP_F32):
        self.cfg, self.batch, self.seq, self.precision = cfg, batch, seq, precision
        h = C.c_void_p()
        check(lib().dop_model_create(C.byref(cfg.to_c()), batch, seq, precision, C.byref(h)))
        self._h = h
        self.n_params = int(lib().dop_model_parameter_count(h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().dop_model_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward_backward(self, params, tokens, targets, stream=None) -> LossGrad:
        import torch
        dev = params.device
        T, V = self.batch * self.seq, self.cfg.vocab
        loss = torch.empty((), dtype=torch.float32, device=dev)
        grad = torch.empty(self.n_params, dtype=torch.float32, device=dev)
        logits = torch.empty(T, V, dtype=torch.float32, device=dev)
        check(lib().dop_model_forward_backward(self._h, ptr(params), ptr(tokens), ptr(targets),
                                               ptr(loss), ptr(grad), ptr(logits),
                                               stream_ptr(stream)))
        return LossGrad(loss, grad, logits)


def forward_backward(cfg: MixtralConfig, params, tokens, targets, batch: int, seq: int,
                     precision: int = DOP_F32) -> LossGrad:
    """`mixtral::forward_backward` (src/mixtral.rs:245-261) on the GPU.
    params: device tensor of the whole flat parameter vector; tokens/targets:
    device int64 tensors of batch*seq ids."""
    m = Model(cfg, batch, seq, precision)
    try:
        return m.forward_backward(params, tokens, targets)
    finally:
        import torch
        torch.cuda.synchronize()
        m.close()


def sgd_step(params, grad, lr: float) -> None:
    """`sgd_step` (src/mixtral.rs:994-1001) on device tensors: p -= lr * g."""
    check(lib().dop_sgd_step(ptr(params), ptr(grad), params.numel(), lr, None))
