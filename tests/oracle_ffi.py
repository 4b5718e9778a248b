"""ctypes binding of the CPU oracle (oracle/liboracle.so).

Test infrastructure: the oracle is the checker the CUDA path is compared
against.  It is built from oracle/oracle.cpp by oracle/Makefile.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
ORACLE_DIR = ROOT / "oracle"
ORACLE_SO = ORACLE_DIR / "liboracle.so"


class MixtralCfg(C.Structure):
    """dop_mixtral_cfg (include/dop.h), the oracle's config argument."""
    _fields_ = [(n, C.c_int64) for n in (
        "vocab", "dim", "layers", "heads", "kv_heads", "head_dim", "intermediate",
        "experts", "top_k")] + [("rms_eps", C.c_float), ("rope_theta", C.c_float),
                                ("sliding_window", C.c_int64)]


class StageC(C.Structure):
    """dop_stage (include/dop.h)."""
    _fields_ = [("kind", C.c_int32), ("relu", C.c_int32)] + [(n, C.c_int64) for n in (
        "batch", "din", "dout", "save_at", "mask_at", "param_at", "tokens", "dim", "x_at",
        "probs_at", "from_", "len")]


def _cfg(cfg) -> MixtralCfg:
    """Any object with the MixtralConfig fields, as the oracle's struct."""
    return MixtralCfg(*(getattr(cfg, f) for f, _ in MixtralCfg._fields_))


def _stages(prog):
    """A program's stages as an array of the oracle's StageC."""
    arr = (StageC * len(prog.stages))()
    for i, st in enumerate(prog.stages_c()):
        C.memmove(C.byref(arr[i]), C.byref(st), C.sizeof(StageC))
    return arr


_lib = None
F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
I64P = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
        L = C.CDLL(str(ORACLE_SO))
        L.orc_layer_params.restype = C.c_int64
        L.orc_layer_params.argtypes = [C.POINTER(MixtralCfg)]
        L.orc_layer_offsets.restype = None
        L.orc_layer_offsets.argtypes = [C.POINTER(MixtralCfg), I64P]
        L.orc_parameter_count.restype = C.c_int64
        L.orc_parameter_count.argtypes = [C.POINTER(MixtralCfg)]
        L.orc_block_forward.restype = C.c_void_p
        L.orc_block_forward.argtypes = [C.POINTER(MixtralCfg), F32P, F32P, C.c_int64, C.c_int64,
                                        C.c_void_p, C.c_void_p, F32P]
        L.orc_block_backward.restype = None
        L.orc_block_backward.argtypes = [C.POINTER(MixtralCfg), F32P, C.c_void_p, F32P, F32P, F32P]
        L.orc_tape_routing.restype = None
        L.orc_tape_routing.argtypes = [C.c_void_p, I64P, F32P, F32P, F32P]
        L.orc_tape_free.restype = None
        L.orc_tape_free.argtypes = [C.c_void_p]
        L.orc_mixtral_forward_backward.restype = C.c_float
        L.orc_mixtral_forward_backward.argtypes = [C.POINTER(MixtralCfg), F32P, I64P, I64P,
                                                   C.c_int64, C.c_int64, F32P, C.c_void_p]
        L.orc_sgd_step.restype = C.c_float
        L.orc_sgd_step.argtypes = [F32P, F32P, C.c_int64, C.c_float]
        L.orc_router_stage.restype = None
        L.orc_router_stage.argtypes = [C.POINTER(MixtralCfg), F32P, F32P, C.c_int64, C.c_void_p,
                                       I64P, F32P, F32P, F32P]
        L.orc_set_literal.restype = None
        L.orc_set_literal.argtypes = [C.c_int]
        L.orc_set_threads.restype = C.c_int
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_program_forward_backward.restype = None
        L.orc_program_forward_backward.argtypes = [
            C.POINTER(StageC), C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64, F32P, F32P,
            C.c_void_p, F32P, C.POINTER(C.c_int64), F32P, F32P]
        _lib = L
    return _lib


def set_literal(on: bool) -> None:
    """True: the crate's literal loop order on one thread; False (default):
    interchanged, threaded loop nests with the same per-output sums."""
    lib().orc_set_literal(1 if on else 0)


def set_threads(n: int) -> int:
    """Host threads the oracle may use (0 = all); returns the number in effect."""
    return int(lib().orc_set_threads(int(n)))


def layer_offsets(cfg) -> dict:
    """Offsets inside one layer slice (src/mixtral.rs:135-171): attn_norm, q,
    k, v, o, ffn_norm, router, gate0, up0, down0, expert_stride, total."""
    E = cfg.experts
    out = np.zeros(7 + 3 * E, np.int64)
    lib().orc_layer_offsets(C.byref(_cfg(cfg)), out)
    names = ("attn_norm", "q", "k", "v", "o", "ffn_norm", "router")
    d = {n: int(out[i]) for i, n in enumerate(names)}
    d["gate0"], d["up0"], d["down0"] = int(out[7]), int(out[7 + E]), int(out[7 + 2 * E])
    d["expert_stride"] = int(out[8] - out[7]) if E > 1 else 3 * cfg.dim * cfg.intermediate
    d["total"] = layer_params(cfg)
    return d


def layer_params(cfg) -> int:
    return int(lib().orc_layer_params(C.byref(_cfg(cfg))))


def parameter_count(cfg) -> int:
    return int(lib().orc_parameter_count(C.byref(_cfg(cfg))))


class BlockResult:
    def __init__(self, y, tape, cfg, T):
        self.y, self._tape, self.cfg, self.T = y, tape, cfg, T

    def routing(self):
        k, E = self.cfg.top_k, self.cfg.experts
        ti = np.zeros(self.T * k, np.int64)
        tp = np.zeros(self.T * k, np.float32)
        tw = np.zeros(self.T * k, np.float32)
        pr = np.zeros(self.T * E, np.float32)
        lib().orc_tape_routing(self._tape, ti, tp, tw, pr)
        return ti.reshape(self.T, k), tw.reshape(self.T, k), tp.reshape(self.T, k), pr.reshape(self.T, E)

    def __del__(self):
        if getattr(self, "_tape", None):
            try:
                lib().orc_tape_free(self._tape)
            except Exception:  # interpreter shutdown
                pass
            self._tape = None


def block_forward(cfg, lp, x, batch, seq, bias=None, forced_top_i=None) -> BlockResult:
    lp = np.ascontiguousarray(lp, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros_like(x)
    b = f = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.float32)
        b = bias.ctypes.data_as(C.c_void_p)
    if forced_top_i is not None:
        forced_top_i = np.ascontiguousarray(forced_top_i, np.int64)
        f = forced_top_i.ctypes.data_as(C.c_void_p)
    tape = lib().orc_block_forward(C.byref(_cfg(cfg)), lp, x, batch, seq, b, f, y)
    r = BlockResult(y, tape, cfg, batch * seq)
    r._keep = (bias, forced_top_i)
    return r


def block_backward(cfg, lp, res: BlockResult, dy, dlp=None):
    lp = np.ascontiguousarray(lp, np.float32)
    dy = np.ascontiguousarray(dy, np.float32)
    dx = np.zeros_like(dy)
    if dlp is None:
        dlp = np.zeros_like(lp)
    lib().orc_block_backward(C.byref(_cfg(cfg)), lp, res._tape, dy, dx, dlp)
    return dx, dlp


def router_stage(cfg, lp, mid, bias=None):
    """The router stage of forward_layer on the feed-forward input `mid`
    [T, D]: (top_i [T, k], top_w, top_p, router_probs [T, E])."""
    lp = np.ascontiguousarray(lp, np.float32)
    mid = np.ascontiguousarray(mid, np.float32).reshape(-1)
    T = mid.size // cfg.dim
    k, E = cfg.top_k, cfg.experts
    ti = np.zeros(T * k, np.int64)
    tp = np.zeros(T * k, np.float32)
    tw = np.zeros(T * k, np.float32)
    pr = np.zeros(T * E, np.float32)
    b = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.float32)
        b = bias.ctypes.data_as(C.c_void_p)
    lib().orc_router_stage(C.byref(_cfg(cfg)), lp, mid, T, b, ti, tp, tw, pr)
    return ti.reshape(T, k), tw.reshape(T, k), tp.reshape(T, k), pr.reshape(T, E)


def mixtral_forward_backward(cfg, P, tokens, targets, batch, seq):
    P = np.ascontiguousarray(P, np.float32)
    grad = np.zeros_like(P)
    logits = np.zeros(batch * seq * cfg.vocab, np.float32)
    loss = lib().orc_mixtral_forward_backward(
        C.byref(_cfg(cfg)), P, np.asarray(tokens, np.int64), np.asarray(targets, np.int64),
        batch, seq, grad, logits.ctypes.data_as(C.c_void_p))
    return float(loss), grad, logits


def sgd_step(params, grad, lr):
    return float(lib().orc_sgd_step(params, np.ascontiguousarray(grad, np.float32), params.size, lr))


def program_forward_backward(prog, x, params, dy=None):
    arr = _stages(prog)
    x = np.ascontiguousarray(x, np.float32)
    params = np.ascontiguousarray(params, np.float32)
    y = np.zeros(max(prog.output_len, prog.input_len, 1) * 4, np.float32)
    ylen = C.c_int64(0)
    dx = np.zeros(prog.input_len, np.float32)
    dp = np.zeros(prog.param_len, np.float32)
    dyp = None
    if dy is not None:
        dy = np.ascontiguousarray(dy, np.float32)
        dyp = dy.ctypes.data_as(C.c_void_p)
    lib().orc_program_forward_backward(arr, len(prog.stages), prog.input_len, prog.param_len,
                                       prog.tape_f32, prog.tape_u8, x, params, dyp, y,
                                       C.byref(ylen), dx, dp)
    return y[: ylen.value].copy(), dx, dp
