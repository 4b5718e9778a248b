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

import sys
sys.path.insert(0, str(ROOT / "dependent-optics_b200"))
from dop._lib import MixtralCfg, StageC  # noqa: E402

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
        L.orc_program_forward_backward.restype = None
        L.orc_program_forward_backward.argtypes = [
            C.POINTER(StageC), C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64, F32P, F32P,
            C.c_void_p, F32P, C.POINTER(C.c_int64), F32P, F32P]
        _lib = L
    return _lib


def layer_params(cfg) -> int:
    return int(lib().orc_layer_params(C.byref(cfg.to_c())))


def parameter_count(cfg) -> int:
    return int(lib().orc_parameter_count(C.byref(cfg.to_c())))


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
    tape = lib().orc_block_forward(C.byref(cfg.to_c()), lp, x, batch, seq, b, f, y)
    r = BlockResult(y, tape, cfg, batch * seq)
    r._keep = (bias, forced_top_i)
    return r


def block_backward(cfg, lp, res: BlockResult, dy, dlp=None):
    lp = np.ascontiguousarray(lp, np.float32)
    dy = np.ascontiguousarray(dy, np.float32)
    dx = np.zeros_like(dy)
    if dlp is None:
        dlp = np.zeros_like(lp)
    lib().orc_block_backward(C.byref(cfg.to_c()), lp, res._tape, dy, dx, dlp)
    return dx, dlp


def mixtral_forward_backward(cfg, P, tokens, targets, batch, seq):
    P = np.ascontiguousarray(P, np.float32)
    grad = np.zeros_like(P)
    logits = np.zeros(batch * seq * cfg.vocab, np.float32)
    loss = lib().orc_mixtral_forward_backward(
        C.byref(cfg.to_c()), P, np.asarray(tokens, np.int64), np.asarray(targets, np.int64),
        batch, seq, grad, logits.ctypes.data_as(C.c_void_p))
    return float(loss), grad, logits


def sgd_step(params, grad, lr):
    return float(lib().orc_sgd_step(params, np.ascontiguousarray(grad, np.float32), params.size, lr))


def program_forward_backward(prog, x, params, dy=None):
    arr = prog.stages_c()
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
