"""ctypes binding of libdop.so (include/dop.h).

The library is built in-tree by dependent-optics_b200/build.py.  Loading it
never falls back to anything: if the shared object is missing the import of
the compute entry points raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
LIB_PATH = PKG / "libdop.so"

DOP_F32 = 0
DOP_BF16 = 1
DOP_STAGE_GEMM = 0
DOP_STAGE_ATTENTION = 1
DOP_STAGE_ADD = 2
DOP_IPC_HANDLE_BYTES = 64
DOP_SELFTEST_MBARRIER_CODE = 90

ERRORS = {
    -1: "DOP_E_INVALID", -2: "DOP_E_CUDA", -3: "DOP_E_NOMEM", -4: "DOP_E_UNSUPPORTED",
    -5: "DOP_E_STATE", -6: "DOP_E_NCCL", -7: "DOP_E_TIMEOUT",
    -20: "DOP_E_NO_DEVICE", -21: "DOP_E_PARAMS_EXCEED_CLUSTER",
    -22: "DOP_E_TAPE_EXCEEDS_CLUSTER", -23: "DOP_E_TILE_EXCEEDS_DEVICES",
    -24: "DOP_E_CODE_EXCEEDS_DEVICES", -25: "DOP_E_ROUTE_UNAVAILABLE",
}


class DopError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class MixtralCfg(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "vocab", "dim", "layers", "heads", "kv_heads", "head_dim", "intermediate",
        "experts", "top_k")] + [("rms_eps", C.c_float), ("rope_theta", C.c_float),
                                ("sliding_window", C.c_int64)]


class LayerLayout(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "attn_norm", "q", "k", "v", "o", "ffn_norm", "router", "gate0", "up0", "down0",
        "expert_stride", "total")]


class StageC(C.Structure):
    _fields_ = [("kind", C.c_int32), ("relu", C.c_int32)] + [(n, C.c_int64) for n in (
        "batch", "din", "dout", "save_at", "mask_at", "param_at", "tokens", "dim", "x_at",
        "probs_at", "from_", "len")]


class Qc(C.Structure):
    _fields_ = [("n", C.c_int64), ("d", C.c_int64)]


class ExprNode(C.Structure):
    _fields_ = [("kind", C.c_int32), ("pad_", C.c_int32)] + [
        (n, C.c_int64) for n in ("a", "b", "c", "d", "var")] + [("q", Qc)]


class LinC(C.Structure):
    _fields_ = [("dom", C.c_uint32), ("cod", C.c_uint32), ("columns", C.c_uint32 * 32)]


# (name, restype, argtypes) of every symbol include/dop.h declares.
_P = C.c_void_p
_I64 = C.c_int64
SIGNATURES = [
    ("dop_last_error", C.c_char_p, []),
    ("dop_version", C.c_char_p, []),
    ("dop_layer_layout_of", C.c_int, [C.POINTER(MixtralCfg), C.POINTER(LayerLayout)]),
    ("dop_parameter_count", _I64, [C.POINTER(MixtralCfg)]),
    ("dop_block_create", C.c_int, [C.POINTER(MixtralCfg), _I64, _I64, C.c_int, C.POINTER(_P)]),
    ("dop_block_destroy", C.c_int, [_P]),
    ("dop_block_set_router_bias", C.c_int, [_P, _P]),
    ("dop_block_forward", C.c_int, [_P, _P, _P, _P, _P]),
    ("dop_block_backward", C.c_int, [_P, _P, _P, _P, _P, _P]),
    ("dop_block_workspace_bytes", _I64, [_P]),
    ("dop_block_routing", C.c_int, [_P, _P, _P, _P, _P, _P]),
    ("dop_block_permutation", C.c_int, [_P, _P, _P, _P, _P]),
    ("dop_block_ffn_input", C.c_int, [_P, _P, _P]),
    ("dop_block_permuted_rows", _I64, [_P]),
    ("dop_block_launches", _I64, [_P]),
    ("dop_block_create_ep", C.c_int, [C.POINTER(MixtralCfg), _I64, _I64, C.c_int, C.c_int,
                                      C.c_int, C.POINTER(_P)]),
    ("dop_block_ep_handle", C.c_int, [_P, _P]),
    ("dop_block_ep_connect", C.c_int, [_P, _P]),
    ("dop_block_set_adjoint_stream", C.c_int, [_P, _P]),
    ("dop_block_set_timing", C.c_int, [_P, C.c_int]),
    ("dop_block_phase_count", C.c_int, [_P]),
    ("dop_block_phase", C.c_int, [_P, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_float)]),
    ("dop_model_create", C.c_int, [C.POINTER(MixtralCfg), _I64, _I64, C.c_int, C.POINTER(_P)]),
    ("dop_model_destroy", C.c_int, [_P]),
    ("dop_model_forward_backward", C.c_int, [_P, _P, _P, _P, _P, _P, _P, _P]),
    ("dop_model_parameter_count", _I64, [_P]),
    ("dop_lens_from_block", C.c_int, [_P, _P, _P, C.POINTER(_P)]),
    ("dop_compose", C.c_int, [_P, _P, C.POINTER(_P)]),
    ("dop_lens_forward", C.c_int, [_P, _P, _P, _P]),
    ("dop_lens_backward", C.c_int, [_P, _P, _P, _P]),
    ("dop_lens_destroy", C.c_int, [_P]),
    ("dop_program_create", C.c_int, [C.POINTER(StageC), _I64, _I64, _I64, _I64, _I64, _I64,
                                     C.POINTER(_P)]),
    ("dop_program_destroy", C.c_int, [_P]),
    ("dop_program_launches", _I64, [_P]),
    ("dop_program_forward", C.c_int, [_P, _P, _P, _P, _P]),
    ("dop_program_backward", C.c_int, [_P, _P, _P, _P, _P, _P]),
    ("dop_program_forward_backward", C.c_int, [_P, _P, _P, _P, _P, _P, _P, _P]),
    ("dop_mse_loss_grad", C.c_int, [_P, _P, _I64, _P, _P, _P]),
    ("dop_gemm_bf16", C.c_int, [_I64, _I64, _I64, _P, _I64, C.c_int, _P, _I64, C.c_int, _P,
                                _I64, C.c_int, C.c_int, _P]),
    ("dop_device_status", C.c_int, []),
    ("dop_clear_device_status", C.c_int, []),
    ("dop_set_wait_limits", C.c_int, [_I64, _I64]),
    ("dop_selftest_wait_expiry", C.c_int, [C.c_int, _P]),
    ("dop_exp2_poly", C.c_int, [_P, _P, C.c_int64, _P]),
    ("dop_gqa_forward", C.c_int, [_I64, _I64, _I64, _I64, _I64, _I64, C.c_int, _P, _P, _P, _P,
                                  _P, _P]),
    ("dop_gqa_backward", C.c_int, [_I64, _I64, _I64, _I64, _I64, _I64, C.c_int, _P, _P, _P, _P,
                                   _P, _P, _P, _P, _P, _P, _P]),
    ("dop_gqa_backward_f32_noalloc", C.c_int, [_I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P,
                                               _P, _P, _P, _P, _P, _P, _P]),
    ("dop_f32_to_bf16", C.c_int, [_P, _P, _I64, _P]),
    ("dop_sgd_step", C.c_int, [_P, _P, _I64, C.c_float, _P]),
    ("dop_derive_links", C.c_int, [_P, _I64, _P, _I64, C.POINTER(_I64)]),
    ("dop_route_message", C.c_int, [_P, _I64, _P, _I64, C.c_int32, C.c_int32, _I64, _P, _I64,
                                    C.POINTER(_I64)]),
    ("dop_stage_mixtral", C.c_int, [C.POINTER(MixtralCfg), _I64, _I64, _I64, C.c_int, _P, _I64,
                                    _P, _I64, C.POINTER(_P)]),
    ("dop_plan_destroy", C.c_int, [_P]),
    ("dop_plan_home_count", _I64, [_P]),
    ("dop_plan_window_count", _I64, [_P]),
    ("dop_plan_hop_count", _I64, [_P]),
    ("dop_plan_home", C.c_int, [_P, _I64, _P]),
    ("dop_plan_window", C.c_int, [_P, _I64, _P]),
    ("dop_plan_window_hop", C.c_int, [_P, _I64, C.c_int, _I64, C.POINTER(_I64)]),
    ("dop_plan_hop", C.c_int, [_P, _I64, _P]),
    ("dop_plan_check", C.c_int, [_P, _P, _I64, _I64]),
    ("dop_plan_trace", C.c_int, [_P, C.c_char_p, _I64, C.POINTER(_I64)]),
    ("dop_run_window", C.c_int, [_P, _P, _P, _P, _P, _P, _P]),
    ("dop_ad_forward", C.c_int, [C.POINTER(ExprNode), _I64, _I64, C.POINTER(Qc), _I64,
                                 C.POINTER(Qc), C.POINTER(_P)]),
    ("dop_ad_backward", C.c_int, [C.POINTER(ExprNode), _I64, _I64, _P, Qc, _I64,
                                  C.POINTER(Qc)]),
    ("dop_ad_stored_scalars", C.c_int, [_P, C.POINTER(Qc), _I64, C.POINTER(_I64)]),
    ("dop_ad_tape_destroy", C.c_int, [_P]),
    ("dop_lin_apply", C.c_uint32, [C.POINTER(LinC), C.c_uint32]),
    ("dop_lin_zero", C.c_int, [C.c_uint32, C.c_uint32, C.POINTER(LinC)]),
    ("dop_lin_identity", C.c_int, [C.c_uint32, C.POINTER(LinC)]),
    ("dop_lin_compose", C.c_int, [C.POINTER(LinC), C.POINTER(LinC), C.POINTER(LinC)]),
    ("dop_lin_add", C.c_int, [C.POINTER(LinC), C.POINTER(LinC), C.POINTER(LinC)]),
    ("dop_lin_transpose", C.c_int, [C.POINTER(LinC), C.POINTER(LinC)]),
    ("dop_lin_kronecker", C.c_int, [C.POINTER(LinC), C.POINTER(LinC), C.POINTER(LinC)]),
    ("dop_lin_all", C.c_int, [C.c_uint32, C.c_uint32, C.POINTER(LinC), _I64,
                              C.POINTER(_I64)]),
]

_lib = None


def lib() -> C.CDLL:
    """Load libdop.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OSError(f"{LIB_PATH} is missing: run dependent-optics_b200/build.py")
        L = C.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != 0:
        raise DopError(status, lib().dop_last_error().decode())


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None passes NULL)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream) -> int | None:
    return None if stream is None else stream.cuda_stream
