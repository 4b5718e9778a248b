"""The C ABI: libdop.so loads, exports every entry point include/dop.h
declares, and rejects bad arguments with a status code (no GPU needed)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from dop import _lib
from dop.mixtral import MixtralConfig

ROOT = Path(__file__).resolve().parent.parent


def declared():
    text = (ROOT / "include" / "dop.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dop_\w+)\s*\(", text)))


def test_header_symbols_exported_and_bound():
    L = _lib.lib()
    names = declared()
    assert len(names) >= 27
    for n in names:
        assert hasattr(L, n), f"libdop.so does not export {n}"
    bound = {s[0] for s in _lib.SIGNATURES}
    assert set(names) == bound


def test_layout_matches_python():
    from dop.mixtral import layer_layout, layout
    for cfg in (MixtralConfig.demo(), MixtralConfig.mixtral_8x7b()):
        ll = layer_layout(cfg)
        lay = layout(cfg)
        L0 = lay.layers[0]
        base = L0.attn_norm
        assert (ll.q, ll.k, ll.v, ll.o, ll.ffn_norm, ll.router) == tuple(
            getattr(L0, n) - base for n in ("q", "k", "v", "o", "ffn_norm", "router"))
        assert ll.gate0 == L0.gate[0] - base and ll.up0 == L0.up[0] - base
        assert ll.down0 == L0.down[0] - base
        assert ll.expert_stride == L0.gate[1] - L0.gate[0]
        assert ll.total == (lay.final_norm - lay.layers[0].attn_norm) // cfg.layers
        assert _lib.lib().dop_parameter_count(C.byref(cfg.to_c())) == lay.total


@pytest.mark.parametrize("bad", [{"kv_heads": 3}, {"head_dim": 7}, {"top_k": 5}, {"experts": 0},
                                 {"sliding_window": 0}])
def test_block_create_rejects_bad_config(bad):
    cfg = MixtralConfig.demo()
    for k, v in bad.items():
        setattr(cfg, k, v)
    h = C.c_void_p()
    st = _lib.lib().dop_block_create(C.byref(cfg.to_c()), 2, 8, _lib.DOP_F32, C.byref(h))
    assert st == -1
    assert _lib.lib().dop_last_error().decode().startswith("invalid argument")


def test_null_handle_errors():
    L = _lib.lib()
    assert L.dop_block_forward(None, None, None, None, None) == -1
    assert L.dop_block_launches(None) == -1
    assert L.dop_lens_forward(None, None, None, None) == -1


def test_program_create_rejects_bad_stage():
    from dop.kernel import Program
    prog = Program.mlp(2, [3, 4, 2])
    arr = prog.stages_c()
    arr[0].save_at = 10_000  # saves past the tape
    h = C.c_void_p()
    st = _lib.lib().dop_program_create(arr, len(prog.stages), prog.input_len, prog.output_len,
                                       prog.param_len, prog.tape_f32, prog.tape_u8, C.byref(h))
    assert st == -1
