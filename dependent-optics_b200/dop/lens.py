"""Lens composition for device tensor lenses.

`compose(g, f)` is g after f, as in the crate (src/dlens.rs:74-113; README:
"compose(g, f) always means g . f: f is applied first"): the composite's get
is get_g . get_f, its put is put_f(x, put_g(get_f x, z')), and its residual is
the pair of the parts' residuals.  Composition happens in libdop
(dop_compose); a composite owns only the intermediate activation buffers.
"""
from __future__ import annotations

import ctypes as C

from ._lib import check, lib, ptr, stream_ptr


class Lens:
    """A device lens handle (dop_lens)."""

    def __init__(self, handle, keep=()):
        self._h = handle
        self._keep = keep  # parts and tensors the handle points into

    @staticmethod
    def of_block(block, params, dparams) -> "Lens":
        h = C.c_void_p()
        check(lib().dop_lens_from_block(block.handle, ptr(params), ptr(dparams), C.byref(h)))
        return Lens(h, (block, params, dparams))

    def forward(self, x, y=None, stream=None):
        import torch
        if y is None:
            y = torch.empty_like(x)
        check(lib().dop_lens_forward(self._h, ptr(x), ptr(y), stream_ptr(stream)))
        return y

    def backward(self, dy, dx=None, stream=None):
        import torch
        if dx is None:
            dx = torch.empty_like(dy)
        check(lib().dop_lens_backward(self._h, ptr(dy), ptr(dx), stream_ptr(stream)))
        return dx

    def close(self):
        if getattr(self, "_h", None):
            lib().dop_lens_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


def compose(g: Lens, f: Lens) -> Lens:
    """g after f."""
    h = C.c_void_p()
    check(lib().dop_compose(g._h, f._h, C.byref(h)))
    return Lens(h, (g, f))
