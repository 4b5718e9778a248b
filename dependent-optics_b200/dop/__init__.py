"""dop — B200 tensor lenses (Python host side of libdop).

Mirrors the dependent-optics crate's tensor-lens API: `mixtral` (config,
layout, the block lens), `kernel` (small programs), `lens.compose`.
"""
from ._lib import DOP_BF16, DOP_F32, DopError, lib  # noqa: F401
from . import kernel, lens, mixtral  # noqa: F401
from .lens import compose  # noqa: F401
from .mixtral import Block, MixtralConfig, layout, parameter_count  # noqa: F401
