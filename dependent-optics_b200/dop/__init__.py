"""dop — B200 tensor lenses (Python host side of libdop).

Mirrors the dependent-optics crate's lens API: `mixtral` (config, layout,
the block lens), `kernel` (small programs), `lens.compose`, `ad` (exact
rational scalar lenses) and `vect` (GF(2) linear maps and their adjoints).
"""
from ._lib import DOP_BF16, DOP_F32, DopError, lib  # noqa: F401
from . import ad, kernel, lens, mixtral, vect  # noqa: F401
from .lens import compose  # noqa: F401
from .mixtral import Block, MixtralConfig, layout, parameter_count  # noqa: F401
